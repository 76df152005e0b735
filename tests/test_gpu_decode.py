"""Incremental decoding over a KV cache (fer_transformer_prefill / _decode).

Decoding token n after a prompt of n tokens must give the logits the full
forward gives at position n: the same weights and blocks, only the attention
of the new query runs through the cache kernel (f32 probabilities, split
over 256-position chunks) instead of the prompt kernel (bf16 probabilities).
Checks:
  - prefill logits equal the forward's bit for bit (all positions, and the
    last-position-only form);
  - each of several decode steps matches the forward at that position within
    DECODE_TOL, and the numpy oracle within the transformer bound 2e-2;
  - chunk boundaries (256, 257 and 601 keys) and a 600-token prompt;
  - repeated decodes from the same prefill are bit-identical;
  - the decode attention kernel against a torch reference on random caches;
  - refused requests (decode before prefill, wrong batch, full cache).

DECODE_TOL = 1e-2 of max |forward logits|: the two attention kernels round
probabilities differently (bf16 vs f32), and the difference passes through
the remaining layers.
"""
import ctypes as C
import importlib.util
from pathlib import Path

import numpy as np
import pytest
import torch

from fercuda_b200 import capi, synth

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
_spec = importlib.util.spec_from_file_location("transformer_ref", ROOT / "oracle" / "transformer_ref.py")
ref = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(ref)

DECODE_TOL = 1e-2
REQUIRED_TOL = 2e-2
SMALL = dict(layers=2, d=256, heads=4, ffn=512, vocab=512)


def tokens_for(B, S, vocab, seed=5):
    u = synth.uniform01(seed, B * S)
    return np.minimum((u * vocab).astype(np.int32), vocab - 1).reshape(B, S)


def rel(y, r):
    y, r = np.asarray(y, np.float64), np.asarray(r, np.float64)
    return float(np.abs(y - r).max() / np.abs(r).max())


class Model:
    def __init__(self, session, max_tokens, **cfg):
        c = {**SMALL, **cfg}
        self.s, self.c = session, c
        self.m = capi.Transformer(session, c["layers"], c["d"], c["heads"], c["ffn"], c["vocab"], max_tokens)

    def _bufs(self, toks, shape):
        t = torch.from_numpy(np.ascontiguousarray(toks)).cuda()
        logits = torch.empty(shape, dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        bt = self.s.import_ptr(capi.FER_DTYPE_I32, list(toks.shape), t.data_ptr())
        bl = self.s.import_ptr(capi.FER_DTYPE_F32, list(shape), logits.data_ptr())
        return t, logits, bt, bl

    def forward(self, toks):
        B, S = toks.shape
        t, logits, bt, bl = self._bufs(toks, (B, S, self.c["vocab"]))
        self.s.wait(self.m.forward(bt, bl))
        self.s.free(bt), self.s.free(bl)
        return logits.cpu().numpy()

    def prefill(self, cache, toks, last_only=False):
        B, S = toks.shape
        shape = (B, self.c["vocab"]) if last_only else (B, S, self.c["vocab"])
        t, logits, bt, bl = self._bufs(toks, shape)
        self.s.wait(self.m.prefill(cache, bt, bl))
        self.s.free(bt), self.s.free(bl)
        return logits.cpu().numpy()

    def decode(self, cache, tok_col):
        t, logits, bt, bl = self._bufs(tok_col.astype(np.int32), (tok_col.shape[0], self.c["vocab"]))
        self.s.wait(self.m.decode(cache, bt, bl))
        self.s.free(bt), self.s.free(bl)
        return logits.cpu().numpy()


@pytest.fixture(scope="module")
def model(session):
    m = Model(session, max_tokens=4096)
    yield m
    m.m.close()


def test_prefill_equals_forward(model):
    toks = tokens_for(3, 128, model.c["vocab"], seed=11)
    cache = model.m.kv_create(4, 512)
    full = model.prefill(cache, toks)
    assert np.array_equal(full.view(np.uint32), model.forward(toks).view(np.uint32))
    last = model.prefill(cache, toks, last_only=True)
    assert np.array_equal(last.view(np.uint32), full[:, -1].view(np.uint32))
    assert model.m.kv_length(cache) == (3, 128)
    model.m.kv_destroy(cache)


@pytest.mark.parametrize("B,S0,steps", [(3, 64, 5), (2, 255, 3), (2, 600, 2)])
def test_decode_matches_forward_and_oracle(model, session, B, S0, steps):
    c = model.c
    toks = tokens_for(B, S0 + steps, c["vocab"], seed=12 + S0)
    cache = model.m.kv_create(B, S0 + steps)
    model.prefill(cache, toks[:, :S0], last_only=True)
    w = np.empty(model.m.weight_elements(), np.uint16)
    session.download(model.m.weight_buffer(), w)
    for k in range(steps):
        n = S0 + k
        got = model.decode(cache, toks[:, n])
        want = model.forward(toks[:, : n + 1])[:, -1]
        assert rel(got, want) <= DECODE_TOL, (n, rel(got, want))
        if k == steps - 1:
            oracle = ref.forward(toks[:, : n + 1], w, c["layers"], c["d"], c["heads"], c["ffn"], c["vocab"])[:, -1]
            assert rel(got, oracle) <= REQUIRED_TOL, rel(got, oracle)
    assert model.m.kv_length(cache) == (B, S0 + steps)
    assert session.device_errors() == 0
    model.m.kv_destroy(cache)


def test_decode_is_bit_identical_run_to_run(model):
    toks = tokens_for(2, 300, model.c["vocab"], seed=21)
    cache = model.m.kv_create(2, 300)
    outs = []
    for _ in range(2):
        model.prefill(cache, toks[:, :298], last_only=True)
        outs.append(np.stack([model.decode(cache, toks[:, 298]), model.decode(cache, toks[:, 299])]))
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))
    model.m.kv_destroy(cache)


def test_refused_requests(model, session):
    toks = tokens_for(2, 16, model.c["vocab"], seed=31)
    cache = model.m.kv_create(2, 17)
    with pytest.raises(capi.FerError):          # decode before any prefill
        model.decode(cache, toks[:, 0])
    model.prefill(cache, toks, last_only=True)
    with pytest.raises(capi.FerError):          # batch differs from the prefill
        model.decode(cache, np.zeros(3, np.int32))
    model.decode(cache, toks[:, 0])             # position 16, the last slot
    with pytest.raises(capi.FerError):          # cache full
        model.decode(cache, toks[:, 1])
    with pytest.raises(capi.FerError):          # prompt longer than the cache
        model.prefill(cache, tokens_for(2, 32, model.c["vocab"]))
    model.m.kv_destroy(cache)


@pytest.mark.parametrize("B,heads,n_keys", [(1, 1, 1), (2, 4, 256), (2, 4, 257), (3, 16, 1000), (1, 2, 4096)])
def test_decode_attention_kernel(B, heads, n_keys):
    """fer_attn_decode against float64 torch on random bf16 caches."""
    k = capi.kernels()
    k.fer_attn_decode.argtypes = [C.c_void_p] * 5 + [C.c_int] * 5 + [C.c_void_p, C.c_void_p]
    k.fer_attn_decode.restype = C.c_int
    k.fer_attn_decode_scratch_floats.argtypes = [C.c_int] * 3
    k.fer_attn_decode_scratch_floats.restype = C.c_size_t
    d, max_seq = heads * 64, n_keys + 7
    g = torch.Generator(device="cuda").manual_seed(40 + n_keys)
    qkv = torch.randn(B, 3 * d, generator=g, device="cuda").bfloat16()
    kc = torch.randn(B, heads, max_seq, 64, generator=g, device="cuda").bfloat16()
    vc = torch.randn(B, heads, max_seq, 64, generator=g, device="cuda").bfloat16()
    nf = k.fer_attn_decode_scratch_floats(B, heads, n_keys)
    scratch = torch.empty(max(nf, 1), device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    outs = []
    for _ in range(2):
        out = torch.full((B, d), float("nan"), device="cuda").bfloat16()
        assert k.fer_attn_decode(qkv.data_ptr(), kc.data_ptr(), vc.data_ptr(), out.data_ptr(),
                                 scratch.data_ptr() if nf else None, B, d, heads, max_seq, n_keys,
                                 err.data_ptr(), torch.cuda.current_stream().cuda_stream) == 0
        torch.cuda.synchronize()
        outs.append(out)
    assert torch.equal(outs[0].view(torch.int16), outs[1].view(torch.int16))
    assert int(err.item()) == 0
    q = qkv[:, :d].double().view(B, heads, 64)
    kk, vv = kc[:, :, :n_keys].double(), vc[:, :, :n_keys].double()
    p = torch.softmax(torch.einsum("bhi,bhji->bhj", q, kk) / 8.0, dim=-1)
    want = torch.einsum("bhj,bhji->bhi", p, vv).reshape(B, d)
    err = (outs[0].double() - want).abs().max() / want.abs().max()
    assert float(err) <= 1e-2, float(err)
