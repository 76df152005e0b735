"""Decoder-only transformer forward (fer_transformer_forward) against the
libtorch-CPU fixture of the benchmark model (tests/golden/, the reference's
block op for op in float32) and against the numpy oracle
(oracle/transformer_ref.py, which rounds to bf16 at the same points as the
GPU path), plus the properties batch sharding relies on:
sequences are independent, so any split of the batch gives bit-identical
logits, and runs are bit-identical.

Tolerance: the required bound for transformer logits is max relative error
<= 2e-2 (normalised by max |reference|); the tests also hold 5e-3 on the
2-layer model and 1e-2 on the 8-layer benchmark model, where rounding
differences (online vs two-pass softmax, f32 vs f64 layer-norm statistics)
compound over the layers."""
import importlib.util
from pathlib import Path

import numpy as np
import pytest

from fercuda_b200 import capi, synth
from tests import fixture_check

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
_spec = importlib.util.spec_from_file_location("transformer_ref", ROOT / "oracle" / "transformer_ref.py")
ref = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(ref)

REQUIRED_TOL = 2e-2
TIGHT = 5e-3
TIGHT_DEEP = 1e-2


def tokens_for(B, S, vocab, seed=5):
    u = synth.uniform01(seed, B * S)
    return np.minimum((u * vocab).astype(np.int32), vocab - 1).reshape(B, S)


def run(session, model, toks, vocab):
    import torch

    B, S = toks.shape
    t = torch.from_numpy(toks).cuda()
    logits = torch.empty((B, S, vocab), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    bt = session.import_ptr(capi.FER_DTYPE_I32, [B, S], t.data_ptr())
    bl = session.import_ptr(capi.FER_DTYPE_F32, [B, S, vocab], logits.data_ptr())
    session.wait(model.forward(bt, bl))
    session.free(bt)
    session.free(bl)
    assert session.device_errors() == 0
    return logits


def weights(session, model, n_elems):
    w = np.empty(n_elems, np.uint16)
    session.download(model.weight_buffer(), w)
    return w


def rel(y, r):
    return float(np.abs(y.astype(np.float64) - r).max() / np.abs(r).max())


SMALL = dict(layers=2, d_model=256, heads=4, ffn=512, vocab=1000)


def test_small_model_vs_oracle_and_batch_split(session):
    c = SMALL
    B, S = 3, 192
    m = capi.Transformer(session, c["layers"], c["d_model"], c["heads"], c["ffn"], c["vocab"], B * S)
    m.init_weights(4, 0.02)
    toks = tokens_for(B, S, c["vocab"])
    y = run(session, m, toks, c["vocab"]).cpu().numpy()
    w = weights(session, m, ref.weight_offsets(c["layers"], c["d_model"], c["ffn"], c["vocab"])["total"])
    r = ref.forward(toks, w, c["layers"], c["d_model"], c["heads"], c["ffn"], c["vocab"])
    err = rel(y, r)
    assert err <= REQUIRED_TOL
    assert err <= TIGHT, err
    # each sequence alone gives the same bits as inside the batch
    for b in range(B):
        yb = run(session, m, toks[b:b + 1], c["vocab"]).cpu().numpy()
        assert np.array_equal(yb[0].view(np.uint32), y[b].view(np.uint32))
    # run to run
    y2 = run(session, m, toks, c["vocab"]).cpu().numpy()
    assert np.array_equal(y2.view(np.uint32), y.view(np.uint32))
    m.close()


def test_odd_sequence_length(session):
    c = SMALL
    B, S = 2, 77       # partial query and key blocks
    m = capi.Transformer(session, c["layers"], c["d_model"], c["heads"], c["ffn"], c["vocab"], B * S)
    toks = tokens_for(B, S, c["vocab"], seed=9)
    y = run(session, m, toks, c["vocab"]).cpu().numpy()
    w = weights(session, m, ref.weight_offsets(c["layers"], c["d_model"], c["ffn"], c["vocab"])["total"])
    r = ref.forward(toks, w, c["layers"], c["d_model"], c["heads"], c["ffn"], c["vocab"])
    assert rel(y, r) <= TIGHT
    m.close()


def test_full_size_model_sequences_vs_oracle():
    """The benchmark model (8 layers, d 1024, 16 heads, ffn 4096, vocab 32000)
    on 8 sequences of 512 tokens: sequences 0 and 7 against the oracle."""
    cfg = synth.TRANSFORMER
    L, d, h, F, V, S = cfg["layers"], cfg["d_model"], cfg["heads"], cfg["ffn"], cfg["vocab"], cfg["seq"]
    B = 8
    with capi.Session(0, pool_bytes=4 << 30) as s:
        m = capi.Transformer(s, L, d, h, F, V, B * S)
        m.init_weights(cfg["weight_seed"], 0.02)
        toks = tokens_for(B, S, V, cfg["token_seed"])
        y = run(s, m, toks, V).cpu().numpy()
        assert np.isfinite(y).all()
        w = weights(s, m, ref.weight_offsets(L, d, F, V)["total"])
        for b in (0, 7):
            r = ref.forward(toks[b:b + 1], w, L, d, h, F, V)
            err = rel(y[b:b + 1], r)
            assert err <= REQUIRED_TOL
            assert err <= TIGHT_DEEP, (b, err)
        m.close()


def test_config_errors(session):
    with pytest.raises(capi.FerError) as e:
        capi.Transformer(session, 2, 256, 8, 512, 1000, 64)     # head_dim 32
    assert e.value.code == capi.FER_STATUS_INVALID_ARGUMENT
    m = capi.Transformer(session, 1, 256, 4, 512, 1000, 64)
    toks = tokens_for(1, 128, 1000)
    with pytest.raises(capi.FerError):
        run(session, m, toks, 1000)                              # 128 tokens > max_tokens 64
    m.close()


def test_graph_replay_is_bit_identical_to_eager(session):
    """The forward is issued eagerly the first time a (tokens, logits, batch,
    seq) signature is seen, captured into a CUDA graph the second time and
    replayed after that: all three give the same bits, and a replay after the
    tokens change follows the new tokens."""
    L, d, h, F, V, B, S = 2, 256, 4, 512, 512, 2, 128
    m = capi.Transformer(session, L, d, h, F, V, B * S)
    m.init_weights(7, 0.02)
    toks = tokens_for(B, S, V, 11)
    bt = session.alloc(capi.FER_DTYPE_I32, [B, S])
    bl = session.alloc(capi.FER_DTYPE_F32, [B, S, V])
    session.upload(bt, toks)
    outs = []
    for _ in range(3):
        session.wait(m.forward(bt, bl))
        y = np.empty((B, S, V), np.float32)
        session.download(bl, y)
        outs.append(y)
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))
    assert np.array_equal(outs[0].view(np.uint32), outs[2].view(np.uint32))
    toks2 = tokens_for(B, S, V, 12)
    session.upload(bt, toks2)
    session.wait(m.forward(bt, bl))
    y2 = np.empty((B, S, V), np.float32)
    session.download(bl, y2)
    ref2 = run(session, m, toks2, V).cpu().numpy()   # other buffers: an eager forward
    assert np.array_equal(y2.view(np.uint32), ref2.view(np.uint32))
    assert session.device_errors() == 0
    session.free(bt)
    session.free(bl)
    m.close()


def test_forward_host_matches_forward_and_download(session):
    """fer_transformer_forward_host (host tokens in, host logits out, the D2H
    copy of chunk i overlapped with chunk i+1's forward) gives the bits of
    fer_transformer_forward on the whole batch followed by a download: for
    the default chunking, one sequence per chunk, ragged chunks (2, 2, 1),
    repeated calls (eager, captured, replayed signatures), pageable and pinned
    host memory. Bad arguments are refused."""
    import torch

    L, d, h, F, V, B, S = 2, 256, 4, 512, 1000, 5, 128
    m = capi.Transformer(session, L, d, h, F, V, B * S)
    m.init_weights(9, 0.02)
    toks = tokens_for(B, S, V, 21)
    want = run(session, m, toks, V).cpu().numpy().view(np.uint32)
    pinned = torch.empty(B * S * V, dtype=torch.float32).pin_memory().numpy()
    for chunk in (0, 1, 2, 3, 5, 2, 2):
        for out in (np.full((B, S, V), np.nan, np.float32), pinned):
            out.fill(np.nan)
            m.forward_host(toks, out, chunk)
            assert np.array_equal(out.reshape(B, S, V).view(np.uint32), want), chunk
    # other tokens through the same (replayed) signatures follow the new tokens
    toks2 = tokens_for(B, S, V, 22)
    m.forward_host(toks2, pinned, 2)
    want2 = run(session, m, toks2, V).cpu().numpy().view(np.uint32)
    assert np.array_equal(pinned.reshape(B, S, V).view(np.uint32), want2)
    with pytest.raises(capi.FerError) as e:
        m.forward_host(toks, pinned, 6)                  # 6 x 128 > max_tokens 640
    assert e.value.code == capi.FER_STATUS_INVALID_ARGUMENT
    with pytest.raises(ValueError):
        m.forward_host(toks, np.empty(7, np.float32))
    with pytest.raises(ValueError):
        m.forward_host(toks.astype(np.int64), pinned)
    assert session.device_errors() == 0
    m.close()


def test_forward_bit_identical_over_ten_runs(session):
    """Ten forwards of the same tokens (the first eager, the second captured,
    the rest replayed, with 8-layer benchmark widths at a short sequence) give
    the same logits bit for bit."""
    L, d, h, F, V, B, S = 8, 1024, 16, 4096, 32000, 2, 128
    m = capi.Transformer(session, L, d, h, F, V, B * S)
    m.init_weights(4, 0.02)
    bt = session.alloc(capi.FER_DTYPE_I32, [B, S])
    bl = session.alloc(capi.FER_DTYPE_F32, [B, S, V])
    session.upload(bt, tokens_for(B, S, V, 5))
    first = None
    for _ in range(10):
        session.wait(m.forward(bt, bl))
        y = np.empty((B, S, V), np.float32)
        session.download(bl, y)
        if first is None:
            first = y
        else:
            assert np.array_equal(first.view(np.uint32), y.view(np.uint32))
    assert session.device_errors() == 0
    session.free(bt)
    session.free(bl)
    m.close()


def test_device_weight_fill_matches_host_generator(session):
    """The device fill (fer_fill_normal_bf16) gives the host generator's bits
    (synth.normal_bf16), element for element, at the transformer's and the
    GEMM benchmark's standard deviations."""
    import ctypes as C

    import torch

    for seed, std, n in ((4, 0.02, 5_000_003), (3, 1.0 / np.sqrt(8192), 1_048_577), (9, 1.0, 4099)):
        dev = torch.empty(n, dtype=torch.int16, device="cuda")
        rc = capi.kernels().fer_fill_normal_bf16(C.c_void_p(dev.data_ptr()), n, seed, C.c_float(std), None)
        assert rc == 0
        torch.cuda.synchronize()
        got = dev.cpu().numpy().view(np.uint16)
        want = synth.normal_bf16(seed, n, 0.0, std)
        assert np.array_equal(got, want), (seed, int((got != want).sum()))


def test_benchmark_batch_vs_libtorch_fixture():
    """The benchmark forward at its full size (B = 64 sequences of 512 tokens,
    8 layers, d 1024, 16 heads, FFN 4096, vocab 32000) against logits that
    PyTorch computed on the CPU in float32 for sequences 0, 21, 42 and 63
    (tests/golden/transformer_b64_fixture.npz). The device weights are the
    fixture's (same sha256); every digest holds the 2e-2 logits tolerance."""
    import hashlib

    cfg = synth.TRANSFORMER
    L, d, h, F, V, S, B = cfg["layers"], cfg["d_model"], cfg["heads"], cfg["ffn"], cfg["vocab"], cfg["seq"], cfg["batch"]
    fx = fixture_check.load()
    seqs = fx["meta"]["seqs"]
    with capi.Session(0, pool_bytes=6 << 30) as s:
        m = capi.Transformer(s, L, d, h, F, V, B * S)
        m.init_weights(cfg["weight_seed"], 0.02)
        w = weights(s, m, m.weight_elements())
        assert hashlib.sha256(w.astype("<u2").tobytes()).hexdigest() == fx["weights_sha256"]
        toks = tokens_for(B, S, V, cfg["token_seed"])
        assert np.array_equal(toks[seqs], fx["tokens"])
        y = run(s, m, toks, V)
        mine = y[seqs].cpu().numpy()
        del y
        assert np.isfinite(mine).all()
        e = fixture_check.check(fx, mine, REQUIRED_TOL)
        assert e["rows"] <= TIGHT_DEEP, e
        print("vs libtorch fixture:", e)
        m.close()
