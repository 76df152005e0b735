"""Generates tests/golden/transformer_b64_fixture.npz: logits of the benchmark
decoder (8 layers, d_model 1024, 16 heads, FFN 4096, vocab 32000, 512 tokens)
for sequences 0, 21, 42 and 63 of the 64-sequence token batch, computed by
PyTorch on the CPU in float32.

The reference computes its transformer through libtorch (tch 0.22 with
LibTorch 2.9; rust/deps/ferrite-torch/Cargo.toml:11), outside the reference
tree. This script runs the reference block op for op through the same
library's CPU kernels (PyTorch's ATen), in float32 as the demo does:
  transformer_block  transformer_demo.rs:48-70
      normed = x.layer_norm([d], ones, zeros, 1e-5); x = x + attention(normed)
      normed = x.layer_norm([d], ones, zeros, 1e-5); x = x + ffn(normed)
  attention          transformer_demo.rs:18-42
      q, k, v = x.matmul(wq), x.matmul(wk), x.matmul(wv), viewed
      [batch, seq, heads, 64] and permuted to [batch, heads, seq, 64];
      scores = q.matmul(k^T) / sqrt(64); softmax(-1, Float); matmul(v);
      permuted back, contiguous, viewed [batch, seq, d]; matmul(wo)
  ffn                transformer_demo.rs:44-46
      x.matmul(w1).gelu("none").matmul(w2)
with the benchmark configuration's additions: token embedding (row lookup of
the bf16 embedding), a causal mask on the scores (masked_fill with -inf
before the softmax), a final layer norm and the LM head. The weights are the
device model's own: the bf16 buffer of fercuda_b200.synth.normal_bf16(4, n,
0, 0.02) in the layout of include/fercuda/b200/ext.h (Wq, Wk, Wv are the
column thirds of the fused Wqkv), upcast to float32; activations stay
float32 throughout (no bf16 rounding anywhere).

Stored (compact; the test recomputes the same digests from the GPU logits):
  tokens     int32 [4, 512]        the sequences' token ids (seed 5)
  row_max    f32 [4, 512]          max logit per position
  row_top2   f32 [4, 512]          second largest logit per position
  row_argmax int32 [4, 512]
  row_lse    f32 [4, 512]          log-sum-exp per position
  proj       f32 [4, 512, 8]       logits . r_j / sqrt(V), r_j = +-1 from
                                   splitmix64 seed 6 (projection_signs)
  rows       f32 [4, 32000]        full logits at (seq, pos) of rows_at
  rows_at    int32 [4, 2]
  weights_sha256                   of the little-endian bf16 weight buffer

Run from the repository root:  python tests/golden/gen_transformer_fixture.py
"""
from __future__ import annotations

import hashlib
import json
import math
import os
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from fercuda_b200 import synth  # noqa: E402

OUT = Path(__file__).resolve().parent / "transformer_b64_fixture.npz"
SEQS = (0, 21, 42, 63)
ROWS_AT = ((0, 511), (21, 0), (42, 255), (63, 300))   # (sequence, position)
N_PROJ = 8
PROJ_SEED = 6


def up128(n: int) -> int:
    return (n + 127) & ~127


def layout(L: int, d: int, F: int, V: int) -> dict:
    """Element offsets of each tensor in the weight buffer."""
    off = 0
    o = {"emb": 0}
    off = up128(V * d)
    o["qkv"], o["o"], o["w1"], o["w2"] = [], [], [], []
    for _ in range(L):
        o["qkv"].append(off)
        off = up128(off + 3 * d * d)
        o["o"].append(off)
        off = up128(off + d * d)
        o["w1"].append(off)
        off = up128(off + d * F)
        o["w2"].append(off)
        off = up128(off + F * d)
    o["lm"] = off
    o["total"] = up128(off + d * V)
    return o


def batch_tokens(B: int, S: int, V: int, seed: int) -> np.ndarray:
    u = synth.uniform01(seed, B * S)
    return np.minimum((u * V).astype(np.int32), V - 1).reshape(B, S)


def projection_signs(V: int, n: int = N_PROJ, seed: int = PROJ_SEED) -> np.ndarray:
    """[n, V] of +-1 (bit 63 of the splitmix64 draws of `seed`)."""
    bits = (synth.splitmix64(seed, n * V) >> np.uint64(63)).astype(np.float64)
    return (1.0 - 2.0 * bits).reshape(n, V)


def digests(logits: np.ndarray, signs: np.ndarray) -> dict:
    """Per-position digests of f32 logits [B, S, V], computed in float64."""
    z = logits.astype(np.float64)
    top = np.partition(z, -2, axis=-1)
    mx = z.max(axis=-1)
    lse = mx + np.log(np.exp(z - mx[..., None]).sum(axis=-1))
    return {
        "row_max": mx.astype(np.float32),
        "row_top2": top[..., -2].astype(np.float32),
        "row_argmax": z.argmax(axis=-1).astype(np.int32),
        "row_lse": lse.astype(np.float32),
        "proj": (z @ signs.T / math.sqrt(z.shape[-1])).astype(np.float32),
    }


def torch_forward(tokens: np.ndarray, wbits: np.ndarray, L: int, d: int, H: int, F: int, V: int,
                  eps: float = 1e-5) -> np.ndarray:
    import torch

    torch.set_num_threads(os.cpu_count() or 1)
    o = layout(L, d, F, V)
    w = torch.from_numpy(synth.bf16_bits_to_f32(wbits))

    def mat(off: int, r: int, c: int):
        return w[off:off + r * c].view(r, c)

    B, S = tokens.shape
    hd = d // H
    ones, zeros = torch.ones(d), torch.zeros(d)
    causal = torch.triu(torch.ones(S, S, dtype=torch.bool), diagonal=1)
    with torch.no_grad():
        x = mat(o["emb"], V, d)[torch.from_numpy(tokens.astype(np.int64))]          # [B, S, d]
        for li in range(L):
            wqkv = mat(o["qkv"][li], d, 3 * d)
            wq, wk, wv = wqkv[:, :d], wqkv[:, d:2 * d], wqkv[:, 2 * d:]
            normed = torch.nn.functional.layer_norm(x, [d], ones, zeros, eps)
            q = normed.matmul(wq).view(B, S, H, hd).permute(0, 2, 1, 3)
            k = normed.matmul(wk).view(B, S, H, hd).permute(0, 2, 1, 3)
            v = normed.matmul(wv).view(B, S, H, hd).permute(0, 2, 1, 3)
            scores = q.matmul(k.transpose(-2, -1)) / math.sqrt(hd)
            scores = scores.masked_fill(causal, float("-inf"))
            probs = scores.softmax(-1, dtype=torch.float32)
            att = probs.matmul(v).permute(0, 2, 1, 3).contiguous().view(B, S, d)
            x = x + att.matmul(mat(o["o"][li], d, d))
            normed = torch.nn.functional.layer_norm(x, [d], ones, zeros, eps)
            ff = torch.nn.functional.gelu(normed.matmul(mat(o["w1"][li], d, F)), approximate="none")
            x = x + ff.matmul(mat(o["w2"][li], F, d))
        normed = torch.nn.functional.layer_norm(x, [d], ones, zeros, eps)
        return normed.matmul(mat(o["lm"], d, V)).numpy()


def main() -> None:
    c = synth.TRANSFORMER
    L, d, H, F, V, S, B = c["layers"], c["d_model"], c["heads"], c["ffn"], c["vocab"], c["seq"], c["batch"]
    t0 = time.time()
    total = layout(L, d, F, V)["total"]
    wbits = synth.normal_bf16(c["weight_seed"], total, 0.0, 0.02)
    sha = hashlib.sha256(wbits.astype("<u2").tobytes()).hexdigest()
    toks = batch_tokens(B, S, V, c["token_seed"])[list(SEQS)]
    print(f"weights {total} bf16 in {time.time() - t0:.1f} s, sha256 {sha}")
    t0 = time.time()
    logits = torch_forward(toks, wbits, L, d, H, F, V, c["eps"])
    print(f"forward of {len(SEQS)} x {S} tokens in {time.time() - t0:.1f} s")
    dg = digests(logits, projection_signs(V))
    rows_at = np.array(ROWS_AT, np.int32)
    rows = np.stack([logits[SEQS.index(b), p] for b, p in ROWS_AT]).astype(np.float32)
    meta = dict(c, seqs=list(SEQS), weight_std=0.02, projection_seed=PROJ_SEED, n_proj=N_PROJ,
                generator="tests/golden/gen_transformer_fixture.py", torch_dtype="float32")
    import torch

    meta["torch_version"] = torch.__version__
    np.savez_compressed(OUT, tokens=toks, rows=rows, rows_at=rows_at, weights_sha256=np.array(sha),
                        meta=np.array(json.dumps(meta, sort_keys=True)), **dg)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes); max |logit| {np.abs(logits).max():.4f}")


if __name__ == "__main__":
    main()
