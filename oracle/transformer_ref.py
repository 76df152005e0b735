"""ORACLE - test infrastructure only. CPU (numpy) restatement of the
reference's transformer block, for checking fer_transformer_forward.

The reference computes its transformer through libtorch (tch 0.22 <->
LibTorch 2.9, rust/deps/ferrite-torch/Cargo.toml:11), a third-party dependency
not in the reference tree; its block is
rust/deps/ferrite-torch/examples/transformer_demo.rs:
  transformer_block :48-70   x + attn(LN1(x)), then x + ffn(LN2(x)), LN eps 1e-5
  attention         :18-42   q,k,v = x@Wq, x@Wk, x@Wv; softmax(q k^T / sqrt(dh)) v; @ Wo
  ffn               :44-46   gelu("none") (exact erf form) between x@W1 and @W2
restated here with the additions the benchmark configuration asks for: token
embedding, causal mask, final LN and LM head, fused Wqkv = [Wq | Wk | Wv].
To compare against the GPU path at tight tolerance the restatement rounds to
bf16 where the GPU path keeps bf16 activations (LN outputs, q/k/v, attention
output, GELU output, the probabilities fed to P.V); everything else is f32.
Parity is unpinned: no reference test holds transformer values (the demo only
prints summary statistics, transformer_demo.rs:148-166).
"""
from __future__ import annotations

import math

import numpy as np


def bf16_round(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, np.float32).view(np.uint32)
    r = ((u >> 16) & 1) + np.uint32(0x7FFF)
    with np.errstate(over="ignore"):
        return ((u + r) & np.uint32(0xFFFF0000)).view(np.float32)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


def up128(n: int) -> int:
    return (n + 127) & ~127


def weight_offsets(layers: int, d: int, ffn: int, vocab: int) -> dict:
    """Element offsets of each tensor in the weight buffer (the layout of
    include/fercuda/b200/ext.h)."""
    off = 0
    out = {"emb": off}
    off = up128(off + vocab * d)
    out["qkv"], out["o"], out["w1"], out["w2"] = [], [], [], []
    for _ in range(layers):
        out["qkv"].append(off)
        off = up128(off + d * 3 * d)
        out["o"].append(off)
        off = up128(off + d * d)
        out["w1"].append(off)
        off = up128(off + d * ffn)
        out["w2"].append(off)
        off = up128(off + ffn * d)
    out["lm"] = off
    out["total"] = up128(off + d * vocab)
    return out


def layer_norm(x: np.ndarray, eps: float) -> np.ndarray:
    mean = x.mean(axis=-1, keepdims=True, dtype=np.float64)
    var = ((x - mean) ** 2).mean(axis=-1, keepdims=True)
    return ((x - mean) / np.sqrt(var + eps)).astype(np.float32)


def gelu_erf(x: np.ndarray) -> np.ndarray:
    from scipy.special import erf

    return (0.5 * x * (1.0 + erf(x.astype(np.float64) / math.sqrt(2.0)))).astype(np.float32)


def forward(tokens: np.ndarray, wbits: np.ndarray, layers: int, d: int, heads: int, ffn: int, vocab: int,
            eps: float = 1e-5) -> np.ndarray:
    """tokens int [B, S]; wbits uint16 weight buffer; returns f32 logits [B, S, V]."""
    o = weight_offsets(layers, d, ffn, vocab)

    def mat(off, rows, cols):
        return bf16_bits_to_f32(wbits[off:off + rows * cols]).reshape(rows, cols)

    B, S = tokens.shape
    hd = d // heads
    emb = mat(o["emb"], vocab, d)
    x = emb[tokens.reshape(-1)].astype(np.float32)                     # [T, d]
    causal = np.triu(np.ones((S, S), bool), k=1)
    for l in range(layers):
        a = bf16_round(layer_norm(x, eps))
        qkv = bf16_round(a @ mat(o["qkv"][l], d, 3 * d))
        att = np.empty((B * S, d), np.float32)
        for b in range(B):
            rows = slice(b * S, (b + 1) * S)
            for h in range(heads):
                q = qkv[rows, h * hd:(h + 1) * hd]
                k = qkv[rows, d + h * hd:d + (h + 1) * hd]
                v = qkv[rows, 2 * d + h * hd:2 * d + (h + 1) * hd]
                s = (q @ k.T) / np.float32(math.sqrt(hd))
                s[causal] = -np.inf
                p = np.exp(s - s.max(axis=1, keepdims=True)).astype(np.float32)
                lsum = p.sum(axis=1, keepdims=True)
                att[rows, h * hd:(h + 1) * hd] = (bf16_round(p) @ v) / lsum
        att = bf16_round(att)
        x = x + att @ mat(o["o"][l], d, d)
        a = bf16_round(layer_norm(x, eps))
        hid = bf16_round(gelu_erf(a @ mat(o["w1"][l], d, ffn)))
        x = x + hid @ mat(o["w2"][l], ffn, d)
    a = bf16_round(layer_norm(x, eps))
    return (a @ mat(o["lm"], d, vocab)).astype(np.float32).reshape(B, S, vocab)
