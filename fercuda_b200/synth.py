"""Seeded synthetic inputs for every workload, byte-identical wherever they are
generated (tests, bench, CPU baseline).

Generator: splitmix64 with the workload's seed. The k-th draw (k = 1, 2, ...)
is mix(seed + k * 0x9E3779B97F4A7C15), so streams are computed in bulk.
  uniform01  = (draw >> 40) * 2^-24                 (24-bit, in [0, 1))
  uniform    = lo + (hi - lo) * uniform01, in float64, rounded once to f32
  normal     = Box-Muller in float64 on two draws per sample:
               u1 = ((d0 >> 11) + 1) * 2^-53, u2 = (d1 >> 11) * 2^-53,
               z = sqrt(-2 ln u1) * cos(2 pi u2); mean + std * z rounded once
  bf16       = round-to-nearest-even of that float32
"""
from __future__ import annotations

import math

import numpy as np

GAMMA = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def splitmix64(seed: int, n: int, start: int = 0) -> np.ndarray:
    """Draws start+1 .. start+n of the splitmix64 stream for `seed`."""
    k = np.arange(start + 1, start + n + 1, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = np.uint64(seed & 0xFFFFFFFFFFFFFFFF) + k * GAMMA
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        z = z ^ (z >> np.uint64(31))
    return z


def uniform01(seed: int, n: int, start: int = 0) -> np.ndarray:
    return (splitmix64(seed, n, start) >> np.uint64(40)).astype(np.float64) * (2.0 ** -24)


def uniform_f32(seed: int, n: int, lo: float, hi: float) -> np.ndarray:
    return (lo + (hi - lo) * uniform01(seed, n)).astype(np.float32)


def normal_f32(seed: int, n: int, mean: float = 0.0, std: float = 1.0, chunk: int = 1 << 24) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    for lo in range(0, n, chunk):
        m = min(chunk, n - lo)
        d = splitmix64(seed, 2 * m, start=2 * lo)
        u1 = ((d[0::2] >> np.uint64(11)).astype(np.float64) + 1.0) * (2.0 ** -53)
        u2 = (d[1::2] >> np.uint64(11)).astype(np.float64) * (2.0 ** -53)
        z = np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * math.pi * u2)
        out[lo:lo + m] = (mean + std * z).astype(np.float32)
    return out


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rounding = ((u >> np.uint32(16)) & np.uint32(1)) + np.uint32(0x7FFF)
    with np.errstate(over="ignore"):
        return ((u + rounding) >> np.uint32(16)).astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def normal_bf16(seed: int, n: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    """bf16 bit patterns (uint16) of normal_f32 draws."""
    return f32_to_bf16_bits(normal_f32(seed, n, mean, std))


# ----------------------------------------------------------------- workloads

FUSED_ELEMENTWISE = dict(n=1 << 20, seed=0, lo=-4.0, hi=4.0, a=1.5, b=-0.25)
SOFTMAX_LAYERNORM = dict(rows=4096, cols=4096, seed=1, eps=1e-5)
TLSF_STRESS = dict(ops=1_000_000, seed=2, min_size=256, max_size=16 << 20,
                   alloc_frac=0.6, live_cap=64 << 30)
GEMM = dict(m=8192, n=8192, k=8192, seed=3)
TRANSFORMER = dict(layers=8, d_model=1024, heads=16, ffn=4096, vocab=32000, seq=512,
                   batch=64, weight_seed=4, token_seed=5, eps=1e-5)


def fused_elementwise_input(n: int | None = None) -> np.ndarray:
    c = FUSED_ELEMENTWISE
    return uniform_f32(c["seed"], c["n"] if n is None else n, c["lo"], c["hi"])


def softmax_layernorm_input(rows: int | None = None, cols: int | None = None) -> np.ndarray:
    c = SOFTMAX_LAYERNORM
    r = c["rows"] if rows is None else rows
    k = c["cols"] if cols is None else cols
    return normal_f32(c["seed"], r * k).reshape(r, k)


def gemm_inputs(m: int | None = None, n: int | None = None, k: int | None = None):
    """A [m,k] and B [k,n] bf16 bit patterns, entries ~ N(0, 1/sqrt(K)).
    A takes the first m*k samples of the seed's stream, B the next k*n."""
    c = GEMM
    m = c["m"] if m is None else m
    n = c["n"] if n is None else n
    k = c["k"] if k is None else k
    std = 1.0 / math.sqrt(k)
    ab = normal_bf16(c["seed"], m * k + k * n, 0.0, std)
    return ab[: m * k].reshape(m, k), ab[m * k:].reshape(k, n)


def tlsf_trace(ops: int | None = None, seed: int | None = None, live_cap: int | None = None,
               min_size: int | None = None, max_size: int | None = None) -> np.ndarray:
    """Allocator-independent alloc/free trace.

    Entry > 0: allocate that many bytes. Entry < 0: free the allocation made
    by the (-entry - 1)-th alloc of the trace. Per op, three draws:
    u (alloc if u < alloc_frac), the size draw (log-uniform over
    [min_size, max_size], rounded to whole bytes) and the victim draw (index
    into the live list, which is kept in insertion order with swap-remove).
    An alloc that would push the requested live bytes past live_cap becomes a
    free; a free with nothing live becomes an alloc."""
    c = TLSF_STRESS
    ops = c["ops"] if ops is None else ops
    seed = c["seed"] if seed is None else seed
    cap = c["live_cap"] if live_cap is None else live_cap
    lo = c["min_size"] if min_size is None else min_size
    hi = c["max_size"] if max_size is None else max_size
    u = uniform01(seed, 3 * ops).reshape(ops, 3)
    sizes = np.rint(np.exp(math.log(lo) + u[:, 1] * (math.log(hi) - math.log(lo)))).astype(np.int64)
    is_alloc = u[:, 0] < c["alloc_frac"]
    pick = u[:, 2]
    out = np.empty(ops, dtype=np.int64)
    live: list[int] = []
    live_sz: list[int] = []
    sizes_l = sizes.tolist()
    alloc_l = is_alloc.tolist()
    pick_l = pick.tolist()
    live_bytes = 0
    n_alloc = 0
    for i in range(ops):
        s = sizes_l[i]
        a = alloc_l[i]
        if a and live_bytes + s > cap:
            a = False
        if not a and not live:
            a = True
        if a:
            out[i] = s
            live.append(n_alloc)
            live_sz.append(s)
            live_bytes += s
            n_alloc += 1
        else:
            j = int(pick_l[i] * len(live))
            out[i] = -(live[j] + 1)
            live_bytes -= live_sz[j]
            live[j] = live[-1]
            live_sz[j] = live_sz[-1]
            live.pop()
            live_sz.pop()
    return out
