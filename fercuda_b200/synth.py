"""Seeded synthetic inputs for every workload, byte-identical wherever they are
generated (tests, bench, CPU baseline).

Generator: splitmix64 with the workload's seed. The k-th draw (k = 1, 2, ...)
is mix(seed + k * 0x9E3779B97F4A7C15), so streams are computed in bulk.
  uniform01  = (draw >> 40) * 2^-24                 (24-bit, in [0, 1))
  uniform    = lo + (hi - lo) * uniform01, in float64, rounded once to f32
  normal     = Box-Muller in float64 on draws 2i+1, 2i+2 for sample i:
               u1 = ((d0 >> 11) + 1) * 2^-53, u2 = (d1 >> 11) * 2^-53,
               z = sqrt(-2 ln u1) * cos(2 pi u2); mean + std * z rounded once
               to f32 (mean and std are taken as f32 values)
  bf16       = round-to-nearest-even of that float32

ln and cos are this module's own series (portable_ln, portable_cos_turns),
evaluated with IEEE float64 +, -, *, / and sqrt only, each rounded to
nearest, in a fixed order. Any IEEE machine that follows the same steps
without contracting a multiply and an add therefore gets the same bits: the
device fill of the transformer weights (kernels/xfmr_kernels.cu,
fill_normal_bf16) reproduces normal_bf16 exactly, which is what lets a
fixture computed on the host pin the device forward.
"""
from __future__ import annotations

import math
import os

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


# Series coefficients, correctly rounded: 1/(2k+1) for ln (atanh series),
# (-1)^k/(2k+1)! for sin, (-1)^k/(2k)! for cos. The device kernel carries the
# same values as hexadecimal literals.
LN_SERIES = tuple(float.fromhex(h) for h in (
    "0x1.0000000000000p+0", "0x1.5555555555555p-2", "0x1.999999999999ap-3", "0x1.2492492492492p-3",
    "0x1.c71c71c71c71cp-4", "0x1.745d1745d1746p-4", "0x1.3b13b13b13b14p-4", "0x1.1111111111111p-4",
    "0x1.e1e1e1e1e1e1ep-5", "0x1.af286bca1af28p-5", "0x1.8618618618618p-5"))
SIN_SERIES = tuple(float.fromhex(h) for h in (
    "0x1.0000000000000p+0", "-0x1.5555555555555p-3", "0x1.1111111111111p-7", "-0x1.a01a01a01a01ap-13",
    "0x1.71de3a556c734p-19", "-0x1.ae64567f544e4p-26", "0x1.6124613a86d09p-33", "-0x1.ae7f3e733b81fp-41",
    "0x1.952c77030ad4ap-49"))
COS_SERIES = tuple(float.fromhex(h) for h in (
    "0x1.0000000000000p+0", "-0x1.0000000000000p-1", "0x1.5555555555555p-5", "-0x1.6c16c16c16c17p-10",
    "0x1.a01a01a01a01ap-16", "-0x1.27e4fb7789f5cp-22", "0x1.1eed8eff8d898p-29", "-0x1.93974a8c07c9dp-37",
    "0x1.ae7f3e733b81fp-45", "-0x1.6827863b97d97p-53"))
LN2 = float.fromhex("0x1.62e42fefa39efp-1")
TWO_PI = float.fromhex("0x1.921fb54442d18p+2")
SQRT_HALF = float.fromhex("0x1.6a09e667f3bcdp-1")


def _horner(coef: tuple, t: np.ndarray) -> np.ndarray:
    """sum coef[k] t^k, highest term first, one rounding per multiply and add."""
    p = np.full_like(t, coef[-1])
    for c in coef[-2::-1]:
        np.multiply(p, t, out=p)
        np.add(p, c, out=p)
    return p


def portable_ln(k: np.ndarray) -> np.ndarray:
    """ln(k * 2^-53) for integers 1 <= k <= 2^53 (uint64). k = f * 2^b with
    f in [sqrt(1/2), sqrt(2)) (exact), ln = (b - 53) ln 2 + 2 atanh(s),
    s = (f - 1) / (f + 1), atanh by its series in s^2 (|s| <= 0.1716, 11
    terms, truncation below 2^-56)."""
    f, b = np.frexp(k.astype(np.float64))
    e = b.astype(np.float64) - 53.0
    low = f < SQRT_HALF
    f[low] *= 2.0
    e[low] -= 1.0
    s = (f - 1.0) / (f + 1.0)
    p = _horner(LN_SERIES, s * s)
    return e * LN2 + (2.0 * s) * p


def portable_cos_turns(k: np.ndarray) -> np.ndarray:
    """cos(2 pi k 2^-53) for integers 0 <= k < 2^53 (uint64). The octant
    q = k >> 50 and the offset r in [0, 1/8) turn are exact; odd octants
    use 1/8 - r, so the series argument x = 2 pi w stays in [0, pi/4]; the
    octant picks sin or cos of x and the sign."""
    q = (k >> np.uint64(50)).astype(np.int64)
    r = (k & np.uint64((1 << 50) - 1)).astype(np.float64) * (2.0 ** -53)
    odd = (q & 1) == 1
    r[odd] = 0.125 - r[odd]
    x = TWO_PI * r
    x2 = x * x
    use_cos = (q == 0) | (q == 3) | (q == 4) | (q == 7)
    v = np.empty_like(x)
    v[use_cos] = _horner(COS_SERIES, x2[use_cos])
    sn = ~use_cos
    v[sn] = x[sn] * _horner(SIN_SERIES, x2[sn])
    neg = (q >= 2) & (q <= 5)
    v[neg] = -v[neg]
    return v


def _normal_chunk(seed: int, lo: int, m: int, mean: float, std: float) -> np.ndarray:
    d = splitmix64(seed, 2 * m, start=2 * lo)
    k1 = (d[0::2] >> np.uint64(11)) + np.uint64(1)
    k2 = d[1::2] >> np.uint64(11)
    z = np.sqrt(-2.0 * portable_ln(k1)) * portable_cos_turns(k2)
    return (mean + std * z).astype(np.float32)


def normal_f32(seed: int, n: int, mean: float = 0.0, std: float = 1.0, chunk: int = 1 << 21) -> np.ndarray:
    """n normal draws (module docstring), chunks evaluated on a thread pool
    (numpy releases the GIL inside its loops)."""
    mean = float(np.float32(mean))
    std = float(np.float32(std))
    out = np.empty(n, dtype=np.float32)
    starts = list(range(0, n, chunk))

    def one(lo: int) -> None:
        m = min(chunk, n - lo)
        out[lo:lo + m] = _normal_chunk(seed, lo, m, mean, std)

    if len(starts) <= 1:
        for lo in starts:
            one(lo)
    else:
        from concurrent.futures import ThreadPoolExecutor

        with ThreadPoolExecutor(max_workers=min(len(starts), os.cpu_count() or 1)) as ex:
            list(ex.map(one, starts))
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
