"""The native tensor-op ABI (include/ptx/gpu/tensor_ops.h) against the
reference's own launchers of the same names (oracle/_ref/libref_kernels.so,
compiled from native/core/kernels/tensor_kernels.cu), on the same device
buffers: floating-point outputs bit-identical, index outputs identical.

Inputs mix normal values with the special values that separate
implementations (NaN, +-inf, +-0, denormals, the softplus / mish thresholds,
exp over/underflow points), at sizes that exercise the packed path, the
scalar tail and unaligned pointers. Reductions, softmax, cumsum, argsort,
topk and the index kernels run on shapes with inner == 1 (contiguous rows)
and inner > 1 (strided views), reduce sizes below and above 256, and ties.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

from fercuda_b200 import capi
from tests import oracle_lib

pytestmark = pytest.mark.gpu

P, SZ, F32, F64, I = C.c_void_p, C.c_size_t, C.c_float, C.c_double, C.c_int


@pytest.fixture(scope="module")
def libs():
    ref = oracle_lib.ref_kernels()
    if ref is None:
        pytest.skip("oracle/_ref not built")
    return capi.kernels(), ref


def bind(lib, name, argtypes, restype=None):
    f = getattr(lib, name)
    f.argtypes = argtypes
    f.restype = restype
    return f


def stream():
    return torch.cuda.current_stream().cuda_stream


SPECIALS = [float("nan"), float("inf"), -float("inf"), 0.0, -0.0, 1e-40, -1e-40, 88.7, 89.0, -103.0, -104.0,
            20.0, -20.0, 20.000002, 1e30, -1e30, 0.5, -0.5, 1.0, -1.0, 3.0, -3.0, 6.0, 1e-8]


def values(n: int, seed: int, dtype=torch.float32, scale=3.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(n, generator=g, device="cuda", dtype=torch.float32) * scale
    k = min(n, len(SPECIALS))
    x[:k] = torch.tensor(SPECIALS[:k], device="cuda")
    if n > 64:
        # distinct positions: an index_put with repeated indices picks its
        # winner nondeterministically on the GPU
        pos = torch.randperm(n, generator=g, device="cuda")[: min(n // 8, 4096)]
        x[pos] = torch.tensor(SPECIALS, device="cuda")[torch.arange(pos.numel(), device="cuda") % len(SPECIALS)]
    return x.to(dtype)


def same_bits(a: torch.Tensor, b: torch.Tensor) -> bool:
    if a.dtype in (torch.float32, torch.int32, torch.uint32):
        return torch.equal(a.view(torch.int32), b.view(torch.int32))
    if a.dtype == torch.float64:
        return torch.equal(a.view(torch.int64), b.view(torch.int64))
    if a.dtype in (torch.float16, torch.bfloat16):
        return torch.equal(a.view(torch.int16), b.view(torch.int16))
    return torch.equal(a, b)


def both(libs, name, argtypes, make_args):
    """Runs `name` from both libraries on fresh outputs; returns (ours, ref)."""
    outs = []
    for lib in libs:
        f = bind(lib, name, argtypes)
        args, out = make_args()
        f(*args)
        torch.cuda.synchronize()
        outs.append(out)
    return outs


SIZES = [1, 7, 1000, (1 << 20) + 3]
UNARY = ["neg", "abs", "exp", "log", "sqrt", "rsqrt", "sin", "cos", "tanh", "ceil", "floor", "round", "sqr", "recip",
         "log2", "log10", "tan", "sinh", "cosh", "sign", "erf", "relu", "relu6", "selu", "gelu", "gelu_tanh",
         "sigmoid", "silu", "softplus", "mish", "hardswish", "hardsigmoid"]
BINARY = ["add", "sub", "mul", "div", "max", "min", "mod"]


@pytest.mark.parametrize("n", SIZES)
@pytest.mark.parametrize("op", UNARY)
def test_unary_f32(libs, op, n):
    x = values(n + 1, 1)
    for off in (0, 1):                                   # aligned and 4-byte-offset pointers
        src = x[off:off + n]

        def mk():
            y = torch.full((n + 1,), 7.0, device="cuda")[off:off + n]
            return (src.data_ptr(), y.data_ptr(), n, stream()), y

        a, b = both(libs, f"ptx_tensor_{op}_f32", [P, P, SZ, P], mk)
        assert same_bits(a, b), (op, n, off)


@pytest.mark.parametrize("n", SIZES)
@pytest.mark.parametrize("op", BINARY)
def test_binary_f32(libs, op, n):
    x, y = values(n, 2), values(n, 3)
    y[: n // 3] = x[: n // 3]                            # equal operands for max / min / mod

    def mk():
        o = torch.empty(n, device="cuda")
        return (x.data_ptr(), y.data_ptr(), o.data_ptr(), n, stream()), o

    a, b = both(libs, f"ptx_tensor_{op}_f32", [P, P, P, SZ, P], mk)
    assert same_bits(a, b)


@pytest.mark.parametrize("op,params", [("add_scalar", (0.1,)), ("sub_scalar", (-3.5,)), ("mul_scalar", (1e-3,)),
                                       ("div_scalar", (3.0,)), ("leaky_relu", (0.01,)), ("elu", (1.3,)),
                                       ("clamp", (-1.5, 2.25)), ("powf", (2.5,)), ("powf", (-1.0,)),
                                       ("affine", (1.5, -0.25))])
def test_parametrised_f32(libs, op, params):
    n = (1 << 18) + 5
    x = values(n, 4)
    types = {"add_scalar": [P, F32, P, SZ, P], "sub_scalar": [P, F32, P, SZ, P], "mul_scalar": [P, F32, P, SZ, P],
             "div_scalar": [P, F32, P, SZ, P]}.get(op, [P, P, SZ] + [F32] * len(params) + [P])

    def mk():
        o = torch.empty(n, device="cuda")
        if op.endswith("_scalar"):
            return (x.data_ptr(), params[0], o.data_ptr(), n, stream()), o
        return (x.data_ptr(), o.data_ptr(), n, *params, stream()), o

    a, b = both(libs, f"ptx_tensor_{op}_f32", types, mk)
    assert same_bits(a, b)


@pytest.mark.parametrize("op", ["eq", "ne", "lt", "le", "gt", "ge"])
def test_compare_f32(libs, op):
    n = (1 << 16) + 3
    x, y = values(n, 5), values(n, 6)
    y[::3] = x[::3]

    def mk():
        o = torch.full((n,), 9, dtype=torch.uint8, device="cuda")
        return (x.data_ptr(), y.data_ptr(), o.data_ptr(), n, stream()), o

    a, b = both(libs, f"ptx_tensor_cmp_{op}_f32", [P, P, P, SZ, P], mk)
    assert torch.equal(a, b) and int(a.max()) <= 1


def test_where_copy_fill_casts(libs):
    n = (1 << 16) + 3
    c = (values(n, 7) > 0).to(torch.uint8)
    t, f = values(n, 8), values(n, 9)

    def mk_where():
        o = torch.empty(n, device="cuda")
        return (c.data_ptr(), t.data_ptr(), f.data_ptr(), o.data_ptr(), n, stream()), o

    a, b = both(libs, "ptx_tensor_where_f32", [P, P, P, P, SZ, P], mk_where)
    assert same_bits(a, b)

    def mk_copy():
        o = torch.empty(n, device="cuda")
        return (t.data_ptr(), o.data_ptr(), n, stream()), o

    a, b = both(libs, "ptx_tensor_copy_f32", [P, P, SZ, P], mk_copy)
    assert same_bits(a, b) and same_bits(a, t)

    def mk_fill():
        o = torch.empty(n, device="cuda")
        return (o.data_ptr(), n, -0.0, stream()), o

    a, b = both(libs, "ptx_tensor_fill_f32", [P, SZ, F32, P], mk_fill)
    assert same_bits(a, b)

    def mk_h():
        o = torch.empty(n, dtype=torch.float16, device="cuda")
        return (t.data_ptr(), o.data_ptr(), n, stream()), o

    a, b = both(libs, "ptx_tensor_cast_f32_to_f16", [P, P, SZ, P], mk_h)
    assert same_bits(a, b)
    h = a

    def mk_f():
        o = torch.empty(n, device="cuda")
        return (h.data_ptr(), o.data_ptr(), n, stream()), o

    a, b = both(libs, "ptx_tensor_cast_f16_to_f32", [P, P, SZ, P], mk_f)
    assert same_bits(a, b)


@pytest.mark.parametrize("op", ["add", "sub", "mul", "div", "neg", "exp", "log", "sqrt", "tanh", "relu", "gelu",
                                "sigmoid", "affine"])
def test_f64(libs, op, n=(1 << 17) + 3):
    x, y = values(n, 10, torch.float64), values(n, 11, torch.float64)

    def mk():
        o = torch.empty(n, dtype=torch.float64, device="cuda")
        if op in ("add", "sub", "mul", "div"):
            return (x.data_ptr(), y.data_ptr(), o.data_ptr(), n, stream()), o
        if op == "affine":
            return (x.data_ptr(), o.data_ptr(), n, 0.7, -1.25, stream()), o
        return (x.data_ptr(), o.data_ptr(), n, stream()), o

    types = ([P, P, P, SZ, P] if op in ("add", "sub", "mul", "div") else
             [P, P, SZ, F64, F64, P] if op == "affine" else [P, P, SZ, P])
    a, b = both(libs, f"ptx_tensor_{op}_f64", types, mk)
    assert same_bits(a, b)


@pytest.mark.parametrize("op", ["add", "sub", "mul", "div", "relu", "gelu", "sigmoid"])
def test_f16(libs, op, n=(1 << 17) + 5):
    x, y = values(n, 12, scale=2.0).half(), values(n, 13, scale=2.0).half()

    def mk():
        o = torch.empty(n, dtype=torch.float16, device="cuda")
        if op in ("add", "sub", "mul", "div"):
            return (x.data_ptr(), y.data_ptr(), o.data_ptr(), n, stream()), o
        return (x.data_ptr(), o.data_ptr(), n, stream()), o

    types = [P, P, P, SZ, P] if op in ("add", "sub", "mul", "div") else [P, P, SZ, P]
    a, b = both(libs, f"ptx_tensor_{op}_f16", types, mk)
    assert same_bits(a, b)


SHAPES = [(1, 1, 1), (1, 1000, 1), (7, 300, 1), (5, 100003, 1), (3, 257, 5), (2, 1000, 40), (4, 5000, 33),
          (2, 3, 70), (1, 100, 1000)]


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("op", ["sum", "mean", "max", "min", "prod"])
def test_reduce_f32(libs, op, shape):
    outer, red, inner = shape
    x = values(outer * red * inner, 14, scale=1.0 if op != "prod" else 0.2) + (1.0 if op == "prod" else 0.0)
    if op in ("sum", "mean"):
        x = torch.nan_to_num(x, nan=0.5, posinf=2.0, neginf=-2.0)    # finite sums; NaN/inf cases below

    def mk():
        o = torch.empty(outer * inner, device="cuda")
        return (x.data_ptr(), o.data_ptr(), outer, red, inner, stream()), o

    a, b = both(libs, f"ptx_tensor_reduce_{op}_f32", [P, P, SZ, SZ, SZ, P], mk)
    assert same_bits(a, b), (op, shape)


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("op", ["sum", "max", "min"])
def test_reduce_f64(libs, op, shape):
    outer, red, inner = shape
    x = torch.nan_to_num(values(outer * red * inner, 15, torch.float64, scale=1.0), nan=0.25)

    def mk():
        o = torch.empty(outer * inner, dtype=torch.float64, device="cuda")
        return (x.data_ptr(), o.data_ptr(), outer, red, inner, stream()), o

    a, b = both(libs, f"ptx_tensor_reduce_{op}_f64", [P, P, SZ, SZ, SZ, P], mk)
    assert same_bits(a, b), (op, shape)


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("op", ["argmax", "argmin"])
def test_arg_reduce(libs, op, shape):
    outer, red, inner = shape
    x = values(outer * red * inner, 16)
    x = torch.round(x * 2) / 2                             # ties

    def mk():
        o = torch.full((outer * inner,), -7, dtype=torch.int32, device="cuda")
        return (x.data_ptr(), o.data_ptr(), outer, red, inner, stream()), o

    a, b = both(libs, f"ptx_tensor_reduce_{op}_f32", [P, P, SZ, SZ, SZ, P], mk)
    assert torch.equal(a, b), (op, shape)


def test_reduce_sum_nan_inf(libs):
    x = values(3 * 700 * 9, 17)                            # NaN and +-inf among the summands

    def mk():
        o = torch.empty(3 * 9, device="cuda")
        return (x.data_ptr(), o.data_ptr(), 3, 700, 9, stream()), o

    a, b = both(libs, "ptx_tensor_reduce_sum_f32", [P, P, SZ, SZ, SZ, P], mk)
    assert same_bits(a, b)


@pytest.mark.parametrize("batch,dim", [(1, 1), (3, 1000), (64, 257), (2, 5000), (300, 64)])
@pytest.mark.parametrize("name,dt", [("log_softmax_f32", torch.float32), ("softmax_f64", torch.float64),
                                     ("softmax_f16", torch.float16), ("softmax_f32", torch.float32)])
def test_softmax_variants(libs, name, dt, batch, dim):
    x = torch.nan_to_num(values(batch * dim, 18, scale=2.0), nan=0.0, posinf=30.0, neginf=-30.0).to(dt)

    def mk():
        o = torch.empty(batch * dim, dtype=dt, device="cuda")
        return (x.data_ptr(), o.data_ptr(), batch, dim, stream()), o

    a, b = both(libs, f"ptx_tensor_{name}", [P, P, SZ, SZ, P], mk)
    assert same_bits(a, b), (name, batch, dim)


@pytest.mark.parametrize("shape", [(4, 1000, 1), (1000, 33, 1), (3, 100, 7), (1, 70000, 1), (2, 5, 300)])
def test_cumsum(libs, shape):
    outer, dim, inner = shape
    x = torch.nan_to_num(values(outer * dim * inner, 19, scale=1.0), nan=0.1, posinf=1.0, neginf=-1.0)

    def mk():
        o = torch.empty(outer * dim * inner, device="cuda")
        return (x.data_ptr(), o.data_ptr(), outer, dim, inner, stream()), o

    a, b = both(libs, "ptx_tensor_cumsum_f32", [P, P, SZ, SZ, SZ, P], mk)
    assert same_bits(a, b)


@pytest.mark.parametrize("rows,cols", [(1, 1), (5, 1000), (3, 1024), (7, 33), (2, 8192), (40, 100)])
@pytest.mark.parametrize("asc", [1, 0])
def test_argsort(libs, rows, cols, asc):
    x = torch.round(values(rows * cols, 20) * 2) / 2         # ties, NaN, inf

    def mk():
        o = torch.zeros(rows * cols, dtype=torch.int32, device="cuda")
        return (x.data_ptr(), o.data_ptr(), rows, cols, asc, stream()), o

    a, b = both(libs, "ptx_tensor_argsort_f32", [P, P, SZ, SZ, I, P], mk)
    assert torch.equal(a, b)
    perm = a.view(rows, cols).long()
    assert torch.equal(torch.sort(perm, 1).values, torch.arange(cols, device="cuda").expand(rows, cols))


@pytest.mark.parametrize("outer,dim,inner,k,largest", [(4, 1000, 1, 10, 1), (3, 100, 5, 7, 0), (2, 50, 1, 60, 1),
                                                       (1, 5000, 1, 64, 0), (6, 257, 3, 1, 1)])
def test_topk(libs, outer, dim, inner, k, largest):
    x = torch.round(values(outer * dim * inner, 21) * 2) / 2

    def mk():
        v = torch.full((outer * k * inner,), 5.5, device="cuda")
        ix = torch.full((outer * k * inner,), -9, dtype=torch.int32, device="cuda")
        mk.ix = ix
        return (x.data_ptr(), v.data_ptr(), ix.data_ptr(), outer, dim, inner, k, largest, stream()), v

    outs = []
    for lib in libs:
        f = bind(lib, "ptx_tensor_topk_f32", [P, P, P, SZ, SZ, SZ, SZ, I, P])
        args, v = mk()
        f(*args)
        torch.cuda.synchronize()
        outs.append((v, mk.ix))
    (va, ia), (vb, ib) = outs
    assert same_bits(va, vb) and torch.equal(ia, ib)


def test_gather_index_select(libs):
    outer, in_dim, idx_dim, inner = 3, 50, 70, 9
    x = values(outer * in_dim * inner, 22)
    g = torch.Generator(device="cuda").manual_seed(23)
    idx = torch.randint(-60, 60, (outer * idx_dim * inner,), generator=g, device="cuda", dtype=torch.int32)

    def mk():
        o = torch.empty(outer * idx_dim * inner, device="cuda")
        return (x.data_ptr(), idx.data_ptr(), o.data_ptr(), outer, in_dim, idx_dim, inner, stream()), o

    a, b = both(libs, "ptx_tensor_gather_f32", [P, P, P, SZ, SZ, SZ, SZ, P], mk)
    assert same_bits(a, b)
    ids = idx[:idx_dim].contiguous()

    def mk2():
        o = torch.empty(outer * idx_dim * inner, device="cuda")
        return (x.data_ptr(), ids.data_ptr(), o.data_ptr(), outer, in_dim, idx_dim, inner, stream()), o

    a, b = both(libs, "ptx_tensor_index_select_f32", [P, P, P, SZ, SZ, SZ, SZ, P], mk2)
    assert same_bits(a, b)


@pytest.mark.parametrize("left,src_dim,dst_dim,right", [(2, 300, 300, 600), (1, 500, 500, 3), (4, 64, 64, 1)])
def test_scatter_add_unique_ids(libs, left, src_dim, dst_dim, right):
    """Unique destination indices: no two sources meet, so the reference's
    atomics and the deterministic column path agree bit for bit."""
    g = torch.Generator(device="cuda").manual_seed(24)
    ids = torch.randperm(dst_dim, generator=g, device="cuda")[:src_dim].to(torch.int32)
    src = values(left * src_dim * right, 25)
    base = values(left * dst_dim * right, 26)

    def mk():
        o = base.clone()
        return (ids.data_ptr(), src.data_ptr(), o.data_ptr(), left, src_dim, dst_dim, right, stream()), o

    a, b = both(libs, "ptx_tensor_scatter_add_f32", [P, P, P, SZ, SZ, SZ, SZ, P], mk)
    assert same_bits(a, b)


def _ftz(x: np.ndarray) -> np.ndarray:
    return np.where(np.abs(x) < np.float32(1.17549435e-38), np.copysign(np.float32(0), x), x).astype(np.float32)


def test_scatter_add_repeated_ids_is_deterministic(libs):
    """Repeated indices with >= 1024 columns: sources added in index order,
    each add as a float atomicAdd performs it (subnormals flushed), the same
    bits as that sequence in numpy float32, every run."""
    ours = libs[0]
    left, src_dim, dst_dim, right = 2, 400, 37, 700
    g = torch.Generator(device="cuda").manual_seed(27)
    ids = torch.randint(-37, 45, (src_dim,), generator=g, device="cuda", dtype=torch.int32)
    src = torch.nan_to_num(values(left * src_dim * right, 28, scale=1.0), nan=0.0, posinf=1.0, neginf=-1.0)
    f = bind(ours, "ptx_tensor_scatter_add_f32", [P, P, P, SZ, SZ, SZ, SZ, P])
    runs = []
    for _ in range(3):
        o = torch.zeros(left * dst_dim * right, device="cuda")
        f(ids.data_ptr(), src.data_ptr(), o.data_ptr(), left, src_dim, dst_dim, right, stream())
        torch.cuda.synchronize()
        runs.append(o)
    assert all(same_bits(runs[0], r) for r in runs[1:])
    s = src.cpu().numpy().reshape(left, src_dim, right)
    want = np.zeros((left, dst_dim, right), np.float32)
    for k, d in enumerate(ids.cpu().numpy()):
        d = d + dst_dim if d < 0 else d
        if 0 <= d < dst_dim:
            want[:, d, :] = _ftz(_ftz(want[:, d, :]) + _ftz(s[:, k, :]))
    assert np.array_equal(runs[0].cpu().numpy().reshape(want.shape).view(np.int32), want.view(np.int32))


class PTXTensorOp(C.Structure):
    _fields_ = [("opcode", C.c_int), ("dtype", C.c_int), ("input_a", P), ("input_b", P), ("output", P),
                ("elem_count", SZ), ("scalar_a", F32), ("scalar_b", F32), ("reduce_dim", C.c_uint32),
                ("reduce_size", C.c_uint32), ("outer_size", C.c_uint32), ("inner_size", C.c_uint32),
                ("stream", P)]


@pytest.mark.parametrize("opcode,dtype,kind", [(0x10, 0, "bin"), (0x10, 1, "bin"), (0x10, 2, "bin"), (0x13, 0, "bin"),
                                               (0x45, 0, "un"), (0x45, 2, "un"), (0x2B, 1, "un"), (0x50, 0, "red"),
                                               (0x53, 1, "red"), (0x60, 2, "red"), (0x61, 0, "red"), (0x80, 0, "un"),
                                               (0x82, 0, "where"), (0x75, 0, "cmp"), (0xC0, 0, "red")])
def test_dispatch_matches_reference_dispatch(libs, opcode, dtype, kind):
    n, outer, red, inner = 3000, 6, 500, 1
    tdt = {0: torch.float32, 1: torch.float64, 2: torch.float16}[dtype]
    x = torch.nan_to_num(values(n, 29, scale=1.0), nan=0.0).to(tdt)
    y = torch.nan_to_num(values(n, 30, scale=1.0), nan=1.0).to(tdt)
    cond = (values(n, 31) > 0).to(torch.uint8)
    start = values(n, 32).to(tdt)                          # WHERE's false branch is the output buffer
    outs = []
    for lib in libs:
        f = bind(lib, "ptx_tensor_dispatch", [C.POINTER(PTXTensorOp)], C.c_int)
        o = (torch.zeros(n, dtype=torch.uint8, device="cuda") if kind == "cmp" else
             start.clone() if kind == "where" else torch.zeros(n, dtype=tdt, device="cuda"))
        op = PTXTensorOp(opcode, dtype, (cond if kind == "where" else x).data_ptr(),
                         (y.data_ptr() if kind in ("bin", "where", "cmp") else None), o.data_ptr(), n, 1.5, -0.5, 0,
                         red, outer, inner, stream())
        o0 = o.clone()
        assert f(C.byref(op)) == 0
        torch.cuda.synchronize()
        outs.append(o)
    if kind == "where":           # output = input_a ? input_b : output, as the reference dispatch does
        want = torch.where(cond.bool(), y, o0)
        assert same_bits(outs[0], want), "ours"
        assert same_bits(outs[1], want), "reference"
    assert same_bits(outs[0], outs[1]), (hex(opcode), dtype)


def test_dispatch_unknown_opcode_and_sync(libs):
    ours = libs[0]
    f = bind(ours, "ptx_tensor_dispatch", [C.POINTER(PTXTensorOp)], C.c_int)
    fs = bind(ours, "ptx_tensor_dispatch_sync", [C.POINTER(PTXTensorOp)], C.c_int)
    x = torch.ones(10, device="cuda")
    op = PTXTensorOp(0x91, 0, x.data_ptr(), None, x.data_ptr(), 10, 0, 0, 0, 0, 0, 0, None)
    assert f(C.byref(op)) != 0                            # CAST has no dispatch entry, as in the reference
    assert f(None) != 0
    op = PTXTensorOp(0x92, 0, None, None, x.data_ptr(), 10, 2.5, 0, 0, 0, 0, 0, None)   # FILL, legacy stream
    assert fs(C.byref(op)) == 0
    assert torch.equal(x, torch.full((10,), 2.5, device="cuda"))


def test_graph_capture_helpers(libs):
    ours = libs[0]
    n = 4096
    x, y = values(n, 33), values(n, 34)
    out = torch.empty(n, device="cuda")
    s = torch.cuda.Stream()
    begin = bind(ours, "ptx_tensor_graph_begin_capture", [P], C.c_int)
    end = bind(ours, "ptx_tensor_graph_end_capture", [P, C.POINTER(P)], C.c_int)
    inst = bind(ours, "ptx_tensor_graph_instantiate", [P, C.POINTER(P)], C.c_int)
    launch = bind(ours, "ptx_tensor_graph_launch", [P, P], C.c_int)
    add = bind(ours, "ptx_tensor_add_f32", [P, P, P, SZ, P])
    gelu = bind(ours, "ptx_tensor_gelu_f32", [P, P, SZ, P])
    graph, exe = P(), P()
    with torch.cuda.stream(s):
        assert begin(s.cuda_stream) == 0
        add(x.data_ptr(), y.data_ptr(), out.data_ptr(), n, s.cuda_stream)
        gelu(out.data_ptr(), out.data_ptr(), n, s.cuda_stream)
        assert end(s.cuda_stream, C.byref(graph)) == 0
    assert inst(graph, C.byref(exe)) == 0
    assert launch(exe, s.cuda_stream) == 0
    s.synchronize()
    want = torch.empty(n, device="cuda")
    add(x.data_ptr(), y.data_ptr(), want.data_ptr(), n, stream())
    gelu(want.data_ptr(), want.data_ptr(), n, stream())
    torch.cuda.synchronize()
    assert same_bits(out, want)
    rt = C.CDLL("libcudart.so.12")                       # the runtime torch loaded
    rt.cudaGraphExecDestroy.argtypes = [P]
    rt.cudaGraphDestroy.argtypes = [P]
    rt.cudaGraphExecDestroy(exe)
    rt.cudaGraphDestroy(graph)


def _time_us(f, args, iters=10):
    for _ in range(3):
        f(*args)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        f(*args)
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters * 1e3


def test_speed_against_reference(libs):
    """Time each launcher against the reference launcher of the same name on
    the same buffers (inputs 256 MiB and up, so both run from HBM); print
    the table (run with -s) and guard against falling behind the reference.
    Bytes are algorithmic (one read of each input, one write of each
    output)."""
    n = 1 << 26
    st = stream()
    a, b, o = torch.randn(n, device="cuda"), torch.randn(n, device="cuda"), torch.empty(n, device="cuda")
    ad, od = a[: n // 2].double(), torch.empty(n // 2, dtype=torch.float64, device="cuda")
    ah, bh, oh = a.half(), b.half(), torch.empty(n, dtype=torch.float16, device="cuda")
    u8, ix = torch.empty(n, dtype=torch.uint8, device="cuda"), torch.empty(8192, dtype=torch.int32, device="cuda")
    cases = [
        ("add_f32 2^26", "ptx_tensor_add_f32", [P, P, P, SZ, P], (a.data_ptr(), b.data_ptr(), o.data_ptr(), n, st), 12 * n),
        ("gelu_f32 2^26", "ptx_tensor_gelu_f32", [P, P, SZ, P], (a.data_ptr(), o.data_ptr(), n, st), 8 * n),
        ("erf_f32 2^26", "ptx_tensor_erf_f32", [P, P, SZ, P], (a.data_ptr(), o.data_ptr(), n, st), 8 * n),
        ("exp_f64 2^25", "ptx_tensor_exp_f64", [P, P, SZ, P], (ad.data_ptr(), od.data_ptr(), n // 2, st), 8 * n),
        ("add_f16 2^26", "ptx_tensor_add_f16", [P, P, P, SZ, P], (ah.data_ptr(), bh.data_ptr(), oh.data_ptr(), n, st),
         6 * n),
        ("cmp_lt_f32 2^26", "ptx_tensor_cmp_lt_f32", [P, P, P, SZ, P], (a.data_ptr(), b.data_ptr(), u8.data_ptr(), n, st),
         9 * n),
        ("reduce_sum 16384x4096 (rows)", "ptx_tensor_reduce_sum_f32", [P, P, SZ, SZ, SZ, P],
         (a.data_ptr(), o.data_ptr(), 16384, 4096, 1, st), 4 * n),
        ("reduce_sum 256x4096x64 (strided)", "ptx_tensor_reduce_sum_f32", [P, P, SZ, SZ, SZ, P],
         (a.data_ptr(), o.data_ptr(), 256, 4096, 64, st), 4 * n),
        ("reduce_max 64x1024x1024 (strided)", "ptx_tensor_reduce_max_f32", [P, P, SZ, SZ, SZ, P],
         (a.data_ptr(), o.data_ptr(), 64, 1024, 1024, st), 4 * n),
        ("argmax 16384x4096", "ptx_tensor_reduce_argmax_f32", [P, P, SZ, SZ, SZ, P],
         (a.data_ptr(), o.data_ptr(), 16384, 4096, 1, st), 4 * n),
        ("log_softmax_f32 16384x4096", "ptx_tensor_log_softmax_f32", [P, P, SZ, SZ, P],
         (a.data_ptr(), o.data_ptr(), 16384, 4096, st), 8 * n),
        ("softmax_f16 16384x4096", "ptx_tensor_softmax_f16", [P, P, SZ, SZ, P], (ah.data_ptr(), oh.data_ptr(), 16384, 4096, st),
         4 * n),
        ("softmax_f64 8192x4096", "ptx_tensor_softmax_f64", [P, P, SZ, SZ, P], (ad.data_ptr(), od.data_ptr(), 8192, 4096, st),
         8 * n),
        ("cumsum 16384x4096", "ptx_tensor_cumsum_f32", [P, P, SZ, SZ, SZ, P], (a.data_ptr(), o.data_ptr(), 16384, 4096, 1, st),
         8 * n),
        ("argsort 8192x1024", "ptx_tensor_argsort_f32", [P, P, SZ, SZ, I, P], (a.data_ptr(), u8.data_ptr(), 8192, 1024, 1, st),
         8 * 8192 * 1024),
        ("topk 1024x32000 k=8", "ptx_tensor_topk_f32", [P, P, P, SZ, SZ, SZ, SZ, I, P],
         (a.data_ptr(), o.data_ptr(), ix.data_ptr(), 1024, 32000, 1, 8, 1, st), 4 * 1024 * 32000),
    ]
    print(f"\n{'launcher':36s} {'ours us':>9s} {'ref us':>9s} {'ours GB/s':>10s} {'ref GB/s':>9s} {'x':>6s}")
    slower = []
    for label, name, types, args, nbytes in cases:
        t = [_time_us(bind(lib, name, types), args) for lib in libs]
        print(f"{label:36s} {t[0]:9.1f} {t[1]:9.1f} {nbytes / t[0] / 1e3:10.0f} {nbytes / t[1] / 1e3:9.0f} "
              f"{t[1] / t[0]:6.2f}")
        if t[0] > 1.1 * t[1]:
            slower.append(label)
    assert not slower, slower
