"""Fused elementwise chain on the GPU, through the C ABI, against
  (a) the reference's own kernels (oracle/_ref, built from the reference
      sources with the reference's flags) run on the same device buffers:
      bit-exact;
  (b) the CPU oracle: bit-exact except sigmoid's expf (CUDA's <= 2 ULP vs
      glibc's <= 1 ULP, carried through 1+e, the division and the product),
      so within 4 ULP;
plus run-to-run determinism and the reference's own affine-intent test."""
import ctypes as C

import numpy as np
import pytest

from fercuda_b200 import capi, synth
from tests import oracle_lib

pytestmark = pytest.mark.gpu

FUSED = capi.FER_JIT_INTENT_FUSION_RELU | capi.FER_JIT_INTENT_FUSION_MUL_SIGMOID_INPUT
A, B = 1.5, -0.25


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def same_bits(x, y):
    bx, by = bits(x), bits(y)
    nan = np.isnan(x) & np.isnan(y)
    return bool(np.all((bx == by) | nan))


def special_values(n):
    vals = np.array([0.0, -0.0, 1.0, -1.0, np.inf, -np.inf, np.nan, 1e-40, -1e-40, 88.0, -88.0, 100.0, -100.0,
                     3.4e38, -3.4e38, 1e-30, 0.16666667, -0.16666667], np.float32)
    return np.resize(vals, n).astype(np.float32)


def run_reference_chain(session, ref, bx, n):
    st = C.c_void_p(session.stream())
    t = [session.alloc(capi.FER_DTYPE_F32, [n]) for _ in range(4)]
    p = [C.c_void_p(session.ptr_of(b)) for b in [bx] + t]
    ref.ptx_tensor_affine_f32(p[0], p[1], n, A, B, st)
    ref.ptx_tensor_relu_f32(p[1], p[2], n, st)
    ref.ptx_tensor_sigmoid_f32(p[0], p[3], n, st)
    ref.ptx_tensor_mul_f32(p[2], p[3], p[4], n, st)
    out = np.empty(n, np.float32)
    session.download(t[3], out)
    for b in t:
        session.free(b)
    return out


def run_fused(session, x):
    n = x.size
    bx, by = session.alloc(capi.FER_DTYPE_F32, [n]), session.alloc(capi.FER_DTYPE_F32, [n])
    session.upload(bx, x)
    session.wait(session.affine(bx, by, n, A, B, FUSED))
    y = np.empty(n, np.float32)
    session.download(by, y)
    return bx, by, y


@pytest.mark.parametrize("n", [1, 3, 5, 1024, 4099, 1 << 20])
def test_chain_bit_exact_vs_reference_kernels(session, n):
    ref = oracle_lib.ref_kernels()
    if ref is None:
        pytest.skip("oracle/_ref not built")
    x = synth.fused_elementwise_input(n)
    bx, by, y = run_fused(session, x)
    y_ref = run_reference_chain(session, ref, bx, n)
    assert same_bits(y, y_ref)
    session.free(bx)
    session.free(by)


def test_chain_special_values_vs_reference(session):
    ref = oracle_lib.ref_kernels()
    if ref is None:
        pytest.skip("oracle/_ref not built")
    x = special_values(1031)
    bx, by, y = run_fused(session, x)
    assert same_bits(y, run_reference_chain(session, ref, bx, x.size))
    session.free(bx)
    session.free(by)


def test_chain_vs_cpu_oracle_full_size(session):
    x = synth.fused_elementwise_input()
    n = x.size
    _, _, y = run_fused(session, x)
    ref = np.empty(n, np.float32)
    oracle_lib.load().orc_chain_f32(oracle_lib.ptr(x), oracle_lib.ptr(ref), n, A, B, 8)
    ulp = np.abs(bits(y).astype(np.int64) - bits(ref).astype(np.int64))
    assert ulp.max() <= 4
    assert (ulp == 0).mean() > 0.9
    # affine + relu stage is exact: where relu clamps, the product is exactly 0
    assert np.all(y[(x * np.float32(A) + np.float32(B)) <= 0] == 0)


def test_chain_deterministic_10_runs(session):
    x = synth.fused_elementwise_input()
    bx, by, first = run_fused(session, x)
    for _ in range(10):
        session.wait(session.affine(bx, by, x.size, A, B, FUSED))
        y = np.empty_like(first)
        session.download(by, y)
        assert np.array_equal(bits(y), bits(first))


def test_chain_api_matches_intent(session):
    x = synth.fused_elementwise_input(100003)
    bx, by, y = run_fused(session, x)
    bz = session.alloc(capi.FER_DTYPE_F32, [x.size])
    session.wait(session.chain(capi.config1_chain(A, B), [bx], bz))
    z = np.empty_like(y)
    session.download(bz, z)
    assert np.array_equal(bits(y), bits(z))


@pytest.mark.parametrize("op,refname", [(capi.FER_CHAIN_SIGMOID, "ptx_tensor_sigmoid_f32"),
                                        (capi.FER_CHAIN_RELU, "ptx_tensor_relu_f32")])
def test_chain_unary_ops_vs_reference(session, op, refname):
    ref = oracle_lib.ref_kernels()
    if ref is None:
        pytest.skip("oracle/_ref not built")
    n = 77777
    x = np.concatenate([special_values(64), synth.normal_f32(11, n - 64, 0.0, 5.0)])
    bx, by, bz = (session.alloc(capi.FER_DTYPE_F32, [n]) for _ in range(3))
    session.upload(bx, x)
    session.wait(session.chain([(capi.FER_CHAIN_LOAD, 0, 0, 0), (op, 0, 0, 0)], [bx], by))
    getattr(ref, refname)(C.c_void_p(session.ptr_of(bx)), C.c_void_p(session.ptr_of(bz)), n,
                          C.c_void_p(session.stream()))
    y, z = np.empty(n, np.float32), np.empty(n, np.float32)
    session.download(by, y)
    session.download(bz, z)
    assert same_bits(y, z)


def test_native_launchers_vs_reference_unaligned(session):
    """ptx_tensor_* of this library against the reference's, on offsets that
    break 16-byte alignment (scalar path) and on aligned buffers."""
    ref = oracle_lib.ref_kernels()
    if ref is None:
        pytest.skip("oracle/_ref not built")
    k = capi.kernels()
    n = 4096 + 3
    x = synth.normal_f32(21, n + 1, 0.0, 4.0)
    w = synth.normal_f32(22, n + 1, 0.0, 4.0)
    bx, bw, b1, b2 = (session.alloc(capi.FER_DTYPE_F32, [n + 1]) for _ in range(4))
    session.upload(bx, x)
    session.upload(bw, w)
    st = C.c_void_p(session.stream())
    for off in (0, 1):
        px, pw = C.c_void_p(session.ptr_of(bx) + 4 * off), C.c_void_p(session.ptr_of(bw) + 4 * off)
        p1, p2 = C.c_void_p(session.ptr_of(b1) + 4 * off), C.c_void_p(session.ptr_of(b2) + 4 * off)
        m = n - off
        for name, args in [("ptx_tensor_affine_f32", (px, None, m, 1.5, -0.25)),
                           ("ptx_tensor_relu_f32", (px, None, m)), ("ptx_tensor_sigmoid_f32", (px, None, m)),
                           ("ptx_tensor_mul_f32", (px, pw, None, m)), ("ptx_tensor_add_f32", (px, pw, None, m))]:
            a1 = tuple(p1 if v is None else v for v in args)
            a2 = tuple(p2 if v is None else v for v in args)
            getattr(k, name)(*a1, st)
            getattr(ref, name)(*a2, st)
            y1, y2 = np.empty(n + 1, np.float32), np.empty(n + 1, np.float32)
            session.download(b1, y1)
            session.download(b2, y2)
            assert same_bits(y1[off:off + m], y2[off:off + m]), (name, off)


def test_reference_affine_intent_golden(session):
    """tests/c_api/test_c_api_jit_intent.cpp:41-70 of the reference."""
    n = 512
    x = (np.arange(n, dtype=np.float32) - 100.0).astype(np.float32)
    bx, by = session.alloc(capi.FER_DTYPE_F32, [n]), session.alloc(capi.FER_DTYPE_F32, [n])
    session.upload(bx, x)
    session.wait(session.affine(bx, by, n, 0.5, 10.0, capi.FER_JIT_INTENT_FUSION_RELU))
    y = np.empty(n, np.float32)
    session.download(by, y)
    expect = np.maximum(0.5 * x + 10.0, 0.0).astype(np.float32)
    assert np.max(np.abs(y - expect)) <= 1e-5
    ref = np.empty(n, np.float32)
    oracle_lib.load().orc_affine_intent_f32(oracle_lib.ptr(x), oracle_lib.ptr(ref), n, 0.5, 10.0, 1)
    assert np.array_equal(bits(y), bits(ref))


def test_affine_intent_fma_semantics(session):
    """Plain affine intent = one fused multiply-add per element (the
    reference's NVRTC build contracts alpha*in+beta), bit-exact to the oracle."""
    n = 65537
    x = synth.normal_f32(31, n, 0.0, 3.0)
    bx, by = session.alloc(capi.FER_DTYPE_F32, [n]), session.alloc(capi.FER_DTYPE_F32, [n])
    session.upload(bx, x)
    session.wait(session.affine(bx, by, n, 1.1, -0.3, 0))
    y = np.empty(n, np.float32)
    session.download(by, y)
    ref = np.empty(n, np.float32)
    oracle_lib.load().orc_affine_intent_f32(oracle_lib.ptr(x), oracle_lib.ptr(ref), n, 1.1, -0.3, 0)
    assert np.array_equal(bits(y), bits(ref))


def test_intent_contract_errors(session):
    n = 64
    bx = session.alloc(capi.FER_DTYPE_F32, [n])
    b2 = session.alloc(capi.FER_DTYPE_F32, [8, 8])
    with pytest.raises(capi.FerError) as e:
        session.affine(bx, b2, n, 1.0, 0.0, 0)
    assert e.value.code == capi.FER_STATUS_INVALID_ARGUMENT
    with pytest.raises(capi.FerError) as e:
        session.affine(bx, 999999, n, 1.0, 0.0, 0)
    assert e.value.code == capi.FER_STATUS_NOT_FOUND
    with pytest.raises(capi.FerError) as e:
        session.affine(bx, bx, 0, 1.0, 0.0, 0)
    assert e.value.code == capi.FER_STATUS_INVALID_ARGUMENT
