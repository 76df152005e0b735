"""Deterministic tcgen05 GEMM (fer_submit_gemm) on the GPU through the C ABI.

Tolerance: the required bound for bf16-in / f32-accumulate GEMM is a max
relative error <= 2e-2 (normalised by max |reference|); products of bf16
values are exact in f32, so the only difference to the reference's
sequential-FMA chain is summation order, and the tests also hold the much
tighter empirical bound REL = 1e-4 to catch descriptor or layout mistakes."""
import ctypes as C

import numpy as np
import pytest

from fercuda_b200 import capi, synth
from tests import oracle_lib

pytestmark = pytest.mark.gpu

REQUIRED_TOL = 2e-2
REL = 1e-4


def run_gemm(session, a_bits, b_bits, out_dtype=capi.FER_DTYPE_F32):
    m, k = a_bits.shape
    n = b_bits.shape[1]
    ba = session.alloc(capi.FER_DTYPE_BF16, [m, k])
    bb = session.alloc(capi.FER_DTYPE_BF16, [k, n])
    bo = session.alloc(out_dtype, [m, n])
    session.upload(ba, np.ascontiguousarray(a_bits))
    session.upload(bb, np.ascontiguousarray(b_bits))
    session.wait(session.gemm(ba, bb, bo))
    out = np.empty((m, n), np.float32 if out_dtype == capi.FER_DTYPE_F32 else np.uint16)
    session.download(bo, out)
    assert session.device_errors() == 0
    return (ba, bb, bo), out


def rel_err(y, ref):
    return float(np.abs(y.astype(np.float64) - ref).max() / max(np.abs(ref).max(), 1e-30))


@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (128, 256, 512), (256, 512, 128), (300, 520, 200),
                                   (1, 8, 8), (129, 264, 72), (1024, 1024, 1024)])
def test_gemm_vs_float64(session, m, n, k):
    a, b = synth.gemm_inputs(m, n, k)
    bufs, y = run_gemm(session, a, b)
    ref = synth.bf16_bits_to_f32(a).astype(np.float64) @ synth.bf16_bits_to_f32(b).astype(np.float64)
    err = rel_err(y, ref)
    assert err <= REQUIRED_TOL
    assert err <= REL, err
    for x in bufs:
        session.free(x)


def test_gemm_bf16_output(session):
    m, n, k = 256, 512, 256
    a, b = synth.gemm_inputs(m, n, k)
    bufs, y32 = run_gemm(session, a, b)
    bufs2, y16 = run_gemm(session, a, b, capi.FER_DTYPE_BF16)
    assert np.array_equal(y16, synth.f32_to_bf16_bits(y32))
    for x in bufs + bufs2:
        session.free(x)


def test_gemm_deterministic_and_unaligned_fallback(session):
    m, n, k = 384, 768, 640
    a, b = synth.gemm_inputs(m, n, k)
    ba, bb, bo = (session.alloc(capi.FER_DTYPE_BF16, [m, k]), session.alloc(capi.FER_DTYPE_BF16, [k, n]),
                  session.alloc(capi.FER_DTYPE_F32, [m, n]))
    session.upload(ba, a)
    session.upload(bb, b)
    first = None
    for _ in range(10):
        session.wait(session.gemm(ba, bb, bo))
        y = np.empty((m, n), np.float32)
        session.download(bo, y)
        if first is None:
            first = y
        assert np.array_equal(y.view(np.uint32), first.view(np.uint32))
    # K not a multiple of 8: CUDA-core path with the reference's chain order,
    # bit-exact to the oracle's sequential fmaf
    a2, b2 = synth.gemm_inputs(37, 45, 29)
    _, y2 = run_gemm(session, a2, b2)
    ref2 = np.empty((37, 45), np.float32)
    oracle_lib.load().orc_matmul_bf16_tile(oracle_lib.ptr(a2), oracle_lib.ptr(b2), oracle_lib.ptr(ref2), 37, 29, 45,
                                           0, 37, 0, 45)
    assert np.array_equal(y2.view(np.uint32), ref2.view(np.uint32))


def test_gemm_full_size_sampled_tiles_vs_oracle(session):
    """8192^3 (the deterministic-GEMM workload): 4 sampled 64x64 output tiles
    against the reference's sequential-fmaf chain (oracle), plus a checksum of
    row sums against a float64 A.(B.1) product."""
    a, b = synth.gemm_inputs()
    m, k = a.shape
    n = b.shape[1]
    bufs, y = run_gemm(session, a, b)
    orc = oracle_lib.load()
    for (r0, c0) in [(0, 0), (4096, 8128), (8128, 256), (1000, 5000)]:
        ref = np.empty((64, 64), np.float32)
        orc.orc_matmul_bf16_tile(oracle_lib.ptr(a), oracle_lib.ptr(b), oracle_lib.ptr(ref), m, k, n, r0, r0 + 64, c0,
                                 c0 + 64)
        err = rel_err(y[r0:r0 + 64, c0:c0 + 64], ref.astype(np.float64))
        assert err <= REL, (r0, c0, err)
    bsum = synth.bf16_bits_to_f32(b).astype(np.float64).sum(axis=1)
    rowsum_ref = synth.bf16_bits_to_f32(a).astype(np.float64) @ bsum
    rowsum = y.astype(np.float64).sum(axis=1)
    assert np.abs(rowsum - rowsum_ref).max() <= 1e-3 * np.abs(rowsum_ref).max()
    for x in bufs:
        session.free(x)


def test_gemm_argument_errors(session):
    ba = session.alloc(capi.FER_DTYPE_F32, [16, 16])
    bb = session.alloc(capi.FER_DTYPE_BF16, [16, 16])
    bo = session.alloc(capi.FER_DTYPE_F32, [16, 16])
    with pytest.raises(capi.FerError) as e:
        session.gemm(ba, bb, bo)
    assert e.value.code == capi.FER_STATUS_INVALID_ARGUMENT
    b2 = session.alloc(capi.FER_DTYPE_BF16, [16, 8])
    bx = session.alloc(capi.FER_DTYPE_BF16, [16, 16])
    with pytest.raises(capi.FerError) as e:
        session.gemm(bx, b2, bo)
    assert e.value.code == capi.FER_STATUS_INVALID_ARGUMENT


def test_gemm_8192_full_matrix_vs_reference_kernel():
    """The configured GEMM (8192^3, bf16 operands N(0, 1/sqrt(K)) from seed 3,
    made by the device generator as the benchmark does) against the
    reference's own GEMM kernel (k_matmul_f32 through fer::ops::matmul,
    src/runtime/ops_bridge.cu:13-31, built from the reference sources) run on
    the same operands upcast to f32: every one of the 67M outputs, not a
    sample. The reference kernel's sequential fmaf chain and the tensor-core
    accumulation differ only in summation order."""
    import torch

    ref = oracle_lib.ref_kernels()
    assert ref is not None, "oracle/_ref/libref_kernels.so missing (build() compiles it)"
    n = 8192
    ab = torch.empty(2 * n * n, dtype=torch.int16, device="cuda")
    rc = capi.kernels().fer_fill_normal_bf16(C.c_void_p(ab.data_ptr()), 2 * n * n, synth.GEMM["seed"],
                                             C.c_float(1.0 / np.sqrt(n)), None)
    assert rc == 0
    a_bits, b_bits = ab[: n * n], ab[n * n:]
    ours = torch.empty(n * n, dtype=torch.float32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    k = capi.kernels()
    k.fer_gemm_bf16_tc_ex.argtypes = [C.c_void_p] * 4 + [C.c_int] * 4 + [C.c_void_p, C.c_void_p]
    k.fer_gemm_bf16_tc_ex.restype = C.c_int
    assert k.fer_gemm_bf16_tc_ex(a_bits.data_ptr(), b_bits.data_ptr(), ours.data_ptr(), None, n, n, n, 0,
                                 err.data_ptr(), None) == 0
    af = a_bits.view(torch.bfloat16).float()
    bf = b_bits.view(torch.bfloat16).float()
    theirs = torch.empty(n * n, dtype=torch.float32, device="cuda")
    ref.refshim_matmul_f32(C.c_void_p(af.data_ptr()), C.c_void_p(bf.data_ptr()), C.c_void_p(theirs.data_ptr()),
                           n, n, n, None)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.isfinite(ours).all()
    e = float((ours.double() - theirs.double()).abs().max() / theirs.double().abs().max())
    assert e <= REQUIRED_TOL
    assert e <= REL, e
