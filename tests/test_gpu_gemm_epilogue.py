"""Epilogues of the tcgen05 GEMM (fer_gemm_bf16_tc_ex) on the GPU.

The transformer forward uses four output forms: f32, bf16, exact-GELU bf16
and f32 plus a residual (in place, through a TMA reduce-add, or from a
separate residual buffer, copied first). Each is checked against a float64
product of the same bf16 operands, on shapes whose edges cut the 128 x 256
tile and the 32-row x 128-byte output boxes.

Tolerance: products of bf16 values are exact in f32, so f32 outputs differ
from float64 only by summation order (REL = 1e-4 of max |reference|); bf16
outputs are compared after rounding the reference to bf16 and may differ by
one bf16 unit where the f32 sums straddle a rounding boundary, plus the same
REL * max |reference| absolute term (near-zero outputs, where summation order
moves the value by more than a bf16 unit of the tiny result).
"""
import ctypes as C

import numpy as np
import pytest
import torch
from scipy.special import erf

from fercuda_b200 import capi, synth

pytestmark = pytest.mark.gpu

REL = 1e-4
EPI_F32, EPI_BF16, EPI_GELU, EPI_RESID = 0, 1, 2, 3


def kern():
    k = capi.kernels()
    k.fer_gemm_bf16_tc_ex.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int,
                                      C.c_int, C.c_void_p, C.c_void_p]
    k.fer_gemm_bf16_tc_ex.restype = C.c_int
    return k


def operands(m, n, k, seed):
    a = synth.normal_bf16(seed, m * k, 0.0, 1.0 / np.sqrt(k)).reshape(m, k)
    b = synth.normal_bf16(seed + 1, k * n, 0.0, 1.0).reshape(k, n)
    return a, b


def f64(bits):
    return synth.bf16_bits_to_f32(bits).astype(np.float64)


def bf16_round(x):
    return synth.bf16_bits_to_f32(synth.f32_to_bf16_bits(np.asarray(x, np.float32)))


def launch(a, b, out, resid, m, n, k, epi):
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ta = torch.from_numpy(a.view(np.int16)).cuda()
    tb = torch.from_numpy(b.view(np.int16)).cuda()
    rc = kern().fer_gemm_bf16_tc_ex(ta.data_ptr(), tb.data_ptr(), out.data_ptr(),
                                    resid.data_ptr() if resid is not None else None, m, n, k, epi,
                                    err.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return out


@pytest.mark.parametrize("m,n,k", [(300, 200, 192), (128, 256, 64), (517, 648, 1000), (64, 40, 8)])
def test_f32_and_bf16_outputs(m, n, k):
    a, b = operands(m, n, k, 11)
    ref = f64(a) @ f64(b)
    y = launch(a, b, torch.empty(m, n, dtype=torch.float32, device="cuda"), None, m, n, k, EPI_F32).cpu().numpy()
    assert np.abs(y - ref).max() <= REL * np.abs(ref).max()
    yb = launch(a, b, torch.empty(m, n, dtype=torch.bfloat16, device="cuda"), None, m, n, k, EPI_BF16)
    yb = yb.float().cpu().numpy()
    rb = bf16_round(ref)
    tol = np.abs(rb) * 2.0 ** -7 + REL * np.abs(ref).max()
    assert (np.abs(yb - rb) <= tol).all()


@pytest.mark.parametrize("m,n,k", [(300, 520, 256), (256, 4096, 1024)])
def test_gelu_bf16_output(m, n, k):
    a, b = operands(m, n, k, 21)
    ref = f64(a) @ f64(b)
    g = 0.5 * ref * (1.0 + erf(ref / np.sqrt(2.0)))
    y = launch(a, b, torch.empty(m, n, dtype=torch.bfloat16, device="cuda"), None, m, n, k, EPI_GELU)
    y = y.float().cpu().numpy()
    rb = bf16_round(g)
    assert (np.abs(y - rb) <= np.abs(rb) * 2.0 ** -7 + REL * np.abs(g).max()).all()


@pytest.mark.parametrize("m,n,k", [(300, 200, 192), (1024, 1024, 1024)])
def test_residual_in_place_and_from_other_buffer(m, n, k):
    a, b = operands(m, n, k, 31)
    x0 = synth.normal_f32(41, m * n).reshape(m, n)
    ref = x0.astype(np.float64) + f64(a) @ f64(b)
    x = torch.from_numpy(x0.copy()).cuda()
    y = launch(a, b, x, x, m, n, k, EPI_RESID).cpu().numpy()                # x += A.B in place
    assert np.abs(y - ref).max() <= REL * np.abs(ref).max()
    r = torch.from_numpy(x0.copy()).cuda()
    out = torch.full((m, n), 7.0, dtype=torch.float32, device="cuda")
    y2 = launch(a, b, out, r, m, n, k, EPI_RESID).cpu().numpy()            # out = r + A.B
    assert np.array_equal(y.view(np.uint32), y2.view(np.uint32))
    assert np.array_equal(r.cpu().numpy(), x0)                               # residual untouched


def test_residual_equals_f32_plus_add_bitwise():
    """The in-place reduce adds each element once: x + acc exactly as f32."""
    m, n, k = 384, 512, 320
    a, b = operands(m, n, k, 51)
    acc = launch(a, b, torch.empty(m, n, dtype=torch.float32, device="cuda"), None, m, n, k, EPI_F32)
    x0 = torch.from_numpy(synth.normal_f32(52, m * n).reshape(m, n)).cuda()
    x = x0.clone()
    launch(a, b, x, x, m, n, k, EPI_RESID)
    assert torch.equal(x, x0 + acc)


def test_partial_overlap_rejected():
    m, n, k = 128, 256, 64
    a, b = operands(m, n, k, 61)
    buf = torch.zeros(2 * m * n, dtype=torch.float32, device="cuda")
    ta = torch.from_numpy(a.view(np.int16)).cuda()
    tb = torch.from_numpy(b.view(np.int16)).cuda()
    rc = kern().fer_gemm_bf16_tc_ex(ta.data_ptr(), tb.data_ptr(), buf.data_ptr(), buf[256:].data_ptr(), m, n, k,
                                    EPI_RESID, None, torch.cuda.current_stream().cuda_stream)
    assert rc != 0


@pytest.mark.parametrize("m,n,k,epi", [(300, 200, 192, EPI_F32), (1024, 3072, 1024, EPI_BF16), (517, 648, 1000, EPI_GELU),
                                       (640, 1024, 4096, EPI_RESID), (129, 256, 64, EPI_F32)])
def test_two_cta_kernel_matches_single_cta_kernel(m, n, k, epi):
    """The default 2-CTA cluster kernel (M > 128) against the single-CTA
    kernel on the same operands: same K order per output, so the same bits."""
    a, b = operands(m, n, k, 71)
    dt = torch.float32 if epi in (EPI_F32, EPI_RESID) else torch.bfloat16
    x0 = torch.from_numpy(synth.normal_f32(72, m * n).reshape(m, n)).cuda()
    outs = []
    k_ = kern()
    k_.fer_gemm_tc_set_mode.argtypes = [C.c_int]
    try:
        for mode in (0, 1):
            k_.fer_gemm_tc_set_mode(mode)
            out = x0.clone() if epi == EPI_RESID else torch.empty(m, n, dtype=dt, device="cuda")
            outs.append(launch(a, b, out, out if epi == EPI_RESID else None, m, n, k, epi))
    finally:
        k_.fer_gemm_tc_set_mode(0)
    ref = f64(a) @ f64(b) + (x0.double().cpu().numpy() if epi == EPI_RESID else 0.0)
    if epi == EPI_GELU:
        ref = 0.5 * ref * (1.0 + erf(ref / np.sqrt(2.0)))
    y = outs[0].float().cpu().numpy()
    assert np.abs(y - ref).max() <= (2.0 ** -7 if dt == torch.bfloat16 else REL) * np.abs(ref).max() + REL
    assert torch.equal(outs[0], outs[1])
