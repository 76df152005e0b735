"""Split-K tensor-core GEMM (fer_gemm_bf16_tc_splitk), the decode-step GEMM.

Against fer_gemm_bf16_tc_ex on the same operands: with one split the bits are
the same (same accumulation, same epilogue arithmetic); with several splits
the K-range partials are added in range order, so the result differs from
the single chain only by rounding: f32 outputs within 1e-5 of max |C|,
bf16 outputs within one bf16 step (4e-3 relative) of it. Every run gives the
same bits. Shapes cover M = 1 .. 200 (one and two 128-row tiles), ragged N and
K (multiples of 8), and all four epilogues.
"""
import ctypes as C

import pytest
import torch

from fercuda_b200 import capi

pytestmark = pytest.mark.gpu

P = C.c_void_p


def lib():
    k = capi.kernels()
    k.fer_gemm_bf16_tc_ex.argtypes = [P, P, P, P] + [C.c_int] * 4 + [P, P]
    k.fer_gemm_bf16_tc_ex.restype = C.c_int
    k.fer_gemm_bf16_tc_splitk.argtypes = [P, P, P] + [C.c_int] * 5 + [P, C.c_size_t, C.c_int, P, P]
    k.fer_gemm_bf16_tc_splitk.restype = C.c_int
    k.fer_gemm_splitk_workspace_bytes.argtypes = [C.c_int] * 3
    k.fer_gemm_splitk_workspace_bytes.restype = C.c_size_t
    k.fer_gemm_splitk_cluster_splits.argtypes = [C.c_int] * 3
    k.fer_gemm_splitk_cluster_splits.restype = C.c_int
    return k


def operands(M, N, K, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    a = (torch.randn(M, K, generator=g, device="cuda") / K ** 0.25).bfloat16()
    b = (torch.randn(K, N, generator=g, device="cuda") / K ** 0.25).bfloat16()
    x = torch.randn(M, N, generator=g, device="cuda")
    return a, b, x


def run(k, fn, a, b, M, N, K, epi, x, splits=0, ws_bytes=None, flags=0):
    f32 = epi in (0, 3)
    c = x.clone() if epi == 3 else torch.full((M, N), float("nan"), device="cuda",
                                             dtype=torch.float32 if f32 else torch.bfloat16)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    if fn == "ex":
        rc = k.fer_gemm_bf16_tc_ex(a.data_ptr(), b.data_ptr(), c.data_ptr(), c.data_ptr() if epi == 3 else None,
                                   M, N, K, epi, err.data_ptr(), st)
    else:
        nbytes = ws_bytes if ws_bytes is not None else k.fer_gemm_splitk_workspace_bytes(M, N, K)
        if splits > 0:
            nbytes = max(nbytes, splits * ((M + 127) // 128) * 128 * N * 4)
        ws = torch.empty(max(nbytes // 4, 4), device="cuda")
        rc = k.fer_gemm_bf16_tc_splitk(a.data_ptr(), b.data_ptr(), c.data_ptr(), M, N, K, epi, splits,
                                       ws.data_ptr(), nbytes, flags, err.data_ptr(), st)
    assert rc == 0
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return c


def bits(t):
    return t.view(torch.int32) if t.dtype == torch.float32 else t.view(torch.int16)


@pytest.mark.parametrize("M,N,K", [(1, 256, 64), (7, 1000, 1024), (64, 1024, 1024), (64, 4096, 1024),
                                   (64, 1024, 4096), (128, 3072, 1024), (200, 512, 520), (64, 32000, 1024)])
@pytest.mark.parametrize("epi", [0, 1, 2, 3])
def test_splitk_vs_single_chain(M, N, K, epi):
    k = lib()
    a, b, x = operands(M, N, K, seed=M * 7 + N + K)
    want = run(k, "ex", a, b, M, N, K, epi, x)
    got = run(k, "splitk", a, b, M, N, K, epi, x)
    again = run(k, "splitk", a, b, M, N, K, epi, x)
    assert torch.equal(bits(got), bits(again))
    one = run(k, "splitk", a, b, M, N, K, epi, x, splits=1)
    assert torch.equal(bits(one), bits(want))
    # static weights (B fetched before the launch wait): same bits
    assert torch.equal(bits(run(k, "splitk", a, b, M, N, K, epi, x, flags=1)), bits(got))
    tol = 1e-5 if epi in (0, 3) else 4e-3
    err = (got.float() - want.float()).abs().max() / want.float().abs().max()
    assert float(err) <= tol, float(err)


@pytest.mark.parametrize("M,N,K", [(1, 256, 64), (7, 1000, 1024), (64, 1024, 1024), (64, 3072, 1024),
                                   (64, 4096, 1024), (64, 1024, 4096), (200, 512, 520), (128, 2048, 2048)])
@pytest.mark.parametrize("epi", [0, 1, 2, 3])
def test_cluster_form_equals_workspace_form(M, N, K, epi):
    k = lib()
    S = k.fer_gemm_splitk_cluster_splits(M, N, K)
    assert S >= 1
    a, b, x = operands(M, N, K, seed=M + 3 * N + K)
    got = run(k, "splitk", a, b, M, N, K, epi, x)
    if S == 1:
        want = run(k, "ex", a, b, M, N, K, epi, x)
    else:
        want = run(k, "splitk", a, b, M, N, K, epi, x, splits=S)
    assert torch.equal(bits(got), bits(want)), S


def test_cluster_plan_uses_large_clusters_for_decode_shapes():
    k = lib()
    num_k = lambda K: (K + 63) // 64
    for N, K in [(1024, 1024), (3072, 1024), (4096, 1024), (1024, 4096)]:
        S = k.fer_gemm_splitk_cluster_splits(64, N, K)
        assert 2 <= S <= min(16, num_k(K)), (N, K, S)
    assert k.fer_gemm_splitk_cluster_splits(64, 32000, 1024) == 1     # 125 tiles: no split


def test_splits_shrink_to_the_workspace():
    k = lib()
    M, N, K = 64, 2048, 4096
    a, b, x = operands(M, N, K, seed=3)
    want = run(k, "ex", a, b, M, N, K, 0, x)
    small = 3 * 128 * N * 4                    # room for three splits only
    got = run(k, "splitk", a, b, M, N, K, 0, x, splits=64, ws_bytes=small)
    assert float((got - want).abs().max() / want.abs().max()) <= 1e-5
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    c = torch.empty(M, N, device="cuda")
    ws = torch.empty(16, device="cuda")
    # the workspace form (explicit count) refuses a workspace too small for one split
    assert k.fer_gemm_bf16_tc_splitk(a.data_ptr(), b.data_ptr(), c.data_ptr(), M, N, K, 0, 5, ws.data_ptr(), 64, 0,
                                     err.data_ptr(), torch.cuda.current_stream().cuda_stream) != 0
