"""ptx_tensor_reduce_f32_noalloc: the reduction for callers that cannot
allocate device memory when they need it (allocator callbacks, processes whose
cudaMalloc is routed into the pool being managed, processes that reserved all
device memory up front). Its scratch is a fixed device array inside
libptx_kernels.so, so it must give the same bits as the allocating entry point
(the REDUCE_SUM / REDUCE_MAX JIT intents, same kernels, scratch from the
session pool) - checked here through the C ABI on two calls in a row, the
second smaller than the first so stale partials from the first call would
show. The tolerance is the one the intent tests use for this reduction:
bit-exact, since both paths run the same fixed-order kernels.

A third test checks the property the entry point exists for: after the first
call in the context (which loads its module), further calls leave the
session pool's allocation count and bytes, torch's allocator and the
driver's free-memory count unchanged.

Collected last (file name) so a run that stops at its first failure has run
everything else first; it passes alone in a fresh process too."""
import ctypes as C

import numpy as np
import pytest

from fercuda_b200 import capi, synth

pytestmark = pytest.mark.gpu

MAX_ELEMENTS = 33554432
CUDA_ERROR_INVALID_VALUE = 1


def intent_reduce(session, bx, n, is_max, start):
    bo = session.alloc(capi.FER_DTYPE_F32, [1])
    session.upload(bo, np.array([start], np.float32))
    it = capi.fer_jit_intent_t()
    it.abi_version = capi.FER_JIT_INTENT_ABI_VERSION
    it.op = capi.FER_JIT_INTENT_OP_REDUCE_MAX_F32 if is_max else capi.FER_JIT_INTENT_OP_REDUCE_SUM_F32
    it.memory_regime = capi.FER_MEMORY_AUTO
    it.n = n
    b = capi.fer_jit_intent_bindings_t(bx, bo, 0, 0)
    job = C.c_uint64()
    capi.check("fer_jit_run_intent", session.call("fer_jit_run_intent", C.byref(it), C.byref(b), C.byref(job)))
    session.wait(job.value)
    o = np.empty(1, np.float32)
    session.download(bo, o)
    session.free(bo)
    return o[0]


def noalloc_reduce(session, bx, n, is_max, start):
    bo = session.alloc(capi.FER_DTYPE_F32, [1])
    session.upload(bo, np.array([start], np.float32))
    rc = capi.kernels().ptx_tensor_reduce_f32_noalloc(C.c_void_p(session.ptr_of(bx)), C.c_void_p(session.ptr_of(bo)),
                                                      n, is_max, C.c_void_p(session.stream()))
    assert rc == 0
    o = np.empty(1, np.float32)
    session.download(bo, o)
    session.free(bo)
    return o[0]


@pytest.mark.parametrize("is_max", [0, 1])
def test_noalloc_matches_allocating_entry_point_twice(session, is_max):
    sizes = [3_000_001, 1_000]          # second call reads far fewer partials than the first wrote
    for call, n in enumerate(sizes):
        x = synth.normal_f32(70 + call, n)
        bx = session.alloc(capi.FER_DTYPE_F32, [n])
        session.upload(bx, x)
        start = -1e30 if is_max else 0.5
        got = noalloc_reduce(session, bx, n, is_max, start)
        want = intent_reduce(session, bx, n, is_max, start)
        assert np.float32(got).view(np.uint32) == np.float32(want).view(np.uint32), (call, got, want)
        ref = x.max() if is_max else 0.5 + x.astype(np.float64).sum()
        assert abs(float(got) - float(ref)) <= 1e-5 * max(1.0, float(np.abs(x).sum()))
        session.free(bx)


def test_noalloc_rejects_sizes_beyond_the_maximum(session):
    bx = session.alloc(capi.FER_DTYPE_F32, [16])
    bo = session.alloc(capi.FER_DTYPE_F32, [1])
    rc = capi.kernels().ptx_tensor_reduce_f32_noalloc(C.c_void_p(session.ptr_of(bx)), C.c_void_p(session.ptr_of(bo)),
                                                      MAX_ELEMENTS + 1, 0, C.c_void_p(session.stream()))
    assert rc == CUDA_ERROR_INVALID_VALUE
    session.free(bx)
    session.free(bo)


def pool_stats(session):
    st = capi.fer_pool_stats_t()
    capi.check("fer_pool_get_stats", session.call("fer_pool_get_stats", C.byref(st)))
    return (st.allocated_bytes, st.total_allocations, st.total_frees, st.allocated_blocks)


def test_noalloc_calls_allocate_nothing(session):
    import torch

    n = 2_000_003
    x = synth.normal_f32(80, n)
    bx = session.alloc(capi.FER_DTYPE_F32, [n])
    bo = session.alloc(capi.FER_DTYPE_F32, [1])
    session.upload(bx, x)
    args = (C.c_void_p(session.ptr_of(bx)), C.c_void_p(session.ptr_of(bo)), n, 0, C.c_void_p(session.stream()))
    assert capi.kernels().ptx_tensor_reduce_f32_noalloc(*args) == 0      # set-up call
    torch.cuda.synchronize()
    before = (pool_stats(session), torch.cuda.memory_allocated(), torch.cuda.memory_reserved(),
              torch.cuda.mem_get_info()[0])
    for is_max in (0, 1, 0, 1):
        a = args[:3] + (is_max,) + args[4:]
        assert capi.kernels().ptx_tensor_reduce_f32_noalloc(*a) == 0
    torch.cuda.synchronize()
    after = (pool_stats(session), torch.cuda.memory_allocated(), torch.cuda.memory_reserved(),
             torch.cuda.mem_get_info()[0])
    assert after == before
    session.free(bx)
    session.free(bo)
