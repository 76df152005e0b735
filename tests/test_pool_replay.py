"""The allocation-trace replay harness (libfercuda_bench.so) on CPU.

fer_bench_fn_replay drives any allocator given as a pair of C function
pointers; here it replays a prefix of the TLSF stress trace (1M-op workload,
seed 2) through this package's TLSF and, when it was built from its sources,
the reference TLSF, both host-only over the same fake 80 GiB range. Both must
complete the same trace with the same number of allocations and frees, and
hand out identical addresses (checked through a recording wrapper).
"""
import ctypes as C

import numpy as np
import pytest

from fercuda_b200 import capi, synth
from tests import oracle_lib

BASE = 1 << 40
POOL = 80 << 30
ALLOC_FN = C.CFUNCTYPE(C.c_void_p, C.c_void_p, C.c_size_t)
FREE_FN = C.CFUNCTYPE(None, C.c_void_p, C.c_void_p)


def bench_lib():
    lib = C.CDLL(str(capi.LIBDIR / "libfercuda_bench.so"))
    lib.fer_bench_fn_replay.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p,
                                        C.POINTER(C.c_size_t), C.c_void_p, C.POINTER(C.c_size_t),
                                        C.POINTER(C.c_double)]
    lib.fer_bench_fn_replay.restype = C.c_int
    return lib


def replay(tlsf_lib, trace):
    """Replays `trace`; returns (rc, n_alloc, n_free, addresses in alloc order)."""
    tlsf_lib.ptx_tlsf_create_from_pool.restype = C.c_void_p
    tlsf_lib.ptx_tlsf_create_from_pool.argtypes = [C.c_void_p, C.c_size_t, C.c_bool]
    tlsf_lib.ptx_tlsf_alloc.restype = C.c_void_p
    tlsf_lib.ptx_tlsf_alloc.argtypes = [C.c_void_p, C.c_size_t]
    tlsf_lib.ptx_tlsf_free.argtypes = [C.c_void_p, C.c_void_p]
    tlsf_lib.ptx_tlsf_destroy.argtypes = [C.c_void_p]
    tlsf_lib.ptx_tlsf_set_warnings_enabled.argtypes = [C.c_void_p, C.c_bool]
    h = tlsf_lib.ptx_tlsf_create_from_pool(C.c_void_p(BASE), POOL, False)
    assert h
    tlsf_lib.ptx_tlsf_set_warnings_enabled(h, False)
    seen = []

    @ALLOC_FN
    def alloc(ctx, n):
        p = tlsf_lib.ptx_tlsf_alloc(ctx, n)
        seen.append(p or 0)
        return p

    @FREE_FN
    def free(ctx, p):
        tlsf_lib.ptx_tlsf_free(ctx, p)

    tr = np.ascontiguousarray(trace, np.int64)
    na_max = int((tr > 0).sum())
    an = np.zeros(max(1, na_max), np.uint32)
    fn = np.zeros(max(1, len(tr) - na_max), np.uint32)
    na, nf, wall = C.c_size_t(), C.c_size_t(), C.c_double()
    rc = bench_lib().fer_bench_fn_replay(C.cast(alloc, C.c_void_p), C.cast(free, C.c_void_p), C.c_void_p(h),
                                         tr.ctypes.data_as(C.c_void_p), len(tr), an.ctypes.data_as(C.c_void_p),
                                         C.byref(na), fn.ctypes.data_as(C.c_void_p), C.byref(nf), C.byref(wall))
    tlsf_lib.ptx_tlsf_destroy(h)
    assert wall.value > 0
    return rc, na.value, nf.value, seen


@pytest.fixture(scope="module")
def trace():
    return synth.tlsf_trace(ops=20_000)


def test_replay_through_this_tlsf(trace):
    rc, na, nf, seen = replay(capi.core(), trace)
    assert rc == 0
    assert na == int((trace > 0).sum()) and nf == len(trace) - na
    assert all(BASE <= p < BASE + POOL and (p - BASE) % 256 == 0 for p in seen)


def test_replay_matches_reference_tlsf(trace):
    ref = oracle_lib.ref_tlsf()
    if ref is None:
        pytest.skip("reference TLSF not built (oracle/_ref)")
    ours = replay(capi.core(), trace)
    theirs = replay(ref, trace)
    assert ours[:3] == theirs[:3]
    assert ours[3] == theirs[3]
