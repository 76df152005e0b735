"""TLSF allocator (libptx_core.so, host bookkeeping) on CPU: same addresses as
the reference allocator (oracle/_ref, compiled from the reference source) and
as the oracle restatement on the seeded stress traces, structural validity,
and the reference's own allocator test restated."""
import ctypes as C

import numpy as np
import pytest

from fercuda_b200 import capi, synth
from tests import oracle_lib

BASE = 1 << 40
P = C.c_void_p


def replay(trace, pool_size):
    """Replays one trace through ours, the oracle and (if built) the
    reference; returns the three address lists (None when not built)."""
    core = capi.core()
    orc = oracle_lib.load()
    ref = oracle_lib.ref_tlsf()
    a = core.ptx_tlsf_create_from_pool(P(BASE), pool_size, False)
    c = orc.orc_tlsf_create(pool_size)
    b = ref.ptx_tlsf_create_from_pool(P(BASE), pool_size, False) if ref else None
    pa, pb, pc = [], [], []
    for e in trace.tolist():
        if e > 0:
            pa.append(core.ptx_tlsf_alloc(a, e) or 0)
            z = orc.orc_tlsf_alloc(c, e)
            pc.append(0 if z == 2 ** 64 - 1 else z + BASE)
            if b:
                pb.append(ref.ptx_tlsf_alloc(b, e) or 0)
        else:
            k = -e - 1
            if pa[k]:
                core.ptx_tlsf_free(a, P(pa[k]))
            if pc[k]:
                orc.orc_tlsf_free(c, pc[k] - BASE)
            if b and pb[k]:
                ref.ptx_tlsf_free(b, P(pb[k]))
    rep = capi.TLSFHealthReport()
    core.ptx_tlsf_validate(a, C.byref(rep))
    stats = capi.TLSFPoolStats()
    core.ptx_tlsf_get_stats(a, C.byref(stats))
    core.ptx_tlsf_destroy(a)
    orc.orc_tlsf_destroy(c)
    if b:
        ref.ptx_tlsf_destroy(b)
    return pa, (pb if b else None), pc, rep, stats


def test_config_trace_full_size_same_addresses():
    """Full stress trace: 1,000,000 ops, seed 2, 256 B - 16 MiB log-uniform,
    60/40, live <= 64 GiB, over an 80 GiB range."""
    trace = synth.tlsf_trace()
    pa, pb, pc, rep, stats = replay(trace, 80 << 30)
    assert all(pa), "an allocation failed in an 80 GiB pool"
    assert pa == pc
    if pb is not None:
        assert pa == pb
    assert rep.is_valid, [m.value for m in rep.error_messages[: rep.error_count]]
    assert stats.total_allocations == len(pa)


@pytest.mark.parametrize("seed,cap,pool", [(7, 1 << 30, (1 << 30) + 4096), (8, 256 << 20, 300 << 20),
                                           (9, 8 << 30, 9 << 30)])
def test_pressure_traces_same_addresses_and_failures(seed, cap, pool):
    """Tight pools: allocations fail (NULL) at the same ops as the reference."""
    trace = synth.tlsf_trace(ops=60000, seed=seed, live_cap=cap)
    pa, pb, pc, rep, _ = replay(trace, pool)
    assert pa == pc
    if pb is not None:
        assert pa == pb
    assert rep.is_valid


def test_giant_blocks_clamped_class():
    """Blocks >= 16 GiB land in the clamped top size class, whose lists the
    reference searches head by head; the decisions must still agree."""
    sizes = [20 << 30, 9 << 30, 17 << 30, 1 << 20, 33 << 30, 12 << 30]
    trace = np.array(sizes + [-1, -3, 40 << 30, 18 << 30, -2, 24 << 30], np.int64)
    pa, pb, pc, rep, _ = replay(trace, (100 << 30) + 12345)
    assert pa == pc
    if pb is not None:
        assert pa == pb
    assert rep.is_valid


def test_reference_tlsf_unit_test_restated():
    """tests/native/test_ptx_tlsf.cpp:23-82 of the reference, over a fake range."""
    core = capi.core()
    a = core.ptx_tlsf_create_from_pool(P(BASE), 32 << 20, True)
    p1 = core.ptx_tlsf_alloc(a, 4096)
    assert p1 and core.ptx_tlsf_owns_ptr(a, P(p1))
    ptrs = [core.ptx_tlsf_alloc(a, 1024 * (i + 1)) for i in range(100)]
    assert all(ptrs)
    st = capi.TLSFPoolStats()
    core.ptx_tlsf_get_stats(a, C.byref(st))
    assert st.allocated_blocks >= 101 and st.total_allocations >= 101
    core.ptx_tlsf_free(a, P(p1))
    for p in ptrs:
        core.ptx_tlsf_free(a, P(p))
    rep = capi.TLSFHealthReport()
    core.ptx_tlsf_validate(a, C.byref(rep))
    assert rep.is_valid and not rep.has_memory_leaks
    core.ptx_tlsf_get_stats(a, C.byref(st))
    assert st.allocated_bytes == 0 and st.free_blocks == 1 and st.largest_free_block == 32 << 20
    o1 = core.ptx_tlsf_alloc_owned(a, 8192, 42)
    o2 = core.ptx_tlsf_alloc_owned(a, 16384, 42)
    assert o1 and o2

    # TLSFOwnerUsage is {u32 id; size_t bytes; u32 count} = 24 bytes with padding
    buf = (C.c_uint8 * (24 * 64 + 8))()
    core.ptx_tlsf_get_owner_stats(a, buf)
    raw = bytes(buf)
    assert int.from_bytes(raw[0:4], "little") == 42
    assert int.from_bytes(raw[8:16], "little") == 8192 + 16384
    assert int.from_bytes(raw[16:20], "little") == 2
    core.ptx_tlsf_free_owner(a, 42)
    core.ptx_tlsf_get_stats(a, C.byref(st))
    assert st.allocated_bytes == 0
    core.ptx_tlsf_defragment(a)
    core.ptx_tlsf_destroy(a)


def test_edge_cases():
    core = capi.core()
    a = core.ptx_tlsf_create_from_pool(P(BASE), 10000, False)   # not a multiple of 256
    assert core.ptx_tlsf_alloc(a, 0) is None
    p = core.ptx_tlsf_alloc(a, 1)
    assert p == BASE
    q = core.ptx_tlsf_alloc(a, 9000)      # 9216 bytes of the 9744 left
    assert q == BASE + 256
    assert core.ptx_tlsf_alloc(a, 1024) is None
    core.ptx_tlsf_free(a, P(p))
    core.ptx_tlsf_free(a, P(p))           # double free: ignored
    core.ptx_tlsf_free(a, P(q))
    core.ptx_tlsf_free(a, P(BASE + 12))   # foreign pointer: ignored
    core.ptx_tlsf_free(a, P(123))         # outside the pool: ignored
    rep = capi.TLSFHealthReport()
    core.ptx_tlsf_validate(a, C.byref(rep))
    assert rep.is_valid
    assert core.ptx_tlsf_alloc(a, 10000) is None      # rounds to 10240 > pool
    assert core.ptx_tlsf_alloc(a, 9984) == BASE       # exact fit of 39 * 256 in 10000
    core.ptx_tlsf_destroy(a)


def test_oracle_restatement_matches_reference_small():
    ref = oracle_lib.ref_tlsf()
    if ref is None:
        pytest.skip("oracle/_ref not built")
    trace = synth.tlsf_trace(ops=20000, seed=3, live_cap=2 << 30)
    pa, pb, pc, _, _ = replay(trace, 3 << 30)
    assert pb == pc
