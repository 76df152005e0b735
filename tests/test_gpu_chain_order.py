"""Back-to-back chain calls keep stream order.

fer_tensor_run_affine_f32 launches its kernel with programmatic dependent
launch and, when the previous chain kernel on the stream cannot conflict,
lets the new kernel read (and, with no shared buffer at all, write) before
that kernel has finished. These tests issue long runs of calls with no host
synchronisation in between, mixing read-after-write, write-after-read,
write-after-write and independent pairs (and interleaved GEMM submissions
from the same session), and compare every buffer with a numpy replay of the
same calls. The affine steps use alpha in {1, -1, 0.5} on values that keep
alpha * x exact, so the fused multiply-add equals numpy's float32 result.
"""
import numpy as np
import pytest

from fercuda_b200 import capi

pytestmark = pytest.mark.gpu

N = 1 << 20


def run_sequence(session, steps, seed, n_buf=5, with_gemm=False):
    rng = np.random.default_rng(seed)
    host = [np.round(rng.uniform(-8, 8, N)).astype(np.float32) for _ in range(n_buf)]
    ids = [session.alloc(capi.FER_DTYPE_F32, [N]) for _ in range(n_buf)]
    for b, h in zip(ids, host):
        session.upload(b, h)
    if with_gemm:
        ga = session.alloc(capi.FER_DTYPE_BF16, [128, 128])
        gb = session.alloc(capi.FER_DTYPE_BF16, [128, 128])
        gc = session.alloc(capi.FER_DTYPE_F32, [128, 128])
        session.upload(ga, np.zeros((128, 128), np.uint16))
        session.upload(gb, np.zeros((128, 128), np.uint16))
    last = 0
    for k in range(steps):
        src, dst = rng.integers(0, n_buf, 2)
        alpha = float(rng.choice([1.0, -1.0, 0.5]))
        beta = float(rng.integers(-3, 4))
        last = session.affine(ids[src], ids[dst], N, alpha, beta, 0)
        host[dst] = (np.float32(alpha) * host[src] + np.float32(beta)).astype(np.float32)
        if with_gemm and k % 7 == 3:
            session.gemm(ga, gb, gc)
    session.wait(last)
    for b, h in zip(ids, host):
        got = np.empty(N, np.float32)
        session.download(b, got)
        assert np.array_equal(got, h)
    for b in ids:
        session.free(b)
    if with_gemm:
        for b in (ga, gb, gc):
            session.free(b)


@pytest.mark.parametrize("seed", [1, 2, 3])
def test_random_dependency_chains(session, seed):
    run_sequence(session, steps=300, seed=seed)


def test_dependency_chains_with_other_kernels_between(session):
    run_sequence(session, steps=200, seed=7, with_gemm=True)


def bf16_bits(x):
    return (np.asarray(x, np.float32).view(np.uint32) >> 16).astype(np.uint16)


def test_chain_reads_what_a_gemm_just_wrote(session):
    """A tensor-core GEMM (also launched with programmatic dependent launch)
    writes C = I @ B; the chain call right after it reads C. The chain kernel
    before the GEMM touches unrelated buffers, so only the GEMM stands
    between the two chain launches."""
    rng = np.random.default_rng(5)
    ga = session.alloc(capi.FER_DTYPE_BF16, [128, 128])
    gb = session.alloc(capi.FER_DTYPE_BF16, [128, 128])
    gc = session.alloc(capi.FER_DTYPE_F32, [128, 128])
    x = session.alloc(capi.FER_DTYPE_F32, [128 * 128])
    y = session.alloc(capi.FER_DTYPE_F32, [128 * 128])
    z = session.alloc(capi.FER_DTYPE_F32, [128 * 128])
    session.upload(ga, bf16_bits(np.eye(128)))
    session.upload(x, np.zeros(128 * 128, np.float32))
    ops = [(capi.FER_CHAIN_LOAD, 0, 0.0, 0.0), (capi.FER_CHAIN_AFFINE, 0, -1.0, 0.0)]
    for k in range(10):
        bvals = np.round(rng.uniform(-8, 8, (128, 128))).astype(np.float32)
        session.upload(gb, bf16_bits(bvals))
        session.affine(x, y, 128 * 128, 1.0, float(k), 0)    # a chain kernel on other buffers
        session.gemm(ga, gb, gc)
        session.wait(session.chain(ops, [gc], z))
        got = np.empty(128 * 128, np.float32)
        session.download(z, got)
        assert np.array_equal(got, -bvals.reshape(-1))
    for b in (ga, gb, gc, x, y, z):
        session.free(b)


def test_fixed_hazard_patterns(session):
    """Each hazard kind directly after the kernel it conflicts with."""
    rng = np.random.default_rng(11)
    a0, c0, e0 = (np.round(rng.uniform(-8, 8, N)).astype(np.float32) for _ in range(3))
    A, B, C, D, E = (session.alloc(capi.FER_DTYPE_F32, [N]) for _ in range(5))
    session.upload(A, a0)
    session.upload(C, c0)
    session.upload(E, e0)
    session.affine(A, B, N, -1.0, 2.0, 0)          # B = 2 - a0
    session.affine(C, A, N, 1.0, 1.0, 0)           # write-after-read on A: A = c0 + 1
    session.affine(B, A, N, 0.5, 0.0, 0)           # write-after-write on A: A = B / 2
    session.affine(A, C, N, 1.0, -1.0, 0)          # read-after-write: C = A - 1
    session.affine(E, D, N, -1.0, 0.0, 0)          # independent: D = -e0
    job = session.affine(C, C, N, 1.0, 3.0, 0)     # in place: C = C + 3
    session.wait(job)
    b = 2.0 - a0
    want = {A: b * 0.5, B: b, C: b * 0.5 - 1.0 + 3.0, D: -e0}
    for buf, w in want.items():
        got = np.empty(N, np.float32)
        session.download(buf, got)
        assert np.array_equal(got, w.astype(np.float32))
    for buf in (A, B, C, D, E):
        session.free(buf)


def replay(session, init, plan, sync_each):
    """Runs `plan` (a list of ("rows", ops, src, dst) / ("chain", alpha,
    beta, src, dst)) on fresh buffers holding `init`; returns their bytes."""
    ids = [session.alloc(capi.FER_DTYPE_F32, list(a.shape)) for a in init]
    for b, a in zip(ids, init):
        session.upload(b, a)
    job = 0
    for step in plan:
        if step[0] == "rows":
            _, ops, src, dst = step
            job = session.rows(ids[src], ids[dst], ops)
        else:
            _, alpha, beta, src, dst = step
            job = session.chain([(capi.FER_CHAIN_LOAD, 0, 0.0, 0.0), (capi.FER_CHAIN_AFFINE, 0, alpha, beta)],
                                [ids[src]], ids[dst])
        if sync_each:
            session.wait(job)
    session.wait(job)
    out = []
    for b, a in zip(ids, init):
        got = np.empty_like(a)
        session.download(b, got)
        out.append(got)
        session.free(b)
    return out


@pytest.mark.parametrize("seed", [21, 22])
def test_rows_and_chains_back_to_back_equal_synchronous_replay(session, seed):
    """Row kernels (fast and reference-order) and chain kernels in a random
    order with random buffer reuse give the same bits back to back as with a
    wait after every call (all of them are deterministic)."""
    rng = np.random.default_rng(seed)
    rows, cols = 512, 1024
    init = [rng.standard_normal((rows, cols)).astype(np.float32) for _ in range(4)]
    fast = capi.FER_ROWS_FAST
    plan = []
    for _ in range(120):
        src, dst = (int(v) for v in rng.integers(0, 4, 2))
        if rng.random() < 0.5:
            ops = int(rng.choice([capi.FER_ROWS_SOFTMAX, capi.FER_ROWS_LAYER_NORM,
                                  capi.FER_ROWS_SOFTMAX | capi.FER_ROWS_LAYER_NORM]))
            if rng.random() < 0.5:
                ops |= fast
            plan.append(("rows", ops, src, dst))
        else:
            plan.append(("chain", float(rng.choice([1.0, -1.0, 0.5])), float(rng.integers(-2, 3)), src, dst))
    a = replay(session, init, plan, sync_each=False)
    b = replay(session, init, plan, sync_each=True)
    for x, y in zip(a, b):
        assert np.array_equal(x.view(np.uint32), y.view(np.uint32))
