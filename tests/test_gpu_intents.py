"""JIT intents other than affine (tests/c_api/test_c_api_jit_intent.cpp covers
affine): reduce_sum / reduce_max (deterministic two-stage rewrite of the
reference's atomic version), the softmax intent (reference JIT softmax
reduction order) and direct conv2d, through fer_jit_run_intent."""
import ctypes as C

import numpy as np
import pytest

from fercuda_b200 import capi, synth

pytestmark = pytest.mark.gpu


def intent(op, n, **kw):
    it = capi.fer_jit_intent_t()
    it.abi_version = capi.FER_JIT_INTENT_ABI_VERSION
    it.op = op
    it.memory_regime = capi.FER_MEMORY_AUTO
    it.n = n
    for k, v in kw.items():
        setattr(it, k, v)
    return it


def run(session, it, inp, out, weights=0, bias=0):
    b = capi.fer_jit_intent_bindings_t(inp, out, weights, bias)
    job = C.c_uint64()
    capi.check("intent", session.call("fer_jit_run_intent", C.byref(it), C.byref(b), C.byref(job)))
    session.wait(job.value)


@pytest.mark.parametrize("n", [1, 511, 512, 513, 1 << 20, 3_000_001])
def test_reduce_sum_deterministic(session, n):
    x = synth.normal_f32(61, n)
    bx, bo = session.alloc(capi.FER_DTYPE_F32, [n]), session.alloc(capi.FER_DTYPE_F32, [1])
    session.upload(bx, x)
    outs = []
    for _ in range(3):
        session.upload(bo, np.array([0.25], np.float32))
        run(session, intent(capi.FER_JIT_INTENT_OP_REDUCE_SUM_F32, n), bx, bo)
        o = np.empty(1, np.float32)
        session.download(bo, o)
        outs.append(o[0])
    assert len({np.float32(v).view(np.uint32).item() for v in outs}) == 1
    ref = 0.25 + x.astype(np.float64).sum()
    assert abs(outs[0] - ref) <= 1e-5 * max(1.0, np.abs(x).sum())
    session.free(bx)
    session.free(bo)


def test_reduce_max(session):
    n = 1_000_003
    x = synth.normal_f32(62, n)
    bx, bo = session.alloc(capi.FER_DTYPE_F32, [n]), session.alloc(capi.FER_DTYPE_F32, [1])
    session.upload(bx, x)
    session.upload(bo, np.array([-1e30], np.float32))
    run(session, intent(capi.FER_JIT_INTENT_OP_REDUCE_MAX_F32, n), bx, bo)
    o = np.empty(1, np.float32)
    session.download(bo, o)
    assert o[0] == x.max()
    session.upload(bo, np.array([100.0], np.float32))
    run(session, intent(capi.FER_JIT_INTENT_OP_REDUCE_MAX_F32, n), bx, bo)
    session.download(bo, o)
    assert o[0] == 100.0


def test_softmax_intent_rows(session):
    rows, cols = 37, 3000
    x = synth.normal_f32(63, rows * cols, 0.0, 2.0).reshape(rows, cols)
    bx, by = session.alloc(capi.FER_DTYPE_F32, [rows, cols]), session.alloc(capi.FER_DTYPE_F32, [rows, cols])
    session.upload(bx, x)
    run(session, intent(capi.FER_JIT_INTENT_OP_SOFTMAX_F32, cols, height=rows), bx, by)
    y = np.empty_like(x)
    session.download(by, y)
    xd = x.astype(np.float64)
    e = np.exp(xd - xd.max(axis=1, keepdims=True))
    p = e / e.sum(axis=1, keepdims=True)
    assert (np.abs(y - p) / p).max() < 1e-5


def test_conv2d_intent(session):
    H, W, Cc, KH, KW, F = 9, 11, 3, 3, 3, 5
    x = synth.normal_f32(64, H * W * Cc)
    w = synth.normal_f32(65, F * Cc * KH * KW)
    bvec = synth.normal_f32(66, F)
    oh, ow = H, W   # pad 1, stride 1
    bx, bw, bb, bo = (session.alloc(capi.FER_DTYPE_F32, [s]) for s in (H * W * Cc, F * Cc * KH * KW, F, oh * ow * F))
    session.upload(bx, x)
    session.upload(bw, w)
    session.upload(bb, bvec)
    it = intent(capi.FER_JIT_INTENT_OP_CONV2D_F32, 0, height=H, width=W, channels=Cc, kernel_h=KH, kernel_w=KW,
                pad_h=1, pad_w=1, stride_h=1, stride_w=1, num_filters=F, fusion_mask=capi.FER_JIT_INTENT_FUSION_RELU)
    run(session, it, bx, bo, bw, bb)
    y = np.empty(oh * ow * F, np.float32)
    session.download(bo, y)
    xi = x.reshape(H, W, Cc).astype(np.float64)
    wi = w.reshape(F, Cc, KH, KW).astype(np.float64)
    xp = np.pad(xi, ((1, 1), (1, 1), (0, 0)))
    ref = np.zeros((oh, ow, F))
    for i in range(oh):
        for j in range(ow):
            patch = xp[i:i + KH, j:j + KW, :]
            ref[i, j] = np.einsum("hwc,fchw->f", patch, wi) + bvec
    ref = np.maximum(ref, 0.0)
    assert np.abs(y.reshape(oh, ow, F) - ref).max() < 1e-4


def test_jobs_with_and_without_temporaries_interleaved(session):
    """A reduce intent (a job with a temporary scratch buffer and its own
    completion event) submitted inside a run of chain jobs (which share
    events): every job reports done after a wait on it, the scratch is
    released, and results follow stream order."""
    n = 1 << 20
    x = np.ones(n, np.float32)
    bx, by, bo = (session.alloc(capi.FER_DTYPE_F32, [n]), session.alloc(capi.FER_DTYPE_F32, [n]),
                  session.alloc(capi.FER_DTYPE_F32, [1]))
    session.upload(bx, x)
    session.upload(bo, np.zeros(1, np.float32))
    jobs = [session.affine(bx, by, n, 1.0, float(k), 0) for k in range(5)]     # by = 1 + 4 at the end
    b = capi.fer_jit_intent_bindings_t(by, bo, 0, 0)
    red = C.c_uint64()
    capi.check("intent", session.call("fer_jit_run_intent", C.byref(intent(capi.FER_JIT_INTENT_OP_REDUCE_SUM_F32, n)),
                                      C.byref(b), C.byref(red)))
    jobs += [session.affine(bx, bx, n, 2.0, 0.0, 0) for _ in range(3)]         # bx = 8 at the end
    done = C.c_uint8()
    session.wait(jobs[2])
    for j in jobs[:5] + [red.value]:
        capi.check("status", session.call("fer_job_status", C.c_uint64(j), C.byref(done)))
    session.wait(red.value)
    session.wait(jobs[-1])
    for j in jobs + [red.value]:
        capi.check("status", session.call("fer_job_status", C.c_uint64(j), C.byref(done)))
        assert done.value == 1
    o = np.empty(1, np.float32)
    session.download(bo, o)
    assert o[0] == np.float32(5.0 * n)
    y = np.empty(n, np.float32)
    session.download(bx, y)
    assert np.all(y == 8.0)
    for buf in (bx, by, bo):
        session.free(buf)
