"""The C-ABI side of the batch-sharded forward on GPUs.

- fer_buffer_row_digests against a numpy restatement of its definition (sum
  mod 2^64 of a mix of every 16-byte chunk and its index in the row).
- A one-rank communicator (fer_comm_init with world 1) and
  fer_transformer_broadcast_weights: the NCCL path runs on a single GPU and
  leaves the weights as they were.
- With two or more GPUs: two processes, one per GPU; rank 1 starts from other
  weights, the broadcast gives it rank 0's (equal weight digests), each rank
  runs its half of the batch, and the per-sequence logits digests equal those
  of rank 0's forward of the whole batch on one GPU.
NVLS is off (NCCL_NVLS_ENABLE=0) in the child processes; nothing here faults
or hangs a GPU on purpose, and every NCCL wait in the library is bounded."""
import os
import socket

import numpy as np
import pytest
import torch  # noqa: F401  (first, so its libnccl.so.2 is the copy the library opens)

from fercuda_b200 import capi, synth

pytestmark = pytest.mark.gpu

M64 = (1 << 64) - 1
G = 0x9E3779B97F4A7C15


def mix64(z):
    z = z & M64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M64
    return z ^ (z >> 31)


def digest_ref(row: bytes) -> int:
    words = np.frombuffer(row, dtype="<u8")
    acc = 0
    for j in range(len(words) // 2):
        lo, hi = int(words[2 * j]), int(words[2 * j + 1])
        acc = (acc + mix64(lo ^ mix64(hi + G * (j + 1)))) & M64
    return acc


def test_row_digests_match_their_definition(session):
    rows, row_bytes = 5, 4096 + 48
    data = synth.splitmix64(77, rows * row_bytes // 8).view(np.uint8).copy()
    b = session.alloc(capi.FER_DTYPE_U8, [rows * row_bytes])
    session.upload(b, data)
    got = session.row_digests(b, row_bytes, rows)
    want = [digest_ref(data[r * row_bytes:(r + 1) * row_bytes].tobytes()) for r in range(rows)]
    assert got == want
    # a digest depends on the row's bytes only: the same bytes at another row give the same value
    data2 = np.concatenate([data[row_bytes:2 * row_bytes], data[:row_bytes]])
    b2 = session.alloc(capi.FER_DTYPE_U8, [2 * row_bytes])
    session.upload(b2, data2)
    assert session.row_digests(b2, row_bytes, 2) == [want[1], want[0]]
    with pytest.raises(capi.FerError):
        session.row_digests(b, 24, 1)                      # not a multiple of 16
    with pytest.raises(capi.FerError):
        session.row_digests(b, row_bytes, rows + 1)        # past the buffer
    session.free(b)
    session.free(b2)


def test_one_rank_communicator_broadcast(session):
    m = capi.Transformer(session, 1, 256, 4, 512, 1000, 64)
    m.init_weights(4, 0.02)
    wb = m.weight_buffer()
    nbytes = 2 * m.weight_elements()
    before = session.row_digests(wb, nbytes, 1)
    with pytest.raises(capi.FerError):
        m.broadcast_weights(0)                             # no communicator yet
    session.comm_init(capi.comm_unique_id(), 0, 1, 60_000)
    with pytest.raises(capi.FerError):
        session.comm_init(capi.comm_unique_id(), 0, 1)     # one per session
    assert m.broadcast_weights(0) == nbytes
    with pytest.raises(capi.FerError):
        m.broadcast_weights(1)                             # root outside the world
    assert session.row_digests(wb, nbytes, 1) == before
    session.comm_destroy()
    with pytest.raises(capi.FerError):
        session.comm_destroy()
    m.close()


SMALL = dict(layers=2, d_model=256, heads=4, ffn=512, vocab=1000, seq=128, batch=4)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tokens(c):
    u = synth.uniform01(5, c["batch"] * c["seq"])
    return np.minimum((u * c["vocab"]).astype(np.int32), c["vocab"] - 1).reshape(c["batch"], c["seq"])


def _rank(rank, world, q_id, q_out):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    c = SMALL
    with capi.Session(rank, pool_bytes=1 << 30) as s:
        m = capi.Transformer(s, c["layers"], c["d_model"], c["heads"], c["ffn"], c["vocab"], c["batch"] * c["seq"])
        m.init_weights(4 if rank == 0 else 99 + rank, 0.02)
        if rank == 0:
            uid = capi.comm_unique_id()
            for _ in range(world - 1):
                q_id.put(uid)
        else:
            uid = q_id.get(timeout=60)
        s.comm_init(uid, rank, world, 60_000)
        m.broadcast_weights(0)
        s.comm_destroy()
        wdig = s.row_digests(m.weight_buffer(), 2 * m.weight_elements(), 1)[0]
        toks = _tokens(c)
        first, count = capi.transformer_shard(c["batch"], world, rank)
        bt = s.alloc(capi.FER_DTYPE_I32, [count, c["seq"]])
        bl = s.alloc(capi.FER_DTYPE_F32, [count, c["seq"], c["vocab"]])
        s.upload(bt, np.ascontiguousarray(toks[first:first + count]))
        s.wait(m.forward(bt, bl))
        mine = s.row_digests(bl, 4 * c["seq"] * c["vocab"], count)
        whole = None
        if rank == 0:
            bt2 = s.alloc(capi.FER_DTYPE_I32, [c["batch"], c["seq"]])
            bl2 = s.alloc(capi.FER_DTYPE_F32, [c["batch"], c["seq"], c["vocab"]])
            s.upload(bt2, toks)
            s.wait(m.forward(bt2, bl2))
            whole = s.row_digests(bl2, 4 * c["seq"] * c["vocab"], c["batch"])
        q_out.put((rank, first, wdig, mine, whole, s.device_errors()))
        m.close()


def test_two_gpu_broadcast_and_sharded_forward():
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = torch.multiprocessing.get_context("spawn")
    q_id, q_out = ctx.Queue(), ctx.Queue()
    world = 2
    procs = [ctx.Process(target=_rank, args=(r, world, q_id, q_out)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q_out.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
    assert [p.exitcode for p in procs] == [0] * world
    res.sort()
    assert len({r[2] for r in res}) == 1, "weight digests differ after the broadcast"
    gathered = [d for r in res for d in r[3]]
    assert gathered == res[0][4], "sharded logits differ from the one-GPU forward"
    assert all(r[5] == 0 for r in res)


def test_comm_argument_errors(session):
    uid = capi.comm_unique_id()
    for rank, world in ((1, 1), (-1, 2), (0, 0)):
        with pytest.raises(capi.FerError) as e:
            session.comm_init(uid, rank, world)
        assert e.value.code == capi.FER_STATUS_INVALID_ARGUMENT
    with pytest.raises(capi.FerError) as e:
        session.row_digests(1 << 40, 16, 1)              # no such buffer
    assert e.value.code == capi.FER_STATUS_NOT_FOUND


def _lonely_rank(q_out):
    import time

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    with capi.Session(0, pool_bytes=256 << 20) as s:
        t0 = time.time()
        try:
            s.comm_init(capi.comm_unique_id(), 0, 2, 3_000)
            first = (None, "", 0.0)
        except capi.FerError as e:
            first = (e.code, e.msg, time.time() - t0)
        m = capi.Transformer(s, 1, 256, 4, 512, 1000, 64)
        m.init_weights(4, 0.02)
        s.comm_init(capi.comm_unique_id(), 0, 1, 30_000)
        sent = m.broadcast_weights(0)
        s.comm_destroy()
        q_out.put(first + (sent == 2 * m.weight_elements(), s.device_errors()))
        m.close()


def test_rank_that_never_joins_times_out():
    """Failure made on the host: a two-rank communicator whose second rank
    never calls fer_comm_init. The first rank's init returns
    FER_STATUS_INTERNAL_ERROR after its 3 s timeout (the communicator is
    aborted) instead of waiting forever, and the session stays usable: a
    one-rank communicator and a weight broadcast work right after. No kernel
    waits on the missing rank at any point; the rank runs in a child process
    so that the test itself is bounded too."""
    import torch

    ctx = torch.multiprocessing.get_context("spawn")
    q_out = ctx.Queue()
    p = ctx.Process(target=_lonely_rank, args=(q_out,))
    p.start()
    try:
        code, msg, waited, sent_ok, errors = q_out.get(timeout=240)
    finally:
        p.join(timeout=60)
        if p.exitcode is None:
            p.kill()
    assert p.exitcode == 0
    assert code == capi.FER_STATUS_INTERNAL_ERROR and "timed out" in msg, (code, msg)
    assert 2.5 <= waited <= 60.0, waited
    assert sent_ok and errors == 0
