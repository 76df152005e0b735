"""Batch sharding of the transformer forward, host side, on CPU.

Two `gloo` ranks stand in for two GPUs: rank 0 makes the weights and a
communicator id, hands the id to the other rank (sharding.share_unique_id,
as bench.py does before fer_comm_init), broadcasts the weights (a gloo
broadcast stands in for fer_transformer_broadcast_weights, which is NCCL on
the GPUs), each rank runs the oracle forward on its shard of the global
batch, and rank 0 checks the gathered logits against the whole-batch forward.
The GPU path's own split-invariance (bit-identical logits for any split) is
covered by the GPU tests; here the shard arithmetic and the collective steps
are.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from fercuda_b200 import sharding, synth
from oracle import transformer_ref as ref

TINY = dict(layers=1, d=128, heads=2, ffn=256, vocab=64, seq=16, batch=4)


def test_shard_ranges_cover_the_batch_once():
    for world in (1, 2, 4, 8):
        seen = []
        for r in range(world):
            lo, hi = sharding.shard_range(64, world, r)
            assert hi - lo == 64 // world
            seen.extend(range(lo, hi))
        assert seen == list(range(64))


def test_shard_range_rejects_uneven_and_bad_rank():
    with pytest.raises(ValueError):
        sharding.shard_range(64, 3, 0)
    with pytest.raises(ValueError):
        sharding.shard_range(64, 2, 2)


def test_shard_tokens_concatenate_to_the_batch():
    toks = np.arange(8 * 5, dtype=np.int32).reshape(8, 5)
    parts = [sharding.shard_tokens(toks, 4, r) for r in range(4)]
    assert all(p.flags.c_contiguous for p in parts)
    assert np.array_equal(np.concatenate(parts), toks)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, q) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        c = TINY
        total = ref.weight_offsets(c["layers"], c["d"], c["ffn"], c["vocab"])["total"]
        w = torch.zeros(2 * total, dtype=torch.uint8)        # the weight buffer as bytes, as on the GPUs
        if rank == 0:
            w.copy_(torch.from_numpy(synth.normal_bf16(4, total, 0.0, 0.02).view(np.uint8)))
        uid = sharding.share_unique_id(dist, bytes(range(128)) if rank == 0 else None)
        assert uid == bytes(range(128))
        dist.broadcast(w, src=0)
        wbits = w.numpy().view(np.uint16)
        u = synth.uniform01(5, c["batch"] * c["seq"])
        toks = np.minimum((u * c["vocab"]).astype(np.int32), c["vocab"] - 1).reshape(c["batch"], c["seq"])
        mine = sharding.shard_tokens(toks, world, rank)
        y = ref.forward(mine, wbits, c["layers"], c["d"], c["heads"], c["ffn"], c["vocab"])
        parts = [torch.empty_like(torch.from_numpy(y)) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(y))
        slowest = sharding.max_over_ranks(torch, dist, float(rank + 1), "cpu")
        if rank == 0:
            whole = ref.forward(toks, wbits, c["layers"], c["d"], c["heads"], c["ffn"], c["vocab"])
            got = torch.cat(parts).numpy()
            q.put((float(np.max(np.abs(got - whole)) / np.max(np.abs(whole))), slowest))
    finally:
        dist.destroy_process_group()


def test_two_rank_broadcast_and_shard_forward():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0, 0], codes
    err, slowest = q.get(timeout=5)
    assert err <= 1e-6, err
    assert slowest == 2.0


def test_c_abi_shard_matches_the_host_split():
    from fercuda_b200 import capi

    for world in (1, 2, 4, 8):
        for r in range(world):
            first, count = capi.transformer_shard(64, world, r)
            assert (first, first + count) == sharding.shard_range(64, world, r)
    with pytest.raises(capi.FerError):
        capi.transformer_shard(64, 3, 0)
    with pytest.raises(capi.FerError):
        capi.transformer_shard(64, 2, 2)
