"""Host-side plumbing of the batch-sharded transformer forward.

One process per GPU. The global batch of sequences is split into equal,
contiguous shards (rank r takes sequences [r*B/N, (r+1)*B/N), the split of
fer_transformer_shard); the weights are made once on rank 0 and copied into
every rank's weight buffer by fer_transformer_broadcast_weights (one NCCL
broadcast over NVLink / NVSwitch, in C++, on a communicator the session
owns); no collective runs inside a forward, because sequences of a batch
never interact. Step time is the maximum over ranks.

What this module adds for Python callers: the shard arithmetic on numpy
token arrays, handing the communicator's unique id from rank 0 to every rank
over an existing torch.distributed group, and the max over ranks of a
timing.

The reference's multi-GPU weight copy is a serial peer copy from the source
GPU to each destination (native/core/runtime/hot_multi_gpu_policy_main.inl:221-249,
`gpu_broadcast_tensor`); here it is one broadcast collective.
"""
from __future__ import annotations

import numpy as np


def shard_range(global_batch: int, world: int, rank: int) -> tuple[int, int]:
    """[start, stop) of rank's sequences. The batch must split evenly."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    if global_batch % world:
        raise ValueError(f"global batch {global_batch} does not split over {world} ranks")
    per = global_batch // world
    return rank * per, (rank + 1) * per


def shard_tokens(tokens: np.ndarray, world: int, rank: int) -> np.ndarray:
    """Rank's contiguous slice of a [batch, seq] token array."""
    lo, hi = shard_range(tokens.shape[0], world, rank)
    return np.ascontiguousarray(tokens[lo:hi])


def share_unique_id(dist, uid: bytes | None) -> bytes:
    """Rank 0's communicator unique id (fer_comm_unique_id, 128 bytes) on
    every rank of the torch.distributed group; other ranks pass None."""
    box = [uid]
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.broadcast_object_list(box, src=0)
    if not isinstance(box[0], (bytes, bytearray)) or len(box[0]) != 128:
        raise RuntimeError("communicator unique id did not arrive")
    return bytes(box[0])


def max_over_ranks(torch, dist, value: float, device) -> float:
    """The maximum of a per-rank scalar (e.g. device milliseconds) over ranks."""
    t = torch.tensor([value], dtype=torch.float64, device=device)
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
