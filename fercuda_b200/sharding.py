"""Host-side plumbing of the batch-sharded transformer forward.

One process per GPU. The global batch of sequences is split into equal,
contiguous shards (rank r takes sequences [r*B/N, (r+1)*B/N)); the weights are
made once on rank 0 and broadcast over the process group (NCCL over NVLink /
NVSwitch on GPUs); no collective runs inside a forward, because sequences of
a batch never interact. Step time is the maximum over ranks.

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


def device_bytes_as_tensor(torch, ptr: int, nbytes: int):
    """A torch uint8 view of `nbytes` of device memory at `ptr` (no copy), so a
    buffer of this library can take part in a torch.distributed collective."""

    class _View:
        __cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3,
                                    "strides": None}

    return torch.as_tensor(_View(), device="cuda")


def broadcast_from_rank0(dist, tensor) -> int:
    """Broadcasts `tensor` in place from rank 0; returns the bytes moved."""
    dist.broadcast(tensor, src=0)
    return tensor.numel() * tensor.element_size()


def max_over_ranks(torch, dist, value: float, device) -> float:
    """The maximum of a per-rank scalar (e.g. device milliseconds) over ranks."""
    t = torch.tensor([value], dtype=torch.float64, device=device)
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
