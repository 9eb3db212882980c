"""Batch sharding across the GPUs of one node (one process per GPU).

The reference has no parallelism beyond intra-op CPU threads; the B200 build
shards the batch: images (YOLO, conv), sequences (attention) and rows (GEMM,
DynamicQuantizeMatMul) are independent, so each rank runs its shard with no
data-path collective. The one real exchange is DQMM's per-tensor range:
every row shard must quantise with the range of the WHOLE tensor, so the
ranks all-reduce {min, max} (two floats) before quantising — then q and the
int32 accumulators are bit-identical to the unsharded result.
"""
from __future__ import annotations


def shard_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """[start, end) of rank's contiguous shard of n items (the first n % world ranks get one more)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of {world}")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def global_minmax(local, group=None):
    """All-reduce a local {min, max} pair (a 2-element float tensor on the
    rank's device, or CPU for gloo) into the global range, in place, with ONE
    collective: {-min, max} reduced by MAX (negation is exact, so the result
    is the exact global minimum and maximum)."""
    import torch
    import torch.distributed as dist

    sign = _SIGNS.get(local.device)
    if sign is None:
        sign = _SIGNS[local.device] = torch.tensor([-1.0, 1.0], dtype=local.dtype, device=local.device)
    t = local * sign
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    torch.mul(t, sign, out=local)
    return local


_SIGNS: dict = {}


def max_over_ranks(values, group=None):
    """Element-wise maximum of a float64 tensor across ranks (step times)."""
    import torch.distributed as dist

    dist.all_reduce(values, op=dist.ReduceOp.MAX, group=group)
    return values
