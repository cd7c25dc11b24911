"""Token-row sharding of the read across ranks (one process per GPU).

Every token row of the depth-routing read is independent (the softmax runs over
sources, not tokens), so a batch of N rows splits into contiguous shards with
no data-path exchange. The only cross-rank step is summing the parameter
gradients that the backward reduces over tokens: the static query, the query
gate and the per-source logit biases. `allreduce_param_grads` does that in one
bucketed all-reduce (NCCL over NVLink on GPUs, gloo on CPU).

Inside DDP those tensors are parameters and DDP already all-reduces their
gradients: do not call this there, or they are summed twice.
"""
from typing import Sequence, Tuple

import torch
import torch.distributed as dist


def token_shard(n_tokens: int, rank: int, world: int) -> Tuple[int, int]:
    """Contiguous [start, stop) rows of rank `rank`; sizes differ by at most one."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"invalid rank {rank} for world size {world}")
    if n_tokens < 0:
        raise ValueError("n_tokens must be non-negative")
    base, extra = divmod(n_tokens, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def allreduce_param_grads(grads: Sequence[torch.Tensor], group=None) -> None:
    """Sum `grads` over all ranks in place, as one flat fp32 bucket."""
    grads = [g for g in grads if g is not None]
    if not grads or not dist.is_initialized() or dist.get_world_size(group) == 1:
        return
    if all(g.dtype == torch.float32 and g.is_contiguous() for g in grads) and len(grads) <= 2:
        # already fp32: reduce in place, no packing copies
        for g in grads:
            dist.all_reduce(g, op=dist.ReduceOp.SUM, group=group)
        return
    flat = torch.cat([g.reshape(-1).to(torch.float32) for g in grads])
    dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
    offset = 0
    for g in grads:
        n = g.numel()
        g.copy_(flat[offset:offset + n].view_as(g).to(g.dtype))
        offset += n
