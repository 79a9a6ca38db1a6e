"""Expert parallelism of the MoE layer over torch.distributed (NCCL on B200s).

Rank ``r`` of ``P`` holds experts ``[r*E/P, (r+1)*E/P)`` (architecture.py:749-756)
and its own batch of ``T`` tokens (decode serving with data-parallel tokens):

1. all-gather the ``P*T`` token batch (NCCL over NVLink);
2. every rank routes the whole batch identically and runs its local experts
   on it: ``wf_moe_forward(..., y_partial)`` -> fp32 partial sums ``[P*T, D]``,
   plus the shared expert for the batch;
3. reduce-scatter the partials, so each rank receives the sum over ranks for
   its own ``T`` rows (the reference's ``dist.all_reduce(y)``,
   architecture.py:791-792, restricted to the rows the rank owns);
4. ``wf_moe_finish`` adds the shared expert's rows and casts to bf16 (793-794).
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def ep_forward(layer, x, input_ids=None, group=None):
    """One expert-parallel MoE forward of this rank's ``x [T, D]`` (T equal on all ranks)."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    T = x.size(0)
    xg = torch.empty(world * T, x.size(1), dtype=x.dtype, device=x.device)
    dist.all_gather_into_tensor(xg, x.contiguous(), group=group)
    ids_g = None
    if input_ids is not None:
        ids = input_ids.reshape(-1).to(torch.int64).contiguous()
        ids_g = torch.empty(world * T, dtype=torch.int64, device=x.device)
        dist.all_gather_into_tensor(ids_g, ids, group=group)
    part = layer.forward(xg, ids_g, partial=True)
    mine = torch.empty(T, x.size(1), dtype=torch.float32, device=x.device)
    dist.reduce_scatter_tensor(mine, part, group=group)
    return layer.finish(mine, row0=rank * T)


def shard_range(n_experts, world, rank):
    """Contiguous expert shard of ``rank`` (architecture.py:749-756)."""
    if n_experts % world:
        raise ValueError(f"{n_experts} experts do not divide over {world} ranks")
    per = n_experts // world
    return rank * per, (rank + 1) * per
