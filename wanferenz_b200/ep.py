"""Expert parallelism of the MoE layer over torch.distributed (NCCL on B200s).

Rank ``r`` of ``P`` holds experts ``[r*E/P, (r+1)*E/P)`` (architecture.py:749-756)
and its own batch of ``T`` tokens (decode serving with data-parallel tokens).
The reference all-reduces a layer that every rank computes for the whole
batch; here the work splits by who owns what:

1. each rank routes its own ``T`` tokens and runs the shared expert on them
   (``MoELayer.route_shared``: one router pass per token in the job, not one
   per rank);
2. all-gather the ``P*T`` tokens and their routing (NCCL over NVLink);
3. every rank runs its local experts on the gathered batch with that routing
   (``MoELayer.forward_routed``) -> fp32 partial sums ``[P*T, D]``;
4. reduce-scatter the partials, so each rank receives the sum over ranks for
   its own rows (the reference's ``dist.all_reduce(y)``, architecture.py:791-792,
   restricted to the rows the rank owns);
5. add the shared expert's rows and cast to bf16 (793-794).
"""

from __future__ import annotations

import torch
import torch.distributed as dist
from torch.distributed import distributed_c10d as c10d


def gather_tokens(x, w, idx, xg, wg, ig, group=None):
    """All-gathers tokens ``x [T, D]`` and their routing ``w [T, k]``, ``idx [T, k]``
    into ``xg, wg, ig [P*T, ...]`` (rank r's rows at ``r*T``).  On NCCL the three
    gathers are issued as one group, so they cost one collective launch."""
    if dist.get_backend(group) == "nccl":
        with c10d._coalescing_manager(group, x.device):
            dist.all_gather_into_tensor(xg, x, group=group)
            dist.all_gather_into_tensor(wg, w, group=group)
            dist.all_gather_into_tensor(ig, idx, group=group)
    else:
        dist.all_gather_into_tensor(xg, x, group=group)
        dist.all_gather_into_tensor(wg, w, group=group)
        dist.all_gather_into_tensor(ig, idx, group=group)


def ep_forward(layer, x, input_ids=None, group=None):
    """One expert-parallel MoE forward of this rank's ``x [T, D]`` (T equal on all ranks)."""
    world = dist.get_world_size(group)
    T = x.size(0)
    x = x.contiguous()
    shared, w, idx = layer.route_shared(x, input_ids)
    xg = torch.empty(world * T, x.size(1), dtype=x.dtype, device=x.device)
    wg = torch.empty(world * T, w.size(1), dtype=w.dtype, device=x.device)
    ig = torch.empty(world * T, idx.size(1), dtype=idx.dtype, device=x.device)
    gather_tokens(x, w.contiguous(), idx.contiguous(), xg, wg, ig, group)
    part = layer.forward_routed(xg, wg, ig)
    mine = torch.empty(T, x.size(1), dtype=torch.float32, device=x.device)
    dist.reduce_scatter_tensor(mine, part, group=group)
    return layer.add_shared(mine, shared)


def shard_range(n_experts, world, rank):
    """Contiguous expert shard of ``rank`` (architecture.py:749-756)."""
    if n_experts % world:
        raise ValueError(f"{n_experts} experts do not divide over {world} ranks")
    per = n_experts // world
    return rank * per, (rank + 1) * per
