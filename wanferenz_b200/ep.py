"""Expert parallelism of the MoE layer over torch.distributed (NCCL on B200s).

Rank ``r`` of ``P`` holds experts ``[r*E/P, (r+1)*E/P)`` (architecture.py:749-756)
and its own batch of ``T`` tokens (decode serving with data-parallel tokens).
The reference all-reduces a layer that every rank computes for the whole
batch; here each token is routed once, on the rank that owns it:

1. route the rank's own ``T`` tokens (``MoELayer.route``);
2. all-gather the ``P*T`` tokens and their routing (one NCCL group);
3. one forward on the gathered batch with that routing: the rank's local
   experts on every row, the shared expert on the rank's own rows only
   (``MoELayer.forward_ep``) -> fp32 partial sums ``[P*T, D]``;
4. combine: each rank receives the sum over ranks for its own rows (the
   reference's ``dist.all_reduce(y)``, architecture.py:791-792, restricted to
   those rows), shared expert included (793), cast to bf16 (794); either
   ``reduce_scatter`` (NCCL reduces, in its own order) or ``all_to_all`` (each
   rank receives the other ranks' partial rows and sums them in ascending rank
   order: the same bytes, one more kernel, results independent of the
   collective's algorithm).

The dispatch is an all-gather: every rank needs every token's row (its
experts may be among the token's k), so a fixed-capacity all-to-all would move
the same bytes.
"""

from __future__ import annotations

import torch
import torch.distributed as dist
from torch.distributed import distributed_c10d as c10d


def gather_tokens(x, w, idx, xg, wg, ig, group=None):
    """All-gathers tokens ``x [T, D]`` and their routing ``w [T, k]``, ``idx [T, k]``
    into ``xg, wg, ig [P*T, ...]`` (rank r's rows at ``r*T``).  On NCCL the three
    gathers are issued as one group, so they cost one collective launch."""
    coalesce = getattr(c10d, "_coalescing_manager", None)  # a private torch API: used when present
    if coalesce is not None and dist.get_backend(group) == "nccl":
        with coalesce(group, x.device):
            dist.all_gather_into_tensor(xg, x, group=group)
            dist.all_gather_into_tensor(wg, w, group=group)
            dist.all_gather_into_tensor(ig, idx, group=group)
    else:
        dist.all_gather_into_tensor(xg, x, group=group)
        dist.all_gather_into_tensor(wg, w, group=group)
        dist.all_gather_into_tensor(ig, idx, group=group)


COMBINES = ("reduce_scatter", "all_to_all")


def ep_forward(layer, x, input_ids=None, group=None, combine="reduce_scatter"):
    """One expert-parallel MoE forward of this rank's ``x [T, D]`` (T equal on all ranks)."""
    if combine not in COMBINES:
        raise ValueError(f"combine must be one of {COMBINES}")
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    T = x.size(0)
    x = x.contiguous()
    w, idx = layer.route(x, input_ids)
    xg = torch.empty(world * T, x.size(1), dtype=x.dtype, device=x.device)
    wg = torch.empty(world * T, w.size(1), dtype=w.dtype, device=x.device)
    ig = torch.empty(world * T, idx.size(1), dtype=idx.dtype, device=x.device)
    gather_tokens(x, w.contiguous(), idx.contiguous(), xg, wg, ig, group)
    part = layer.forward_ep(xg, wg, ig, shared_rows=(rank * T, T))
    if combine == "all_to_all":
        recv = torch.empty(world, T, x.size(1), dtype=torch.float32, device=x.device)
        dist.all_to_all_single(recv, part, group=group)
        return layer.sum_ranks(recv)
    mine = torch.empty(T, x.size(1), dtype=torch.float32, device=x.device)
    dist.reduce_scatter_tensor(mine, part, group=group)
    return layer.to_bf16(mine)


def shard_range(n_experts, world, rank):
    """Contiguous expert shard of ``rank`` (architecture.py:749-756)."""
    if n_experts % world:
        raise ValueError(f"{n_experts} experts do not divide over {world} ranks")
    per = n_experts // world
    return rank * per, (rank + 1) * per
