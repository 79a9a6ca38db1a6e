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

The dispatch is an all-gather.  NCCL's all-to-all needs its split sizes on
the host, so a dispatch that sends each token only to the ranks owning one of
its experts would either move fixed-capacity blocks (the all-gather's bytes)
or wait for the counts on the host every layer (no CUDA-graph capture).  With
top-6 routing over P ranks a token needs P * (1 - (1 - 1/P)^6) of them on
average (~4.4 of 8), so compacted sends would move up to ~40 % fewer bytes at
P = 8; at decode sizes these collectives are latency-bound, not byte-bound.
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


def _pieces(n, cap):
    """Row ranges ``[a, b)`` of at most ``cap`` rows covering ``[0, n)``."""
    return [(a, min(n, a + cap)) for a in range(0, n, cap)]


def route_rows(layer, x, input_ids=None):
    """``layer.route`` over ``x`` in pieces of at most ``layer.max_tokens`` rows."""
    cap = layer.max_tokens
    if x.size(0) <= cap:
        return layer.route(x, input_ids)
    parts = [layer.route(x[a:b], None if input_ids is None else input_ids[a:b]) for a, b in _pieces(x.size(0), cap)]
    return torch.cat([p[0] for p in parts]), torch.cat([p[1] for p in parts])


def forward_rows(layer, xg, wg, ig, shared_rows, out):
    """``layer.forward_ep`` over the gathered batch in pieces of at most
    ``layer.max_tokens`` rows (a layer's workspace holds that many), each
    piece with the shared-row window clipped to it; writes ``out [P*T, D]``."""
    r0, n = shared_rows
    for a, b in _pieces(xg.size(0), layer.max_tokens):
        s0, s1 = max(a, r0), min(b, r0 + n)
        win = (s0 - a, s1 - s0) if s1 > s0 else (0, 0)
        out[a:b] = layer.forward_ep(xg[a:b], wg[a:b], ig[a:b], shared_rows=win)
    return out


def ep_forward(layer, x, input_ids=None, group=None, combine="reduce_scatter"):
    """One expert-parallel MoE forward of this rank's ``x [T, D]`` (T equal on all ranks).

    The gathered batch of ``P*T`` rows may exceed the layer's ``max_tokens``
    (its workspace capacity): it then runs in pieces of at most that many rows.
    """
    if combine not in COMBINES:
        raise ValueError(f"combine must be one of {COMBINES}")
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    T = x.size(0)
    x = x.contiguous()
    w, idx = route_rows(layer, x, input_ids)
    xg = torch.empty(world * T, x.size(1), dtype=x.dtype, device=x.device)
    wg = torch.empty(world * T, w.size(1), dtype=w.dtype, device=x.device)
    ig = torch.empty(world * T, idx.size(1), dtype=idx.dtype, device=x.device)
    gather_tokens(x, w.contiguous(), idx.contiguous(), xg, wg, ig, group)
    if world * T <= layer.max_tokens:
        part = layer.forward_ep(xg, wg, ig, shared_rows=(rank * T, T))
    else:
        part = torch.empty(world * T, x.size(1), dtype=torch.float32, device=x.device)
        forward_rows(layer, xg, wg, ig, (rank * T, T), part)
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


class PeerGroup:
    """Expert parallelism over peer memory for one layer (``wf_moe_forward_ep_p2p``).

    Each rank allocates one buffer (set-up, ``wf_ep_alloc``), exports it with CUDA
    IPC, and maps every other rank's; a forward then moves tokens, routing and
    partial output rows over NVLink inside the fused kernel, with no NCCL call.
    ``layer`` is this rank's shard (``n_local_experts = E / P``,
    ``expert_offset = rank * n_local_experts``) whose ``max_tokens`` holds the
    gathered batch (``P * T``).  Every rank must make the same sequence of
    forwards, each on one stream.
    """

    def __init__(self, layer, group=None):
        import ctypes

        from . import _lib as L

        self.lib = L.load()
        self.layer = layer
        self.group = group
        if dist.is_available() and dist.is_initialized():
            self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        else:
            self.world, self.rank = 1, 0
        nbytes = self.lib.wf_ep_buffer_bytes(ctypes.byref(layer.cfg), self.world)
        if nbytes == 0:
            raise ValueError(f"expert-parallel buffer: {self.lib.wf_last_error().decode()}")
        own = ctypes.c_void_p()
        L.check(self.lib.wf_ep_alloc(nbytes, ctypes.byref(own)), "wf_ep_alloc")
        self._own = own
        handle = (ctypes.c_uint8 * 64)()
        L.check(self.lib.wf_ipc_get_handle(own, handle), "wf_ipc_get_handle")
        handles = [bytes(handle)]
        if self.world > 1:
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(handle), group=group)
        self.bufs = (ctypes.c_void_p * self.world)()
        self._opened = []
        for p in range(self.world):
            if p == self.rank:
                self.bufs[p] = own.value
                continue
            ptr = ctypes.c_void_p()
            h = (ctypes.c_uint8 * 64).from_buffer_copy(handles[p])
            L.check(self.lib.wf_ipc_open_handle(h, ctypes.byref(ptr)), "wf_ipc_open_handle")
            self.bufs[p] = ptr.value
            self._opened.append(ptr)
        if self.world > 1:
            dist.barrier(group=group)

    def forward(self, x, input_ids=None, out=None, routing=False, out_routing=None):
        """This rank's ``x [T, D]`` bf16 -> ``y [T, D]`` bf16 (and its routing when asked,
        or into ``out_routing = (weights [T, k] f32, indices [T, k] int64)``)."""
        import ctypes

        from . import _lib as L

        lay = self.layer
        x = x.contiguous()
        T = x.size(0)
        if input_ids is not None:
            input_ids = input_ids.reshape(-1).to(torch.int64).contiguous()
        y = out if out is not None else torch.empty(T, lay.dim, dtype=torch.bfloat16, device=x.device)
        rw = ri = None
        if out_routing is not None:
            rw, ri = out_routing
        elif routing:
            rw = torch.empty(T, lay.topk, dtype=torch.float32, device=x.device)
            ri = torch.empty(T, lay.topk, dtype=torch.int64, device=x.device)
        rc = self.lib.wf_moe_forward_ep_p2p(
            ctypes.byref(lay.cfg), ctypes.byref(lay.wstruct), L.ptr(x), L.ptr(input_ids), T, self.rank, self.world,
            self.bufs, L.ptr(y), L.ptr(rw), L.ptr(ri), L.ptr(lay.workspace), lay.workspace.numel(), L.stream_ptr())
        L.check(rc, "wf_moe_forward_ep_p2p")
        return (y, rw, ri) if routing else y

    __call__ = forward

    def close(self):
        """Unmaps the peers' buffers and frees this rank's (after every rank is done)."""
        from . import _lib as L

        torch.cuda.synchronize()
        if self.world > 1:
            dist.barrier(group=self.group)
        for ptr in self._opened:
            L.check(self.lib.wf_ipc_close_handle(ptr), "wf_ipc_close_handle")
        self._opened = []
        if self._own is not None:
            if self.world > 1:
                dist.barrier(group=self.group)
            L.check(self.lib.wf_ep_free(self._own), "wf_ep_free")
            self._own = None
