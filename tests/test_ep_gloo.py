"""Expert-parallel host logic on 2 and 4 CPU ranks (gloo).

``wanferenz_b200.ep.ep_forward`` (route the owned tokens, all-gather tokens
and routing, local experts on the gathered batch with the given routing plus
the shared expert on the rank's own rows, reduce-scatter, bf16) is driven with
a CPU stand-in layer whose parts come from the oracle (architecture.py:749-756,
785-794).  The result must equal the single-process oracle up to the fp32
summation order of the partials.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import fixtures as F
from oracle import moe_oracle as O

SPEC = F.LayerSpec(D=256, I=128, E=16, topk=4, score_func="sigmoid", route_scale=1.5, seed=51)


class OracleShard:
    """CPU stand-in with MoELayer's route / forward_ep / to_bf16 contract, including
    its capacity: at most ``max_tokens`` rows per call (the workspace's size)."""

    def __init__(self, syn, lo, hi, max_tokens=64):
        self.syn, self.lo, self.hi, self.max_tokens = syn, lo, hi, max_tokens

    def route(self, x, input_ids=None):
        assert x.size(0) <= self.max_tokens, "route: more rows than the workspace holds"
        p = self.syn.params()
        w, idx, _ = O.gate(x.float().numpy(), p["gate_w"], p.get("gate_b"), p["topk"], p["score_func"],
                           p["route_scale"], p.get("tid2eid"), input_ids)
        return torch.from_numpy(w), torch.from_numpy(idx)

    def forward_ep(self, x, weights, indices, shared_rows=(0, 0)):
        assert x.size(0) <= self.max_tokens, "forward_ep: more rows than the workspace holds"
        r0, n = shared_rows
        assert 0 <= r0 and r0 + n <= x.size(0), "shared rows outside the batch"
        xf = x.float().numpy()
        p, _, _ = O.moe_forward(xf, self.syn.params(), None, expert_range=(self.lo, self.hi),
                                return_partial=True, routing=(weights.numpy(), indices.numpy()))
        r0, n = shared_rows
        p[r0:r0 + n] += O.expert_fp8(xf[r0:r0 + n], *self.syn.shared(), weights=None,
                                     swiglu_limit=SPEC.swiglu_limit, ue8m0=SPEC.ue8m0)
        return torch.from_numpy(p.astype(np.float32))

    def to_bf16(self, y):
        return torch.from_numpy(O.round_bf16(y.numpy().astype(np.float32))).to(torch.bfloat16)

    def sum_ranks(self, parts):
        acc = parts[0].numpy().astype(np.float32)
        for p in range(1, parts.size(0)):
            acc = (acc + parts[p].numpy()).astype(np.float32)
        return torch.from_numpy(O.round_bf16(acc)).to(torch.bfloat16)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, T, q, combine="reduce_scatter", max_tokens=64):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from wanferenz_b200.ep import ep_forward, shard_range

        syn = F.SyntheticLayer(SPEC)
        x16, _ = syn.activations(T * world, draw=rank * 0 + 5)
        x = torch.from_numpy(O.bf16_to_f32(x16)).to(torch.bfloat16)
        mine = x[rank * T:(rank + 1) * T]
        lo, hi = shard_range(SPEC.E, world, rank)
        y = ep_forward(OracleShard(syn, lo, hi, max_tokens), mine, combine=combine)
        q.put((rank, y.float().numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,T,combine,cap", [(2, 1, "reduce_scatter", 64), (2, 3, "reduce_scatter", 64),
                                                 (2, 3, "all_to_all", 64), (4, 2, "reduce_scatter", 64),
                                                 (4, 2, "all_to_all", 64),
                                                 # gathered batch (P*T) above the workspace capacity: pieces
                                                 (2, 5, "reduce_scatter", 4), (4, 3, "all_to_all", 5)])
def test_ep_forward_matches_single_process(world, T, combine, cap):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, T, q, combine, cap)) for r in range(world)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=180) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    syn = F.SyntheticLayer(SPEC)
    x16, _ = syn.activations(T * world, draw=5)
    y_ref, _, _ = O.moe_forward(O.bf16_to_f32(x16), syn.params(), None)
    got = np.concatenate([out[r] for r in range(world)])
    d = np.abs(got - y_ref)
    assert d.mean() <= 2e-3
    assert (d / np.maximum(np.abs(y_ref), 0.01 * np.sqrt((y_ref ** 2).mean()))).max() <= 1e-2


def _dead_worker(rank, world, port, q):
    import datetime

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(0)  # this rank leaves between steps, with nothing in flight
    try:
        t = torch.zeros(4)
        dist.all_reduce(t)
        q.put("completed")
    except Exception as e:  # the survivor must see an error, not hang
        q.put(type(e).__name__)


def test_lost_rank_surfaces_as_error_not_hang():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dead_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert res != "completed"
