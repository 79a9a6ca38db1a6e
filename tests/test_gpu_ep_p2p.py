"""Expert parallelism over peer memory (wf_moe_forward_ep_p2p, ep.PeerGroup).

* One rank: the peer-memory path (tokens and routing through the rank's own
  buffer, partial rows through its receive buffer, the finish kernel) gives
  outputs bit-identical to the regular fused forward, eagerly and replayed from
  a CUDA graph (the hand-off epochs are counted on the device).
* Two and four ranks, one process per GPU (skipped with fewer GPUs): each rank
  holds its share of the experts and its own tokens; every rank's output meets the
  layer tolerance against the single-process oracle (architecture.py:777-794).
"""

import os
import socket

import numpy as np
import pytest
import torch

from oracle import fixtures as F
from oracle import moe_oracle as O
from tests import gpu_util as U

pytestmark = pytest.mark.gpu

SPEC = F.LayerSpec(D=512, I=256, E=16, topk=4, score_func="sqrtsoftplus", route_scale=1.5, swiglu_limit=10.0,
                   seed=101)


@pytest.fixture(autouse=True)
def fused_engine(monkeypatch):
    monkeypatch.setenv("WF_DISABLE_TC", "0")
    monkeypatch.setenv("WF_FUSED", "1")


@pytest.mark.parametrize("spec,T", [(SPEC, 5), (F.CONFIG2, 16)], ids=["mini", "config2"])
def test_single_rank_matches_fused_forward(spec, T):
    from wanferenz_b200.ep import PeerGroup

    syn = F.SyntheticLayer(spec)
    x16, _ = syn.activations(T, draw=6)
    layer = U.quant_layer(syn, max_tokens=max(T, 16), seed=3) if spec.D >= 2048 else \
        U.device_layer(syn, list(range(spec.E)), max_tokens=max(T, 16))
    x = U.bf16_tensor(x16)
    y_ref, w_ref, i_ref = layer.forward(x, routing=True)
    peers = PeerGroup(layer)
    try:
        for call in range(3):
            y, rw, ri = peers.forward(x, routing=True)
            torch.cuda.synchronize()
            layer.read_error()
            assert torch.equal(ri, i_ref) and torch.equal(rw, w_ref), f"call {call}: routing differs"
            assert torch.equal(y, y_ref), f"call {call}: output differs from the fused forward"
        # three forwards captured in one graph, replayed twice
        xs = [U.bf16_tensor(syn.activations(T, draw=20 + k)[0]) for k in range(3)]
        refs = [layer.forward(xx) for xx in xs]
        outs = [torch.empty_like(r) for r in refs]
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for xx, o in zip(xs, outs):
                peers.forward(xx, out=o)
        for _ in range(2):
            for o in outs:
                o.zero_()
            g.replay()
            torch.cuda.synchronize()
            layer.read_error()
            for k in range(3):
                assert torch.equal(outs[k], refs[k]), f"graph replay, forward {k} differs"
        del g
    finally:
        peers.close()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, T, q):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WF_DISABLE_TC="0", WF_FUSED="1")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from wanferenz_b200.ep import PeerGroup, shard_range

        syn = F.SyntheticLayer(SPEC)
        x16, _ = syn.activations(T * world, draw=8)
        lo, hi = shard_range(SPEC.E, world, rank)
        layer = U.device_layer(syn, list(range(SPEC.E)), max_tokens=T * world, expert_range=(lo, hi))
        peers = PeerGroup(layer)
        x = U.bf16_tensor(x16[rank * T:(rank + 1) * T])
        outs = []
        for _ in range(3):
            y, rw, ri = peers.forward(x, routing=True)
            outs.append((U.to_f32(y), rw.cpu().numpy(), ri.cpu().numpy()))
        torch.cuda.synchronize()
        layer.read_error()
        peers.close()
        q.put((rank, outs))
    except Exception as e:  # the parent reports it
        import traceback

        q.put((rank, traceback.format_exc()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,T", [(2, 3), (2, 16), (4, 5)])
def test_ranks_match_oracle(world, T):
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, T, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
    for r in range(world):
        assert not isinstance(res[r], str), f"rank {r} failed:\n{res[r]}"
    syn = F.SyntheticLayer(SPEC)
    x16, ids = syn.activations(T * world, draw=8)
    xf = O.bf16_to_f32(x16)
    y_ref, w_ref, i_ref = O.moe_forward(xf, syn.params(), ids)
    y_ref32, _, _ = O.moe_forward(xf, syn.params(), ids, acc=np.float32)
    for call in range(3):
        y = np.concatenate([res[r][call][0] for r in range(world)])
        ri = np.concatenate([res[r][call][2] for r in range(world)])
        tie = U.near_tie_rows(xf, syn, what=f"{world} ranks T={T}")
        np.testing.assert_array_equal(ri[~tie], i_ref[~tie])
        U.assert_layer_close_envelope(y[~tie], y_ref[~tie], y_ref32[~tie], f"{world} ranks T={T} call {call}")
        if call:
            assert np.array_equal(y, np.concatenate([res[r][0][0] for r in range(world)])), "calls differ"
