"""Expert parallelism over NCCL (ep.ep_forward), one process per GPU.

Each rank holds 1/P of the experts and its own T tokens; it routes them
(``wf_moe_route``), all-gathers tokens and routing over NCCL, runs its local
experts on the gathered batch plus the shared expert on its own rows
(``wf_moe_forward_ep``), and gets its rows back through a reduce-scatter
(or an all-to-all and the rank-ordered sum, ``wf_moe_sum_ranks``).  Every
rank's output meets the layer tolerance against the single-process oracle
(architecture.py:777-794); a repeated call is bit-identical.  Skipped with
fewer GPUs than ranks.
"""

import os

import numpy as np
import pytest
import torch

from oracle import fixtures as F
from oracle import moe_oracle as O
from tests import gpu_util as U
from tests.test_gpu_ep_p2p import SPEC, _free_port

pytestmark = pytest.mark.gpu


def _rank_main(rank, world, port, T, combine, q):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WF_DISABLE_TC="0", WF_FUSED="0",
                      NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from wanferenz_b200.ep import ep_forward, shard_range

        syn = F.SyntheticLayer(SPEC)
        x16, _ = syn.activations(T * world, draw=8)
        lo, hi = shard_range(SPEC.E, world, rank)
        layer = U.device_layer(syn, list(range(SPEC.E)), max_tokens=T * world, expert_range=(lo, hi))
        x = U.bf16_tensor(x16[rank * T:(rank + 1) * T])
        outs = []
        for _ in range(2):
            y = ep_forward(layer, x, combine=combine)
            outs.append(U.to_f32(y))
        torch.cuda.synchronize()
        layer.read_error()
        q.put((rank, outs))
    except Exception:  # the parent reports it
        import traceback

        q.put((rank, traceback.format_exc()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,T,combine", [(2, 8, "reduce_scatter"), (2, 8, "all_to_all"),
                                             (4, 4, "reduce_scatter")])
def test_ranks_match_oracle(world, T, combine):
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, T, combine, q)) for r in range(world)]
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
    y_ref, _, _ = O.moe_forward(xf, syn.params(), ids)
    y_ref32, _, _ = O.moe_forward(xf, syn.params(), ids, acc=np.float32)
    tie = U.near_tie_rows(xf, syn, what=f"nccl {world} ranks T={T}")
    for call in range(2):
        y = np.concatenate([res[r][call] for r in range(world)])
        U.assert_layer_close_envelope(y[~tie], y_ref[~tie], y_ref32[~tie], f"nccl {world} ranks {combine} call {call}")
    y0 = np.concatenate([res[r][0] for r in range(world)])
    y1 = np.concatenate([res[r][1] for r in range(world)])
    assert np.array_equal(y0, y1), "repeated calls differ"
