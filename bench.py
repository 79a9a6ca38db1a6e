#!/usr/bin/env python
"""Benchmark of the WANferenz MoE decode layer on B200.

Workload: DeepSeek-V4-Flash-shaped MoE layer (hidden 4096, 256 routed FP4
experts x inter 2048, 1 FP8 shared expert, top-6 sigmoid routing, route scale
1.5), random-init weights from the reference's fixture recipe (N(0, 0.02) ->
FP4 E2M1 + UE8M0 per 32; shared FP8 E4M3 per 128x128), synthetic N(0, 1) bf16
tokens.  One step = one layer forward over one batch of ``--tokens`` tokens
per GPU.  ``--layers`` distinct layers are cycled so each step's weights are
cold in L2 (8 layers x ~27 MB of router + shared weights alone > 126 MB L2);
no L2 flush is used.

N > 1 (torchrun, one rank per GPU): expert parallel, each rank holds 256/N
experts and its own ``--tokens`` tokens (weak scaling); each rank routes its
own tokens, tokens and routing are all-gathered over NCCL, every rank runs its
local experts on the gathered batch (plus the shared expert on its own rows),
and a reduce-scatter returns each rank its tokens' sums (the reference's
all-reduce, architecture.py:791-792, restricted to the owner's rows).

``--impl reference`` times the reference algorithm on the host cores, every
step a forward of all ``--tokens`` tokens: the torch CPU restatement of the
reference's path (``oracle/torch_port.py``, bit-identical to the reference on
its golden cases; the reference itself is Python/TileLang and is not
installed on the GPU box).  Both arms print the same ``config`` (the workload
identity); measurements go to ``detail`` and ``timing``.

The default line also carries, in ``detail``, the T = 1 / 4 / 16 sweep,
BASELINE config 4 (64 tokens, Zipf(1.2) routing) and config 3 (the FP8
block-scaled GEMM at M = 1 and 16); ``--no-extras`` skips the last two.

Prints ONE JSON line (rank 0).
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

D, I, E, K_TOP = 4096, 2048, 256, 6
FP4_EXPERT_BYTES = 3 * I * D // 2 + 3 * I * D // 32      # w1, w3, w2 + scales = 13,369,344
SHARED_BYTES = 3 * I * D + 3 * (I // 128) * (D // 128)    # 25,166,592 (+ e8m0 scales)
ROUTER_BYTES = E * D * 2 + E * 4
METRIC = "MoE layer tokens/s (V4-Flash decode layer: hidden 4096, 256 FP4 experts x 2048, top-6, FP8 shared)"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=("b200", "reference"))
    ap.add_argument("--tokens", type=int, default=16, help="tokens per GPU per step")
    ap.add_argument("--layers", type=int, default=8)
    ap.add_argument("--sweep", default="1,4,16", help="extra token counts measured at N=1")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--routing", default="uniform", choices=("uniform", "zipf"),
                    help="zipf: BASELINE config 4 popularity, gate bias += beta*log(rank^-1.2)")
    ap.add_argument("--zipf-beta", type=float, default=0.08)
    ap.add_argument("--replays", type=int, default=10,
                    help="timed replays of the K-step graph; the median replay gives the step time")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the config-3 and config-4 sub-results of the default line")
    ap.add_argument("--suite", default="moe", choices=("moe", "fp8_gemm"),
                    help="fp8_gemm: BASELINE config 3, the FP8 block-scaled GEMM sweep (one JSON line, N=1)")
    ap.add_argument("--ep", default="nccl", choices=("p2p", "nccl"),
                    help="N > 1: p2p = tokens, routing and partial rows moved over NVLink by the fused kernel "
                         "(wf_moe_forward_ep_p2p); nccl = route, NCCL all-gather, expert forward, NCCL combine")
    ap.add_argument("--combine", default="reduce_scatter", choices=("reduce_scatter", "all_to_all"),
                    help="--ep nccl: NCCL reduce-scatter of the partials, or all-to-all + ascending-rank sum")
    ap.add_argument("--init", default="quant", choices=("quant", "random"),
                    help="quant: N(0,0.02) weights through the FP4 quantizer; random: random FP4 bytes "
                         "with typical scales (fewer launches, for profiler captures)")
    return ap.parse_args()


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def workload_config(args, world):
    """The workload identity, the same in both arms' JSON lines (measurements go elsewhere)."""
    T = args.tokens
    if args.routing == "uniform":
        wl = f"BASELINE config 2: V4-Flash MoE decode layer, {T} tokens per GPU, uniform routing"
    else:
        wl = (f"BASELINE config 4: config-2 layer, {T} tokens per GPU, Zipf(1.2) routing "
              f"(gate bias += {args.zipf_beta} * log(rank^-1.2))")
    return {"workload": wl, "routing": args.routing, "tokens_per_gpu": T, "global_tokens": T * world,
            "hidden": D, "experts": E, "inter": I, "topk": K_TOP,
            "parallelism": f"ep{world}" if world > 1 else "single",
            "l2": f"{args.layers} distinct layers cycled (per-step weights cold in L2), no flush"}


def cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


# ---------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------
class Clocks:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.1)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------
# synthetic layers (GPU-side generation with the reference's fixture recipe)
# ---------------------------------------------------------------------------
def fp8_block_quant_torch(w):
    """fp4_grouped._fp8_block_quant (fp4_grouped.py:354-365) in torch on the GPU (fixture only)."""
    import torch

    n, k = w.shape
    b = w.float().unflatten(0, (n // 128, 128)).unflatten(-1, (k // 128, 128))
    amax = b.abs().amax(dim=(1, 3)).clamp_min(1e-4)
    scale = torch.pow(2.0, torch.ceil(torch.log2(amax / 448.0)))
    q = (b / scale[:, None, :, None]).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)
    return q.reshape(n, k).view(torch.uint8), scale.to(torch.float8_e8m0fnu).view(torch.uint8)


def make_layer(seed, rank, world, max_tokens, device, init="quant", zipf_beta=0.0):
    import torch

    from wanferenz_b200 import ops
    from wanferenz_b200.moe import MoELayer, MoEWeights

    El = E // world
    e0 = rank * El
    g = torch.Generator(device=device)
    g.manual_seed(1000 + seed)  # router + shared: identical on every rank
    gate_w = (torch.randn(E, D, device=device, generator=g) * 0.02).to(torch.bfloat16)
    gate_b = torch.randn(E, device=device, generator=g) * 0.01
    if zipf_beta > 0:
        # Zipf(s=1.2) expert popularity over a seeded permutation
        perm = torch.randperm(E, device=device, generator=g)
        rank_of = torch.empty(E, device=device)
        rank_of[perm] = torch.arange(1, E + 1, device=device, dtype=torch.float32)
        gate_b = gate_b + zipf_beta * torch.log(rank_of.pow(-1.2))
    sh = [(torch.randn(*shp, device=device, generator=g) * 0.02).to(torch.bfloat16)
          for shp in ((I, D), (I, D), (D, I))]
    q = [fp8_block_quant_torch(t) for t in sh]
    w13 = torch.empty(El, 2 * I, D // 2, dtype=torch.uint8, device=device)
    w13_s = torch.empty(El, 2 * I, D // 32, dtype=torch.uint8, device=device)
    w2 = torch.empty(El, D, I // 2, dtype=torch.uint8, device=device)
    w2_s = torch.empty(El, D, I // 32, dtype=torch.uint8, device=device)
    if init == "random":
        for t, hi in ((w13, 256), (w2, 256), (w13_s, 125), (w2_s, 125)):
            t.copy_(torch.randint(0 if hi == 256 else 118, hi, t.shape, dtype=torch.uint8, device=device,
                                  generator=g))
    for e in range(e0, e0 + El) if init == "quant" else ():
        g.manual_seed(1000003 * (seed + 1) + e)
        a = (torch.randn(2 * I, D, device=device, generator=g) * 0.02).to(torch.bfloat16)
        wq, ws = ops.fp4_act_quant(a)
        w13[e - e0].copy_(wq.view(torch.uint8)); w13_s[e - e0].copy_(ws.view(torch.uint8))
        b = (torch.randn(D, I, device=device, generator=g) * 0.02).to(torch.bfloat16)
        wq, ws = ops.fp4_act_quant(b)
        w2[e - e0].copy_(wq.view(torch.uint8)); w2_s[e - e0].copy_(ws.view(torch.uint8))
    weights = MoEWeights(gate_w=gate_w, gate_b=gate_b, tid2eid=None, w13=w13, w13_s=w13_s, w2=w2,
                         w2_s=w2_s, shared_w13=torch.cat([q[0][0], q[1][0]]),
                         shared_s13=torch.cat([q[0][1], q[1][1]]), shared_w2=q[2][0],
                         shared_s2=q[2][1])
    return MoELayer(weights, dim=D, inter_dim=I, n_experts=E, topk=K_TOP, score_func="sigmoid",
                    route_scale=1.5, n_local_experts=El, expert_offset=e0, max_tokens=max_tokens)


# ---------------------------------------------------------------------------
# algorithmic bytes per kernel for one step, from the step's routing
# ---------------------------------------------------------------------------
def tc_engine():
    """The library runs the expert phases on tcgen05 unless WF_DISABLE_TC is set (this
    benchmark's layers always have e8m0 scales, the other condition)."""
    return os.environ.get("WF_DISABLE_TC", "0") in ("", "0")


def fused_engine():
    """On tcgen05 the whole layer is one launch when WF_FUSED=1 (three launches otherwise)."""
    return tc_engine() and os.environ.get("WF_FUSED", "0") not in ("", "0")


def kernel_names():
    if fused_engine():
        return ["k_moe_fused"]
    if tc_engine():
        return ["k_moe_up", "k_moe_tc<2>", "k_moe_tc<3>"]
    return ["k_moe_up", "k_moe_mid", "k_moe_down"]


# ncu traffic (dram__bytes_read.sum + dram__bytes_write.sum) per launch of the tcgen05
# expert phases, 16 tokens, uniform routing: profiles/moe_layer_launches_config2_T16.md
MEASURED_TRAFFIC_T16 = {"k_moe_tc<2>": 728.0e6, "k_moe_tc<3>": 366.2e6}


def step_bytes(indices, T, e0, El, router=True, shared=True):
    """Bytes each kernel must move at minimum, given this step's expert indices [T, k].

    ``router=False`` drops the gate (routing given); ``shared=False`` drops the
    shared expert (its weights and its activation traffic)."""
    import numpy as np

    idx = np.asarray(indices)
    local = idx[(idx >= e0) & (idx < e0 + El)]
    n_exp = len(np.unique(local))
    pairs = sum(len(set(r[(r >= e0) & (r < e0 + El)].tolist())) for r in idx)
    w13 = 2 * I * (D // 2 + D // 32)
    w2 = D * (I // 2 + I // 32)
    s13 = (2 * I * D + 2 * (I // 128) * (D // 128)) if shared else 0
    s2 = (D * I + (D // 128) * (I // 128)) if shared else 0
    Ts = T if shared else 0
    rb = ROUTER_BYTES if router else T * idx.shape[1] * 12
    if fused_engine():
        # router + token quantization + routed and shared w1/w3 + w2 + combine, one launch
        k = (rb + T * D * 2 + T * D + T * D // 128 + n_exp * (w13 + w2) + s13 + s2 + 2 * (pairs * I + Ts * I)
             + (pairs + Ts) * D * 2 * 2 + T * D * (2 if shared else 4))
        return {"k_moe_fused": k, "experts": n_exp, "pairs": pairs}
    n1, n2, n3 = kernel_names()
    if tc_engine():
        # router + token quantization | routed + shared w1/w3 -> E4M3 hidden | w2 + combine
        k1 = rb + T * D * 2 + T * D + T * D // 128
        k2 = n_exp * w13 + s13 + T * D + pairs * I + Ts * I
        k3 = n_exp * w2 + s2 + pairs * I + Ts * I + (pairs + Ts) * D * 2 * 2 + T * D * (2 if shared else 4)
    else:
        k1 = rb + s13 + T * D * 2 + Ts * I * 2
        k2 = n_exp * w13 + s2 + T * D * 2 + pairs * I * 2 + Ts * I * 2 + Ts * D * 2
        k3 = n_exp * w2 + pairs * I * 2 + pairs * D * 2 * 2 + T * D * 2 * 2
    return {n1: k1, n2: k2, n3: k3, "experts": n_exp, "pairs": pairs}


EP_PHASES = ["route", "all_gather", "experts", "combine", "to_bf16"]


def p2p_step_bytes(idx_g, Tloc, world, e0, El):
    """Bytes of one expert-parallel step over peer memory, per rank: the router over
    the rank's own tokens, its local experts on the gathered batch, the shared expert
    on its own rows, the tokens / routing / partial rows it sends over NVLink and the
    finish's reads."""
    rt = step_bytes(idx_g, Tloc * world, e0, El, router=False, shared=False)
    s13 = 2 * I * D + 2 * (I // 128) * (D // 128)
    s2 = D * I + (D // 128) * (I // 128)
    sent = (world - 1) * Tloc * (D + D // 128 + 8 * K_TOP) + (world - 1) * Tloc * D * 4
    k = (ROUTER_BYTES + Tloc * D * 2 + sum(rt[n] for n in kernel_names()) + s13 + s2 + Tloc * (I * 2 + D * 2 * 2)
         + sent + world * Tloc * D * 4 + Tloc * D * 2)
    return {"ep_step": k, "experts_touched": rt["experts"], "pairs": rt["pairs"], "nvlink_bytes_sent": sent}


def ep_step_bytes(idx_g, Tloc, world, e0, El, combine="reduce_scatter"):
    """Per-phase bytes of one expert-parallel step (``wanferenz_b200.ep.ep_forward``)."""
    import numpy as np

    rt = step_bytes(idx_g, Tloc * world, e0, El, router=False, shared=False)
    names = kernel_names()
    s13 = 2 * I * D + 2 * (I // 128) * (D // 128)
    s2 = D * I + (D // 128) * (I // 128)
    tok = 2 * D + 12 * K_TOP
    # shared expert on the Tloc own rows: its weights, hidden and output rows
    shared = s13 + s2 + Tloc * (I * 2 + D * 2 * 2)
    return {"route": ROUTER_BYTES + Tloc * D * 2 + Tloc * K_TOP * 12,
            "all_gather": (world - 1) * Tloc * tok,            # bytes each rank receives
            "experts": sum(rt[k] for k in names) + shared,
            "combine": (world - 1) * Tloc * D * 4,             # bytes each rank receives
            "to_bf16": Tloc * D * ((4 * world if combine == "all_to_all" else 4) + 2),
            "experts_touched": rt["experts"], "pairs": rt["pairs"]}


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def run_gpu(args):
    import ctypes

    import numpy as np
    import torch
    import torch.distributed as dist

    from wanferenz_b200 import _lib as L
    from wanferenz_b200 import ep

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dom_name = None
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        # NCCL's version banner would go to stdout ahead of the result line
        os.environ["NCCL_DEBUG"] = "WARN"
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
    T = args.tokens
    Tg = T * world
    zb = args.zipf_beta if args.routing == "zipf" else 0.0
    layers = [make_layer(s, rank, world, max(Tg, 16), dev, args.init, zb) for s in range(args.layers)]
    lib = L.load()
    peers = [ep.PeerGroup(lay) for lay in layers] if world > 1 and args.ep == "p2p" else []
    hbm, peak_kind = peaks()
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()

    def measure(lays, Tloc, K, W, R):
        """K graph-captured steps replayed R times (headline: the median replay) + K eager
        steps with per-kernel events."""
        n = K + W
        Tgl = Tloc * world
        xs = [torch.randn(Tloc, D, device=dev).to(torch.bfloat16) for _ in range(n)]
        ys = [torch.empty(Tloc, D, dtype=torch.bfloat16, device=dev) for _ in range(n)]
        idx = [torch.empty(Tgl, K_TOP, dtype=torch.int64, device=dev) for _ in range(n)]
        evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(n)]
        for row in evs:  # torch creates the CUDA event on first record
            for e in row:
                e.record()
        xg = [torch.empty(Tgl, D, dtype=torch.bfloat16, device=dev) for _ in range(n)]
        wg = [torch.empty(Tgl, K_TOP, dtype=torch.float32, device=dev) for _ in range(n)]
        part = [torch.empty(Tgl, D, dtype=torch.float32, device=dev) for _ in range(n)]
        mine = [torch.empty(Tloc, D, dtype=torch.float32, device=dev) for _ in range(n)]
        recv = ([torch.empty(world, Tloc, D, dtype=torch.float32, device=dev) for _ in range(n)]
                if args.combine == "all_to_all" else None)
        rw = [torch.empty(Tloc, K_TOP, dtype=torch.float32, device=dev) for _ in range(n)]
        ri = [torch.empty(Tloc, K_TOP, dtype=torch.int64, device=dev) for _ in range(n)]
        pev = [[torch.cuda.Event(enable_timing=True) for _ in range(len(EP_PHASES) + 1)] for _ in range(n)]

        def one_ep(i, timed=False):
            """``wanferenz_b200.ep.ep_forward`` through the C ABI."""
            lay = lays[i % len(lays)]
            st = L.stream_ptr()
            cfg, wst, ws, wsn = ctypes.byref(lay.cfg), ctypes.byref(lay.wstruct), L.ptr(lay.workspace), \
                lay.workspace.numel()
            ev = pev[i] if timed else None
            if ev:
                ev[0].record()
            L.check(lib.wf_moe_route(cfg, wst, L.ptr(xs[i]), None, Tloc, L.ptr(rw[i]), L.ptr(ri[i]), ws, wsn, st),
                    "wf_moe_route")
            if ev:
                ev[1].record()
            ep.gather_tokens(xs[i], rw[i], ri[i], xg[i], wg[i], idx[i])
            if ev:
                ev[2].record()
            L.check(lib.wf_moe_forward_ep(cfg, wst, L.ptr(xg[i]), Tgl, L.ptr(wg[i]), L.ptr(idx[i]), rank * Tloc,
                                          Tloc, L.ptr(part[i]), ws, wsn, st), "wf_moe_forward_ep")
            if ev:
                ev[3].record()
            if recv is None:
                dist.reduce_scatter_tensor(mine[i], part[i])
            else:
                dist.all_to_all_single(recv[i], part[i])
            if ev:
                ev[4].record()
            if recv is None:
                L.check(lib.wf_moe_to_bf16(L.ptr(mine[i]), Tloc * D, L.ptr(ys[i]), st), "wf_moe_to_bf16")
            else:
                L.check(lib.wf_moe_sum_ranks(L.ptr(recv[i]), world, Tloc * D, L.ptr(ys[i]), st), "wf_moe_sum_ranks")
            if ev:
                ev[5].record()

        def one_p2p(i, timed=False):
            """``wanferenz_b200.ep.PeerGroup.forward``: one call, the fused kernel and the finish."""
            ev = pev[i] if timed else None
            if ev:
                ev[0].record()
            peers[i % len(peers)].forward(xs[i], out=ys[i], out_routing=(rw[i], ri[i]))
            if ev:
                ev[1].record()

        def one(i, timed=False):
            if world > 1:
                return one_p2p(i, timed) if args.ep == "p2p" else one_ep(i, timed)
            lay = lays[i % len(lays)]
            st = L.stream_ptr()
            ev = (ctypes.c_void_p * 4)(*[ctypes.c_void_p(e.cuda_event) for e in evs[i]])
            args_ = (ctypes.byref(lay.cfg), ctypes.byref(lay.wstruct), L.ptr(xs[i]), 0, Tloc,
                     L.ptr(ys[i]), 0, 0, L.ptr(idx[i]), L.ptr(lay.workspace), lay.workspace.numel(), st)
            if timed:
                L.check(lib.wf_moe_forward_timed(*args_, ev), "wf_moe_forward_timed")
            else:
                L.check(lib.wf_moe_forward(*args_), "wf_moe_forward")

        for i in range(W):
            one(i)
        torch.cuda.synchronize()
        # the K timed steps as one CUDA graph (NCCL collectives included for N > 1;
        # every rank captures the same sequence), so host launch gaps stay out
        g = torch.cuda.CUDAGraph()
        n0 = lib.wf_launch_count()
        with torch.cuda.graph(g):
            for i in range(W, n):
                one(i)
        launches = int(lib.wf_launch_count() - n0)  # this library's kernels in one replay
        g.replay()  # one untimed replay (graph upload)
        torch.cuda.synchronize()
        t0 = [torch.cuda.Event(enable_timing=True) for _ in range(R)]
        t1 = [torch.cuda.Event(enable_timing=True) for _ in range(R)]
        with Clocks(local) as clk:
            for r in range(R):
                barrier()
                torch.cuda.synchronize()
                t0[r].record()
                g.replay()
                t1[r].record()
                torch.cuda.synchronize()
            barrier()
        reps = [t0[r].elapsed_time(t1[r]) for r in range(R)]
        # per-kernel durations: eager steps queued behind ~2 ms of copies, so the
        # host runs ahead of the GPU and no launch gap falls inside a kernel's events
        big = torch.empty(1 << 30, dtype=torch.uint8, device=dev)
        for _ in range(10):
            big.add_(1)
        if world > 1:
            # the ranks' queues line up here on the device, so the first timed
            # collective does not absorb their skew
            dist.all_reduce(torch.zeros(1, device=dev))
        for i in range(W, n):
            one(i, timed=True)
        torch.cuda.synchronize()
        del big
        names = kernel_names() if world == 1 else (["ep_step"] if args.ep == "p2p" else EP_PHASES)
        kern = {k: [] for k in names}
        for i in range(W, n):
            e = evs[i] if world == 1 else pev[i]
            for j, k in enumerate(names):
                kern[k].append(e[j].elapsed_time(e[j + 1]))
        if world > 1 and args.ep == "p2p":
            # this rank's routing of its own tokens; the accounting wants the gathered batch's
            for i in range(W, n):
                dist.all_gather_into_tensor(idx[i], ri[i])
        routing = [idx[i].cpu().numpy() for i in range(W, n)]
        del g
        return reps, kern, routing, clk.summary(), launches

    def stats(lays, Tloc, K, W, R=1):
        reps, kern, routing, clk, launches = measure(lays, Tloc, K, W, R)
        t = torch.tensor(reps, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)  # per replay, the slowest rank
        reps = sorted(float(v) for v in t.tolist())
        total_ms = reps[len(reps) // 2]  # median replay of K steps
        ms = total_ms / K
        lay0 = lays[0]
        if world == 1:
            byts = [step_bytes(r, Tloc, lay0.expert_offset, lay0.n_local_experts) for r in routing]
        elif args.ep == "p2p":
            byts = [p2p_step_bytes(r, Tloc, world, lay0.expert_offset, lay0.n_local_experts) for r in routing]
        else:
            byts = [ep_step_bytes(r, Tloc, world, lay0.expert_offset, lay0.n_local_experts, args.combine)
                    for r in routing]
        mean = {k: float(np.mean([b[k] for b in byts])) for k in byts[0]}
        kms = {k: float(np.mean(v)) for k, v in kern.items()}
        layer_bytes = sum(mean[k] for k in (kernel_names() if world == 1 else
                                            (["ep_step"] if args.ep == "p2p" else ["route", "experts", "to_bf16"])))
        hist = [np.bincount(r.ravel(), minlength=E) for r in routing]
        tpe = {"experts_empty": float(np.mean([(h == 0).sum() for h in hist])),
               "experts_over_16": float(np.mean([(h > 16).sum() for h in hist])),
               "max_tokens_per_expert": float(np.mean([h.max() for h in hist]))}
        return dict(ms=ms, total_ms=total_ms, reps_ms=reps, kms=kms, bytes=mean, layer_bytes=layer_bytes,
                    clocks=clk, tpe=tpe, launches=launches)

    def summary(r, Tloc):
        gbs = r["layer_bytes"] / (r["ms"] * 1e-3) / 1e9
        return {"us_per_step": round(r["ms"] * 1e3, 2), "tokens_per_s": round(Tloc * world / (r["ms"] * 1e-3), 1),
                "layer_GBps": round(gbs, 1), "layer_frac_of_measured_hbm": round(gbs / hbm, 3),
                "experts_touched": round(r["bytes"]["experts" if world == 1 else "experts_touched"], 1),
                "tokens_per_expert": r["tpe"],
                "kernel_us": {k: round(v * 1e3, 2) for k, v in r["kms"].items()}}

    main = stats(layers, T, args.steps, args.warmup, args.replays)
    sweep = {}
    extras = {}
    if world == 1:
        for s_ in [int(v) for v in args.sweep.split(",") if v]:
            r = main if s_ == T else stats(layers, s_, args.steps, args.warmup)
            sweep[f"T{s_}"] = summary(r, s_)
        if not args.no_extras and args.routing == "uniform":
            # 64 tokens, Zipf(1.2) popularity, on layers of its own
            zl = [make_layer(s_, 0, 1, 64, dev, args.init, args.zipf_beta) for s_ in range(args.layers)]
            extras["config4_T64_zipf"] = summary(stats(zl, 64, args.steps, args.warmup), 64)
            del zl
            torch.cuda.empty_cache()
            # the FP8 block-scaled GEMM at M = 1 and 16; the
            # attention's dense projections on the same GEMM (model path, e8m0)
            extras["config3_fp8_gemm"] = fp8_gemm_points((1, 16), hbm)
            extras["attention_fp8_projections"] = fp8_gemm_points((1, 16), hbm, ATTN_PROJECTIONS, ("e8m0",))
    # dominant kernel roofline
    kms = main["kms"]
    # the dominant HBM-bound kernel (multi-GPU: of the compute phases; the collectives
    # are reported in kernel_us beside them)
    dom = max((k for k in kms if k not in ("all_gather", "combine")), key=kms.get)
    if dom == "ep_step":
        dom_name = "k_moe_fused + k_ep_finish (expert parallelism over peer memory)"
    ach = main["bytes"][dom] / (kms[dom] * 1e-3) / 1e9
    value = T * world / (main["ms"] * 1e-3)
    traffic, traffic_src = None, None
    if dom in MEASURED_TRAFFIC_T16 and T == 16 and world == 1 and args.routing == "uniform":
        traffic = MEASURED_TRAFFIC_T16[dom]
        traffic_src = ("ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch, same workload "
                       "(1 layer, random FP4 bytes): profiles/moe_layer_launches_config2_T16.md")

    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(layers, T, args.steps, args.warmup, dev, world, rank, args.combine, peers)
    out = {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(main["ms"], 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "e2m1/e4m3 x e4m3 -> f32",
        "data": "synthetic (seeded N(0,0.02) weights quantized like the reference fixtures; N(0,1) bf16 tokens)",
        "config": workload_config(args, world),
        "timing": {"method": ("CUDA graph of the K steps" + (" (NCCL collectives captured)" if world > 1 else "") +
                              ", replayed R times, each replay bracketed by a barrier and a device synchronize "
                              "and timed with CUDA events on the launching stream; the step time is the median "
                              "replay / K" + (" (each replay's time the max over ranks)" if world > 1 else "")),
                   "replays": args.replays, "replay_ms": [round(v, 4) for v in main["reps_ms"]]},
        "detail": {**summary(main, T), "ep": args.ep if world > 1 else None,
                   "combine": args.combine if world > 1 and args.ep == "nccl" else None,
                   "sweep": sweep, **extras},
        "roofline": {"bound": "hbm", "kernel": dom_name if dom == "ep_step" else dom, "achieved": round(ach, 1),
                     "peak": hbm,
                     "peak_kind": peak_kind, "unit": "GB/s", "frac": round(ach / hbm, 4),
                     "traffic": traffic, "traffic_source": traffic_src,
                     "algorithmic_bytes_per_launch": round(main["bytes"][dom])},
        "clocks": main["clocks"],
        # counted: this library's kernels recorded into the graph of the K timed steps
        "gpu_launches": main["launches"],
        "e2e": e2e,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline(T)
    for pg in peers:
        pg.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(out), flush=True)


def run_e2e(layers, T, K, W, dev, world, rank, combine="reduce_scatter", peers=()):
    """Public API (MoELayer.forward), host pinned input -> device -> host output every step.

    A serving loop's pipelining: the copies run on their own stream, so step i's
    output copy and step i+1's input copy overlap step i's compute (two device
    input buffers; each copy and forward waits on the events it depends on).
    The timed region ends once the last output is on the host."""
    import torch
    import torch.distributed as dist

    if world > 1:
        return run_e2e_graphs(layers, T, K, W, dev, world, combine, peers)
    n = K + W
    xh = [torch.randn(T, D).to(torch.bfloat16).pin_memory() for _ in range(n)]
    yh = [torch.empty(T, D, dtype=torch.bfloat16).pin_memory() for _ in range(n)]
    xd = [torch.empty(T, D, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    main = torch.cuda.current_stream(dev)
    cs = torch.cuda.Stream(dev)
    x_in = [torch.cuda.Event() for _ in range(2)]    # input i % 2 landed
    x_free = [torch.cuda.Event() for _ in range(2)]  # forward i % 2 done reading it
    y_ok = torch.cuda.Event()

    def h2d(i):
        b = i % 2
        with torch.cuda.stream(cs):
            if i >= 2:
                cs.wait_event(x_free[b])
            xd[b].copy_(xh[i], non_blocking=True)
            x_in[b].record(cs)

    def one(i, prefetch=True):
        lay = layers[i % len(layers)]
        b = i % 2
        main.wait_event(x_in[b])
        if world == 1:
            y = lay.forward(xd[b])
        elif peers:
            y = peers[i % len(peers)].forward(xd[b])
        else:
            from wanferenz_b200.ep import ep_forward
            y = ep_forward(lay, xd[b], combine=combine)
        x_free[b].record(main)
        if prefetch and i + 1 < n:
            h2d(i + 1)
        y_ok.record(main)
        with torch.cuda.stream(cs):
            cs.wait_event(y_ok)
            yh[i].copy_(y, non_blocking=True)
            y.record_stream(cs)

    h2d(0)
    for i in range(W):
        one(i, prefetch=i + 1 < W)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    done = torch.cuda.Event()
    # every timed step's input and output copies lie between t0 and t1
    t0.record(main)
    cs.wait_event(t0)
    h2d(W)
    for i in range(W, n):
        one(i)
    done.record(cs)
    main.wait_event(done)
    t1.record(main)
    torch.cuda.synchronize()
    ms = torch.tensor([t0.elapsed_time(t1)], device=dev)
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms = float(ms.item()) / K
    return {"value": round(T * world / (ms * 1e-3), 1), "unit": "tokens/s",
            "us_per_step": round(ms * 1e3, 2), "h2d_bytes_per_step": T * D * 2,
            "d2h_bytes_per_step": T * D * 2, "copies": "own stream, overlapped with compute",
            "api": ("wanferenz_b200.moe.MoELayer.forward" if world == 1 else
                    "wanferenz_b200.ep.PeerGroup.forward" if peers else "wanferenz_b200.ep.ep_forward")}


def run_e2e_graphs(layers, T, K, W, dev, world, combine="reduce_scatter", peers=()):
    """run_e2e for N > 1 ranks: each layer's public call (``ep.ep_forward`` or
    ``PeerGroup.forward``, exchange included) is captured once in a CUDA graph, as a
    serving loop would, and replayed every step; the host copies stay outside the
    graphs, on their own stream, overlapping the previous step's compute.  Every
    rank captures and replays the same sequence."""
    import torch
    import torch.distributed as dist

    n = K + W
    nl = len(layers)
    xh = [torch.randn(T, D).to(torch.bfloat16).pin_memory() for _ in range(n)]
    yh = [torch.empty(T, D, dtype=torch.bfloat16).pin_memory() for _ in range(n)]
    xin = [torch.empty(T, D, dtype=torch.bfloat16, device=dev) for _ in range(nl)]

    def fwd(l):
        if peers:
            return peers[l].forward(xin[l])
        from wanferenz_b200.ep import ep_forward
        return ep_forward(layers[l], xin[l], combine=combine)

    for l in range(nl):  # eager first: lazy initialisation stays out of the capture
        fwd(l)
    torch.cuda.synchronize()
    graphs, yout = [], []
    for l in range(nl):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            yout.append(fwd(l))
        graphs.append(g)
    torch.cuda.synchronize()
    main = torch.cuda.current_stream(dev)
    cs = torch.cuda.Stream(dev)
    x_in = [torch.cuda.Event() for _ in range(nl)]
    x_free = [torch.cuda.Event() for _ in range(nl)]
    y_ok = [torch.cuda.Event() for _ in range(nl)]
    y_free = [torch.cuda.Event() for _ in range(nl)]
    used = [False] * nl

    def h2d(i):
        l = i % nl
        with torch.cuda.stream(cs):
            if used[l]:
                cs.wait_event(x_free[l])
            xin[l].copy_(xh[i], non_blocking=True)
            x_in[l].record(cs)

    def one(i, prefetch=True):
        l = i % nl
        main.wait_event(x_in[l])
        if used[l]:
            main.wait_event(y_free[l])  # the previous output copy of this graph is done
        graphs[l].replay()
        used[l] = True
        x_free[l].record(main)
        y_ok[l].record(main)
        if prefetch and i + 1 < n:
            h2d(i + 1)
        with torch.cuda.stream(cs):
            cs.wait_event(y_ok[l])
            yh[i].copy_(yout[l], non_blocking=True)
            y_free[l].record(cs)

    h2d(0)
    for i in range(W):
        one(i, prefetch=i + 1 < W)
    torch.cuda.synchronize()
    dist.barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    done = torch.cuda.Event()
    t0.record(main)
    cs.wait_event(t0)
    h2d(W)
    for i in range(W, n):
        one(i)
    done.record(cs)
    main.wait_event(done)
    t1.record(main)
    torch.cuda.synchronize()
    ms = torch.tensor([t0.elapsed_time(t1)], device=dev)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms = float(ms.item()) / K
    del graphs, yout  # graphs holding NCCL calls go before the process group
    torch.cuda.synchronize()
    return {"value": round(T * world / (ms * 1e-3), 1), "unit": "tokens/s",
            "us_per_step": round(ms * 1e3, 2), "h2d_bytes_per_step": T * D * 2,
            "d2h_bytes_per_step": T * D * 2,
            "copies": "own stream, overlapped with compute; each layer's call replayed from a CUDA graph",
            "api": "wanferenz_b200.ep.PeerGroup.forward" if peers else "wanferenz_b200.ep.ep_forward"}


# ---------------------------------------------------------------------------
# CPU legs: the oracle port of the reference's torch CPU path
# ---------------------------------------------------------------------------
def cpu_layer(seed=0):
    """Oracle-side layer with the config-2 shapes; expert bytes random (cost does not depend on values)."""
    import numpy as np

    from oracle import fixtures as F

    spec = F.CONFIG2
    syn = F.SyntheticLayer(F.LayerSpec(**{**spec.as_dict(), "seed": seed}))
    cache = {}
    r = np.random.default_rng(seed)

    def expert(e):
        if e not in cache:
            cache[e] = (r.integers(0, 256, (I, D // 2), dtype=np.uint8),
                        r.integers(118, 125, (I, D // 32), dtype=np.uint8),
                        r.integers(0, 256, (I, D // 2), dtype=np.uint8),
                        r.integers(118, 125, (I, D // 32), dtype=np.uint8),
                        r.integers(0, 256, (D, I // 2), dtype=np.uint8),
                        r.integers(118, 125, (D, I // 32), dtype=np.uint8))
        return cache[e]

    sh = (r.integers(0, 126, (I, D), dtype=np.uint8), r.integers(118, 125, (I // 128, D // 128), dtype=np.uint8),
          r.integers(0, 126, (I, D), dtype=np.uint8), r.integers(118, 125, (I // 128, D // 128), dtype=np.uint8),
          r.integers(0, 126, (D, I), dtype=np.uint8), r.integers(118, 125, (D // 128, I // 128), dtype=np.uint8))
    params = syn.params()
    params["experts"] = expert
    params["shared"] = sh
    return syn, params


def cpu_forward_time(T, reps=1, seed=0, warmup=0):
    """Seconds per config-2 layer forward of T tokens by the torch CPU restatement of the
    reference's path (``oracle/torch_port.py``: the reference's ops, all host threads)."""
    import torch

    from oracle import moe_oracle as O
    from oracle import torch_port as P

    torch.set_num_threads(os.cpu_count())
    syn, params = cpu_layer(seed)
    times = []
    for rep in range(warmup + reps):
        x16, _ = syn.activations(T, draw=100 + rep)
        x = O.bf16_to_f32(x16)
        # the synthetic expert bytes are made on first use: outside the timed region
        _, idx = P.gate(P._t(x), params)
        for e in idx.unique().tolist():
            params["experts"](e)
        t = time.perf_counter()
        P.moe_forward(x, params)
        if rep >= warmup:
            times.append(time.perf_counter() - t)
    return times


def cpu_baseline(T):
    import numpy as np

    t = cpu_forward_time(T, reps=2, warmup=1)
    s = float(np.median(t))
    return {"value": round(T / s, 3), "unit": "tokens/s", "cores": os.cpu_count(), "cpu_model": cpu_model(),
            "kind": "port",
            "sample": f"config-2 layer forwards of {T} tokens (median of 2 after 1 warm-up) by the torch "
                      f"CPU restatement of the reference's path (oracle/torch_port.py: the reference's "
                      f"ops, fp32 BLAS, {os.cpu_count()} host threads); {s:.2f} s each"}


def run_reference(args):
    """--impl reference: the reference algorithm (the torch restatement of its CPU path)
    on the host cores, every step a forward of all ``--tokens`` tokens of the workload."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    T = args.tokens
    cpu_forward_time(T, reps=0, warmup=max(args.warmup, 1), seed=1)
    times = cpu_forward_time(T, reps=args.steps, seed=2)
    s = sum(times) / len(times)
    value = T / s
    sample = (f"all {T} tokens of each step through the torch CPU restatement of the reference's "
              f"MoE.forward (oracle/torch_port.py; the reference's ops, fp32 BLAS, "
              f"{os.cpu_count()} host threads on {cpu_model()})")
    out = {
        "metric": METRIC, "value": round(value, 3), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(s * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "impl": "reference",
        "config": workload_config(args, world),
        "cpu_baseline": {"value": round(value, 3), "unit": "tokens/s", "cores": os.cpu_count(),
                         "cpu_model": cpu_model(), "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out), flush=True)


# the attention's dense FP8 projections the reference routes to the same GEMM
# (fp8_vector.py:505-513), (name, N, K)
ATTN_PROJECTIONS = (("attn.wq_a", 1024, 4096), ("attn.wkv", 512, 4096), ("attn.wq_b", 32768, 1024),
                    ("attn.wo_b", 4096, 8192), ("idx.wq_b", 8192, 1024))
CONFIG3_SHAPES = (("config3", 4096, 4096), ("config3", 12288, 4096), ("config3", 4096, 16384),
                  ("config3", 129280, 4096))


def fp8_gemm_points(Ms, hbm, shapes=CONFIG3_SHAPES, kinds=("f32", "e8m0")):
    """``fp8_gemm`` (architecture.py:121-134 -> torch_ops.py:93-99) for
    the M in ``Ms`` and the four (N, K) of the model's dense projections, E4M3 weights
    with one fp32 (config 3) or e8m0 (model path) scale per 128x128 block, bf16
    activations quantized per token (1x128 scales).  Each point: R calls cycling
    enough weight copies to exceed L2, captured in a CUDA graph, replayed and timed
    with CUDA events.  Bytes per call: N*K + scales + M*K*2 + M*N*2."""
    import torch

    from wanferenz_b200 import ops

    dev = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    res = []
    for (name, N, K) in shapes:
        w = (torch.randn(N, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        q, s8 = fp8_block_quant_torch(w)
        del w
        s32 = s8.view(torch.float8_e8m0fnu).float()
        wq = q.view(torch.float8_e4m3fn)
        copies = max(1, -(-300_000_000 // (N * K)))
        wqs = [wq] + [wq.clone() for _ in range(copies - 1)]
        # f32: config 3 as stated (fp32 scales on both sides); e8m0: the model path
        # (scale_fmt="ue8m0", e8m0 scales on both sides, architecture.py:121-134)
        for kind, bs in (("f32", s32), ("e8m0", s8.view(torch.float8_e8m0fnu))):
            if kind not in kinds:
                continue
            for M in Ms:
                x = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
                if kind == "f32":
                    aq, a_s = ops.act_quant(x, 128)
                else:
                    aq, a_s = ops.act_quant(x, 128, scale_fmt="ue8m0", scale_dtype=torch.float8_e8m0fnu)
                R = 4 * copies if copies > 1 else 8
                for _ in range(3):  # warm-up (workspace growth, module load)
                    ops.fp8_gemm(aq, a_s, wqs[0], bs)
                torch.cuda.synchronize()
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph):
                    for r in range(R):
                        ops.fp8_gemm(aq, a_s, wqs[r % copies], bs)
                graph.replay()
                torch.cuda.synchronize()
                t0 = torch.cuda.Event(enable_timing=True)
                t1 = torch.cuda.Event(enable_timing=True)
                reps = 5
                t0.record()
                for _ in range(reps):
                    graph.replay()
                t1.record()
                torch.cuda.synchronize()
                us = t0.elapsed_time(t1) * 1e3 / (reps * R)
                del graph
                nbytes = N * K + (N // 128) * (K // 128) * (4 if kind == "f32" else 1) + M * K * 2 + M * N * 2
                gbs = nbytes / (us * 1e-6) / 1e9
                res.append({"shape": name, "N": N, "K": K, "M": M, "scale": kind, "us": round(us, 2),
                            "GBps": round(gbs, 1), "frac": round(gbs / hbm, 3)})
        del wqs, wq, q, s8, s32
        torch.cuda.empty_cache()
    return res


def run_fp8_gemm_suite(args):
    """``--suite fp8_gemm``: the whole config-3 sweep, M in {1, 2, 4, 8, 16}, one JSON line."""
    import torch

    torch.cuda.set_device(0)
    hbm, peak_kind = peaks()
    res = fp8_gemm_points((1, 2, 4, 8, 16), hbm)
    res += fp8_gemm_points((1, 4, 16), hbm, ATTN_PROJECTIONS, ("e8m0",))
    out = {"suite": "fp8_gemm", "metric": "FP8 block-scaled GEMM us/call (BASELINE config 3; the attention "
                                          "projections of fp8_vector.py:505-513)",
           "unit": "us", "higher_is_better": False, "peak_GBps": hbm, "peak_kind": peak_kind,
           "timing": "CUDA graph of R calls over weight copies > L2, CUDA events", "results": res}
    print(json.dumps(out), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    elif args.suite == "fp8_gemm":
        run_fp8_gemm_suite(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
