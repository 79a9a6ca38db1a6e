"""The MoE decode layer on the B200 kernels, and the drop-in for the reference model.

``MoELayer`` owns one layer's device weights (in the reference's bank layout,
wanferenz/kernels/fp4_grouped.py:136-201) and workspace, and runs
``MoE.forward`` (wanferenz/model/architecture.py:777-794) as one
``wf_moe_forward`` call: router, routed FP4 SwiGLU experts, FP8 shared expert
and the ascending-expert combine, in three kernel launches with no host sync
and no allocation, so a forward can be captured in a CUDA graph.

``bank_layout(module)`` and ``install(mod)`` mirror the reference's plugin
interface (``fp4_grouped.bank_layout`` 191-201 and ``install`` 339-351): the
first stacks every MoE's experts into a load-time bank, the second replaces
``mod.MoE.forward`` with ``b200_forward`` (marker attribute ``_wf_b200``) and
keeps the replaced function in ``_REF_FORWARD``.
"""

from __future__ import annotations

import ctypes
import dataclasses
from typing import Optional

import torch

from . import _lib as L

_REF_FORWARD = None
_MOD = None


class WfUnsupported(RuntimeError):
    """The layer's configuration is outside what the B200 kernels implement."""


@dataclasses.dataclass
class MoEWeights:
    """Device tensors of one layer (shapes use D, I, E, E_local, k)."""

    gate_w: torch.Tensor                 # [E, D] bf16
    gate_b: Optional[torch.Tensor]       # [E] f32, None on hash layers
    tid2eid: Optional[torch.Tensor]      # [vocab, k] int32 on hash layers
    w13: torch.Tensor                    # [E_local, 2I, D/2] uint8 packed E2M1 (w1 rows, w3 rows)
    w13_s: torch.Tensor                  # [E_local, 2I, D/32] uint8 e8m0
    w2: torch.Tensor                     # [E_local, D, I/2] uint8
    w2_s: torch.Tensor                   # [E_local, D, I/32] uint8
    shared_w13: torch.Tensor             # [2I, D] uint8 e4m3 (w1 rows, w3 rows)
    shared_s13: torch.Tensor             # [2I/128, D/128] uint8 e8m0 or f32
    shared_w2: torch.Tensor              # [D, I] uint8 e4m3
    shared_s2: torch.Tensor              # [D/128, I/128] uint8 e8m0 or f32


def _u8(t):
    return t.contiguous().view(torch.uint8) if t.dtype != torch.uint8 else t.contiguous()


def _scale(t):
    if t.dtype == torch.float32:
        return t.contiguous()
    return _u8(t)


class MoELayer:
    """One MoE layer's weights + workspace; ``forward`` is the whole layer."""

    def __init__(self, weights: MoEWeights, *, dim, inter_dim, n_experts, topk, score_func="sigmoid",
                 route_scale=1.0, swiglu_limit=0.0, hash_layer=False, vocab=0, ue8m0=True,
                 n_local_experts=None, expert_offset=0, max_tokens=64, check_scales=True):
        self.lib = L.load()
        self.dim, self.inter_dim, self.n_experts, self.topk = dim, inter_dim, n_experts, topk
        self.n_local_experts = n_local_experts or n_experts
        self.expert_offset = expert_offset
        self.hash_layer = bool(hash_layer)
        self.max_tokens = max_tokens
        w = weights
        self.weights = dataclasses.replace(
            w,
            gate_w=w.gate_w.contiguous(),
            gate_b=None if w.gate_b is None else w.gate_b.float().contiguous(),
            tid2eid=None if w.tid2eid is None else w.tid2eid.to(torch.int32).contiguous(),
            w13=_u8(w.w13), w13_s=_u8(w.w13_s), w2=_u8(w.w2), w2_s=_u8(w.w2_s),
            shared_w13=_u8(w.shared_w13), shared_s13=_scale(w.shared_s13),
            shared_w2=_u8(w.shared_w2), shared_s2=_scale(w.shared_s2))
        w = self.weights
        self.device = w.w13.device
        if score_func not in L.WF_SCORE:
            raise WfUnsupported(f"score_func {score_func!r}")
        self.cfg = L.MoeConfig(dim=dim, inter_dim=inter_dim, n_experts=n_experts,
                               n_local_experts=self.n_local_experts, expert_offset=expert_offset,
                               topk=topk, score_func=L.WF_SCORE[score_func],
                               hash_layer=int(self.hash_layer), ue8m0=int(ue8m0),
                               max_tokens=max_tokens, vocab=int(vocab),
                               route_scale=float(route_scale), swiglu_limit=float(swiglu_limit))
        shared_kind = L.WF_SCALE_F32 if w.shared_s13.dtype == torch.float32 else L.WF_SCALE_E8M0
        self.wstruct = L.MoeWeights(
            gate_w=L.ptr(w.gate_w), gate_bias=L.ptr(w.gate_b), tid2eid=L.ptr(w.tid2eid),
            w13=L.ptr(w.w13), w13_s=L.ptr(w.w13_s), w2=L.ptr(w.w2), w2_s=L.ptr(w.w2_s),
            shared_w13=L.ptr(w.shared_w13), shared_s13=L.ptr(w.shared_s13),
            shared_w2=L.ptr(w.shared_w2), shared_s2=L.ptr(w.shared_s2),
            shared_scale_kind=shared_kind)
        nbytes = self.lib.wf_moe_workspace_bytes(ctypes.byref(self.cfg))
        if nbytes == 0:
            raise WfUnsupported(f"configuration rejected: {self.lib.wf_last_error().decode()}")
        # zero-filled once: the kernels leave their counters at zero after every call
        self.workspace = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
        self._check_shapes()
        if check_scales:
            for s in (w.w13_s, w.w2_s):
                ok = self.lib.wf_fp4_scales_in_range(L.ptr(s), s.numel(), L.stream_ptr())
                if ok < 0:
                    L.check(ok, "wf_fp4_scales_in_range")
                if ok == 0:
                    raise WfUnsupported("FP4 weight scales contain e8m0 byte 0 (2^-127) or 255 (NaN)")

    def _check_shapes(self):
        w, D, I = self.weights, self.dim, self.inter_dim
        El = self.n_local_experts
        want = {
            "gate_w": (w.gate_w, (self.n_experts, D)),
            "w13": (w.w13, (El, 2 * I, D // 2)), "w13_s": (w.w13_s, (El, 2 * I, D // 32)),
            "w2": (w.w2, (El, D, I // 2)), "w2_s": (w.w2_s, (El, D, I // 32)),
            "shared_w13": (w.shared_w13, (2 * I, D)), "shared_w2": (w.shared_w2, (D, I)),
            "shared_s13": (w.shared_s13, (2 * I // 128, D // 128)),
            "shared_s2": (w.shared_s2, (D // 128, I // 128)),
        }
        for name, (t, shape) in want.items():
            if tuple(t.shape) != shape:
                raise WfUnsupported(f"{name} has shape {tuple(t.shape)}, expected {shape}")
            if t.device != self.device:
                raise WfUnsupported(f"{name} is on {t.device}, expected {self.device}")
        if w.gate_w.dtype != torch.bfloat16:
            raise WfUnsupported("gate weight must be bf16")

    # ------------------------------------------------------------------
    def forward(self, x, input_ids=None, *, partial=False, out=None, routing=False):
        """``MoE.forward`` on ``x [T, D]`` bf16 (architecture.py:777-794).

        ``partial=True`` returns the local experts' fp32 routed sum instead
        (expert-parallel mode; finish with ``finish``).  ``routing=True`` also
        returns the router's ``(weights [T,k] f32, indices [T,k] int64)``.
        """
        if x.dtype != torch.bfloat16 or x.dim() != 2 or x.size(1) != self.dim:
            raise WfUnsupported("x must be bf16 [T, dim]")
        x = x.contiguous()
        T = x.size(0)
        if self.hash_layer:
            if input_ids is None:
                raise WfUnsupported("hash layers need input_ids")
            input_ids = input_ids.reshape(-1).to(torch.int64).contiguous()
        if partial and T > self.max_tokens:
            raise WfUnsupported("partial mode needs T <= max_tokens (the shared output is per call)")
        if partial:
            y = out if out is not None else torch.empty(T, self.dim, dtype=torch.float32, device=x.device)
        else:
            y = out if out is not None else torch.empty(T, self.dim, dtype=torch.bfloat16, device=x.device)
        rw = ri = None
        if routing:
            rw = torch.empty(T, self.topk, dtype=torch.float32, device=x.device)
            ri = torch.empty(T, self.topk, dtype=torch.int64, device=x.device)
        st = L.stream_ptr()
        for t0 in range(0, T, self.max_tokens):
            t1 = min(T, t0 + self.max_tokens)
            n = t1 - t0
            xs = x[t0:t1]
            ids = input_ids[t0:t1] if input_ids is not None else None
            ys = y[t0:t1]
            rc = self.lib.wf_moe_forward(
                ctypes.byref(self.cfg), ctypes.byref(self.wstruct), L.ptr(xs), L.ptr(ids), n,
                0 if partial else L.ptr(ys), L.ptr(ys) if partial else 0,
                L.ptr(rw[t0:t1]) if routing else 0, L.ptr(ri[t0:t1]) if routing else 0,
                L.ptr(self.workspace), self.workspace.numel(), st)
            L.check(rc, "wf_moe_forward")
        return (y, rw, ri) if routing else y

    __call__ = forward

    def finish(self, y_partial, row0=0, out=None):
        """Expert-parallel epilogue: ``bf16(y_partial + shared(x)[row0:row0+T])`` (architecture.py:791-794)."""
        T = y_partial.size(0)
        y = out if out is not None else torch.empty(T, self.dim, dtype=torch.bfloat16, device=y_partial.device)
        L.check(self.lib.wf_moe_finish(ctypes.byref(self.cfg), L.ptr(y_partial.contiguous()), T, row0,
                                       L.ptr(y), L.ptr(self.workspace), self.workspace.numel(),
                                       L.stream_ptr()), "wf_moe_finish")
        return y

    # ------------------------------------------------------------------------
    # expert-parallel split by token ownership (wanferenz_b200.ep)
    # ------------------------------------------------------------------------
    def forward_ep(self, x, weights, indices, shared_rows=(0, 0), out=None):
        """Local experts on a gathered batch ``x [T, D]`` with its given routing
        (``weights [T, k]``, global ``indices [T, k]``), plus the shared expert on
        rows ``[r0, r0 + n)`` = ``shared_rows``: the fp32 partial ``[T, D]`` to be
        summed over ranks (``wf_moe_forward_ep``)."""
        x = x.contiguous()
        T = x.size(0)
        if T > self.max_tokens:
            raise WfUnsupported("forward_ep: T exceeds max_tokens")
        weights = weights.to(torch.float32).contiguous()
        indices = indices.to(torch.int64).contiguous()
        yp = out if out is not None else torch.empty(T, self.dim, dtype=torch.float32, device=x.device)
        r0, n = shared_rows
        L.check(self.lib.wf_moe_forward_ep(ctypes.byref(self.cfg), ctypes.byref(self.wstruct), L.ptr(x), T,
                                           L.ptr(weights), L.ptr(indices), int(r0), int(n), L.ptr(yp),
                                           L.ptr(self.workspace), self.workspace.numel(), L.stream_ptr()),
                "wf_moe_forward_ep")
        return yp

    def to_bf16(self, y, out=None):
        """``bf16(y)`` of an fp32 ``y`` (``wf_moe_to_bf16``)."""
        y = y.contiguous()
        o = out if out is not None else torch.empty(y.shape, dtype=torch.bfloat16, device=y.device)
        L.check(self.lib.wf_moe_to_bf16(L.ptr(y), y.numel(), L.ptr(o), L.stream_ptr()), "wf_moe_to_bf16")
        return o

    def sum_ranks(self, parts, out=None):
        """``bf16(parts[0] + ... + parts[P-1])`` of fp32 ``parts [P, T, D]``, summed in
        ascending rank order (``wf_moe_sum_ranks``)."""
        parts = parts.contiguous()
        P = parts.size(0)
        o = out if out is not None else torch.empty(parts.shape[1:], dtype=torch.bfloat16, device=parts.device)
        L.check(self.lib.wf_moe_sum_ranks(L.ptr(parts), P, parts[0].numel(), L.ptr(o), L.stream_ptr()),
                "wf_moe_sum_ranks")
        return o

    def route(self, x, input_ids=None):
        """``Gate.forward`` (architecture.py:696-718): ``(weights [T,k] f32, indices [T,k] int64)``."""
        x = x.contiguous()
        T = x.size(0)
        if T > self.max_tokens:
            raise WfUnsupported("route: T exceeds max_tokens")
        if input_ids is not None:
            input_ids = input_ids.reshape(-1).to(torch.int64).contiguous()
        rw = torch.empty(T, self.topk, dtype=torch.float32, device=x.device)
        ri = torch.empty(T, self.topk, dtype=torch.int64, device=x.device)
        L.check(self.lib.wf_moe_route(ctypes.byref(self.cfg), ctypes.byref(self.wstruct), L.ptr(x),
                                      L.ptr(input_ids), T, L.ptr(rw), L.ptr(ri), L.ptr(self.workspace),
                                      self.workspace.numel(), L.stream_ptr()), "wf_moe_route")
        return rw, ri

    def read_error(self):
        """Raises if a call since the last read set the device error word (synchronizes; clears the word)."""
        L.check(self.lib.wf_moe_read_error(L.ptr(self.workspace), self.workspace.numel(),
                                           L.stream_ptr()), "wf_moe_read_error")


# ----------------------------------------------------------------------------
# weight helpers
# ----------------------------------------------------------------------------
def dequant_fp4(q, s):
    """Packed E2M1 ``[.., K/2]`` + e8m0 ``[.., K/32]`` -> f32 ``[.., K]`` (torch glue, not a hot path)."""
    table = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0,
                          -4.0, -6.0], device=q.device)
    u = q.view(torch.uint8)
    v = torch.stack([table[(u & 15).long()], table[(u >> 4).long()]], -1).flatten(-2)
    return v * s.float().repeat_interleave(32, -1)


def stack_bank(experts, dim, inter_dim):
    """Stacks FP4 ``Expert`` modules into the bank layout (fp4_grouped.py:142-188)."""
    w13 = torch.stack([torch.cat([_u8(e.w1.weight), _u8(e.w3.weight)]) for e in experts])
    w13_s = torch.stack([torch.cat([_u8(e.w1.scale), _u8(e.w3.scale)]) for e in experts])
    w2 = torch.stack([_u8(e.w2.weight) for e in experts])
    w2_s = torch.stack([_u8(e.w2.scale) for e in experts])
    return w13, w13_s, w2, w2_s


def _rebind_to_bank(experts, w13, w13_s, w2, w2_s, I):
    """Expert parameters become views into the bank (``_relayout_moe(preserve=False)``,
    fp4_grouped.py:168-186): one copy of the weights, in the bank's layout."""
    with torch.no_grad():
        for j, e in enumerate(experts):
            e.w1.weight.data = w13[j, :I].view(torch.float4_e2m1fn_x2)
            e.w3.weight.data = w13[j, I:].view(torch.float4_e2m1fn_x2)
            e.w1.scale.data = w13_s[j, :I].view(torch.float8_e8m0fnu)
            e.w3.scale.data = w13_s[j, I:].view(torch.float8_e8m0fnu)
            e.w2.weight.data = w2[j].view(torch.float4_e2m1fn_x2)
            e.w2.scale.data = w2_s[j].view(torch.float8_e8m0fnu)
            e.w1.weight.scale = e.w1.scale
            e.w3.weight.scale = e.w3.scale
            e.w2.weight.scale = e.w2.scale


def _check_supported(moe):
    """Raises ``WfUnsupported`` unless the routed experts are FP4 and the shared expert FP8."""
    lo, hi = moe.experts_start_idx, moe.experts_end_idx
    experts = [moe.experts[i] for i in range(lo, hi)]
    if not experts or experts[0].w1.weight.dtype != torch.float4_e2m1fn_x2:
        raise WfUnsupported("routed experts are not FP4")
    if moe.shared_experts.w1.weight.dtype != torch.float8_e4m3fn:
        raise WfUnsupported("shared expert is not FP8")


def bank_from_module(moe, mod, preserve=True):
    """Host half of the load-time bank: ``(MoEWeights, MoELayer keyword arguments)`` of a
    reference ``MoE`` module (architecture.py:744-775), on the experts' own device.

    The routed experts are stacked into the ``[E_local, 2I, D/2]`` bank (fp4_grouped.py:
    142-188) and the shared expert's w1/w3 into ``[2I, D]`` (fp8_vector.py:316-351).  With
    ``preserve=False`` the experts' parameters are rebound as views into the bank, so
    the weights exist once.  Raises ``WfUnsupported`` for layers the kernels do not
    cover (routed experts not FP4, shared expert not FP8)."""
    _check_supported(moe)
    lo, hi = moe.experts_start_idx, moe.experts_end_idx
    experts = [moe.experts[i] for i in range(lo, hi)]
    e0 = experts[0]
    sh = moe.shared_experts
    D, I = moe.dim, e0.w1.weight.size(0)
    w13, w13_s, w2, w2_s = stack_bank(experts, D, I)
    if not preserve:
        _rebind_to_bank(experts, w13, w13_s, w2, w2_s, I)
    sw13 = torch.cat([_u8(sh.w1.weight), _u8(sh.w3.weight)])
    ss13 = torch.cat([_scale(sh.w1.scale), _scale(sh.w3.scale)])
    g = moe.gate
    weights = MoEWeights(
        gate_w=g.weight.detach().to(torch.bfloat16), gate_b=None if g.bias is None else g.bias.detach(),
        tid2eid=getattr(g, "tid2eid", None) if g.hash else None,
        w13=w13, w13_s=w13_s, w2=w2, w2_s=w2_s, shared_w13=sw13, shared_s13=ss13,
        shared_w2=_u8(sh.w2.weight), shared_s2=_scale(sh.w2.scale))
    kwargs = dict(dim=D, inter_dim=I, n_experts=moe.n_routed_experts, topk=g.topk,
                  score_func=g.score_func, route_scale=float(g.route_scale),
                  swiglu_limit=float(e0.swiglu_limit), hash_layer=bool(g.hash),
                  vocab=g.tid2eid.size(0) if g.hash else 0,
                  ue8m0=getattr(mod, "scale_fmt", "ue8m0") is not None,
                  n_local_experts=hi - lo, expert_offset=lo)
    return weights, kwargs


def _to_device(w: MoEWeights, device):
    return MoEWeights(**{f.name: (None if getattr(w, f.name) is None else getattr(w, f.name).to(device))
                         for f in dataclasses.fields(w)})


def _grouped_bank_of(layer):
    """The layer's device bank under the reference's bank keys (fp4_grouped.py:136, 186):
    what ``graphs/decoder.py``'s capture gate looks for as ``moe._grouped_bank``."""
    w = layer.weights
    return {"w13": w.w13, "w13_s": w.w13_s, "w2": w.w2, "w2_s": w.w2_s}


def _layer_from_module(moe, mod, preserve=True, max_tokens=64):
    """Builds a ``MoELayer`` from a reference ``MoE`` module: ``bank_from_module``, then
    the upload to the current CUDA device (a no-op for a module already there)."""
    weights, kwargs = bank_from_module(moe, mod, preserve=preserve)
    dev = torch.device("cuda", torch.cuda.current_device())
    if weights.w13.device != dev:
        weights = _to_device(weights, dev)
        if not preserve:
            _rebind_to_bank([moe.experts[i] for i in range(moe.experts_start_idx, moe.experts_end_idx)],
                            weights.w13, weights.w13_s, weights.w2, weights.w2_s, kwargs["inter_dim"])
    return MoELayer(weights, max_tokens=max_tokens, **kwargs)


def bank_layout(module, preserve=True, max_tokens=64):
    """Stacks every MoE in ``module`` into a load-time bank and attaches its ``MoELayer``.

    Mirrors ``fp4_grouped.bank_layout`` (fp4_grouped.py:191-201): returns the number of
    MoE modules laid out, and leaves each one's bank in ``moe._grouped_bank`` (the
    attribute the reference's CUDA-graph capture gate checks, graphs/decoder.py:258-264).
    A layer the kernels do not cover is skipped, as the reference skips non-FP4 layers.
    """
    n = 0
    for m in module.modules():
        if hasattr(m, "experts") and hasattr(m, "experts_start_idx") and getattr(m, "_wf_layer", None) is None:
            try:
                m._wf_layer = _layer_from_module(m, _MOD, preserve=preserve, max_tokens=max_tokens)
            except WfUnsupported:
                continue
            m._grouped_bank = _grouped_bank_of(m._wf_layer)
            n += 1
    return n


# free device memory a lazily stacked bank must leave (fp4_grouped.py:204, _BANK_HEADROOM_BYTES)
BANK_HEADROOM_BYTES = 2 << 30


def _bank_fits(moe, max_tokens=64):
    """Whether stacking this layer's bank beside its per-expert weights leaves the
    headroom free (fp4_grouped.py:207-218): the lazy path copies the weights."""
    lo, hi = moe.experts_start_idx, moe.experts_end_idx
    need = sum(t.numel() * t.element_size()
               for e in (moe.experts[i] for i in range(lo, hi))
               for k in ("w1", "w2", "w3") for t in (getattr(e, k).weight, getattr(e, k).scale))
    sh = moe.shared_experts
    need += sum(t.numel() * t.element_size() for k in ("w1", "w3") for t in (getattr(sh, k).weight,
                                                                            getattr(sh, k).scale))
    free, _total = torch.cuda.mem_get_info()
    return free - need >= BANK_HEADROOM_BYTES


def _decline(self, x, input_ids, why):
    """The reference plugins' convention for a configuration they do not cover
    (fp4_grouped.py:256-262): count the reason and run the replaced forward."""
    counts = getattr(self, "_grouped_declined", None)
    if counts is None:
        counts = self._grouped_declined = {}
    counts[why] = counts.get(why, 0) + 1
    return _REF_FORWARD(self, x, input_ids)


BANK_DECLINED = "bank does not fit beside the per-expert weights"


def b200_forward(self, x, input_ids):
    """Replacement of ``MoE.forward`` (architecture.py:777-794) on the B200 kernels.

    A configuration the kernels do not cover (``WfUnsupported``: experts not
    FP4, shared expert not FP8, shapes outside the kernels' limits, a batch over
    the workspace in the all-reduce mode) declines to the replaced forward and
    is counted in ``self._grouped_declined``, the reference's tally
    (fp4_grouped.py:256-262); so does a layer without a load-time bank whose
    lazily stacked bank would not fit in free device memory (fp4_grouped.py:
    221-232).  A missing CUDA device or library and CUDA errors raise.
    Successful steps count in ``self._grouped_steps``, the counter the
    reference's graph-capture probe reads (graphs/decoder.py:223-246).
    """
    layer = getattr(self, "_wf_layer", None)
    if layer is False:
        return _decline(self, x, input_ids, self._wf_unsupported)
    if layer is None:
        try:
            _check_supported(self)
            if not _bank_fits(self):
                raise WfUnsupported(BANK_DECLINED)
            self._wf_layer = layer = _layer_from_module(self, _MOD)
        except WfUnsupported as e:
            self._wf_layer, self._wf_unsupported = False, str(e)
            return _decline(self, x, input_ids, str(e))
    try:
        y = _b200_step(self, layer, x, input_ids)
    except WfUnsupported as e:
        return _decline(self, x, input_ids, str(e))
    self._grouped_steps = getattr(self, "_grouped_steps", 0) + 1
    return y


def _b200_step(self, layer, x, input_ids):
    shape = x.size()
    xv = x.view(-1, self.dim)
    ids = input_ids.flatten() if input_ids is not None else None
    world = int(getattr(_MOD, "world_size", 1) or 1)
    if world > 1:
        import torch.distributed as dist

        yp = layer.forward(xv, ids, partial=True)
        dist.all_reduce(yp)
        y = layer.finish(yp)
    else:
        y = layer.forward(xv, ids)
    return y.view(shape)


# Markers: ours, and the reference's grouped-MoE marker (fp4_grouped.py:347), which
# its lever audit (serving/controls.py:38-68) and CUDA-graph capture gate
# (graphs/decoder.py:213-220) read: this forward is a grouped MoE forward with a
# load-time bank and no host sync, the contract that gate stands for.
b200_forward._wf_b200 = True
b200_forward._v4_grouped = True


def install(mod):
    """Replaces ``mod.MoE.forward`` with ``b200_forward`` (fp4_grouped.install, 339-351).

    Raises if the CUDA library cannot be loaded or no CUDA device is present:
    there is no fallback path.  Returns False if already installed.
    """
    global _REF_FORWARD, _MOD
    if getattr(mod.MoE.forward, "_wf_b200", False):
        return False
    if not torch.cuda.is_available():
        raise RuntimeError("wanferenz_b200.install: no CUDA device")
    L.load()
    _REF_FORWARD = mod.MoE.forward
    _MOD = mod
    mod.MoE.forward = b200_forward
    return True


def b200_draft_forward(self, x, input_ids):
    """The drafter MoE's forward on the B200 kernels (decoding/expert_bank.py:108-164).

    The reference's drafter path computes each (token, expert) pair on its own and
    sums a token's experts in ascending id in fp32, then adds the shared expert:
    ``MoE.forward``'s arithmetic, checked bit-exact by its own self-test
    (expert_bank.py:261-344), for any number of draft tokens.  So this is the
    layer forward itself, on the drafter layer's load-time bank, with the
    drafter's tallies (``_draft_steps``, ``_draft_declined``); a configuration
    the kernels do not cover runs the class forward, as the reference's decline
    does (expert_bank.py:96-105)."""
    try:
        y = _b200_step(self, self._wf_layer, x, input_ids)
    except WfUnsupported as e:
        tally = getattr(self, "_draft_declined", None)
        if tally is None:
            tally = self._draft_declined = {}
        tally[str(e)] = tally.get(str(e), 0) + 1
        return type(self).forward(self, x, input_ids)
    self._draft_steps = getattr(self, "_draft_steps", 0) + 1
    return y


b200_draft_forward._wf_b200 = True


def install_drafter(dstail, mod=None, max_tokens=64):
    """Routes the DSpark drafter's MoE layers through the B200 kernels
    (``expert_bank.install_drafter``, decoding/expert_bank.py:167-196).

    For every block of ``dstail.mtp`` whose ``ffn`` is an FP4 MoE with an FP8
    shared expert, builds its load-time bank (the experts' parameters become
    views into it, ``preserve=False``) and patches that instance's ``forward``.
    Unlike the reference's drafter path, hash-routed layers are covered too.
    Returns the number of layers patched."""
    import types

    global _MOD
    if mod is not None:
        _MOD = mod
    took = 0
    for blk in getattr(dstail, "mtp", ()):
        moe = getattr(blk, "ffn", None)
        if moe is None or not hasattr(moe, "experts_start_idx"):
            continue
        try:
            _check_supported(moe)
        except WfUnsupported:
            continue
        if getattr(moe, "_wf_layer", None) in (None, False):
            moe._wf_layer = _layer_from_module(moe, _MOD, preserve=False, max_tokens=max_tokens)
            moe._grouped_bank = _grouped_bank_of(moe._wf_layer)
        moe.forward = types.MethodType(b200_draft_forward, moe)
        took += 1
    return took


def uninstall(mod):
    global _REF_FORWARD
    if _REF_FORWARD is None:
        return False
    mod.MoE.forward = _REF_FORWARD
    _REF_FORWARD = None
    return True


def coverage(module):
    """Per MoE layer: ``(steps on the B200 path, declined reasons)`` (fp4_grouped.coverage, 327-336)."""
    return {getattr(m, "layer_id", i): (getattr(m, "_grouped_steps", 0), dict(getattr(m, "_grouped_declined", {})))
            for i, m in enumerate(mm for mm in module.modules() if hasattr(mm, "experts_start_idx"))}
