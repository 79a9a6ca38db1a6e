"""Checkpoint -> expert bank, without building per-expert modules.

The reference serves a converted checkpoint (``model*-mp*.safetensors`` plus
``config.json``, written by wanferenz/model/conversion.py:55-116) by building
every ``Block``, ``load_state_dict``-ing each layer (wanferenz/serving/
partition.py:759-801) and then restacking each MoE's experts into a bank
(``fp4_grouped.bank_layout``, fp4_grouped.py:142-201).  This module reads the
same files straight into the bank layout the kernels consume:

* ``layers.{L}.ffn.experts.{e}.w1|w3|w2.weight`` (float4_e2m1fn_x2, packed E2M1)
  and ``.scale`` (float8_e8m0fnu, one per 32) -> ``w13 [E_local, 2I, D/2]``
  (w1 rows, then w3 rows), ``w13_s``, ``w2 [E_local, D, I/2]``, ``w2_s``;
* ``layers.{L}.ffn.shared_experts.w1|w3|w2.weight`` (float8_e4m3fn) and
  ``.scale`` (128 x 128 blocks) -> the stacked shared expert;
* ``layers.{L}.ffn.gate.weight`` (bf16), ``.bias`` (f32; score-routed layers)
  or ``.tid2eid`` (int32; the first ``n_hash_layers`` layers).

Each expert goes from the file to its slice of the bank on the target device
(one ~13 MB copy at a time), so loading a layer holds one copy of its weights.
The layer shape and routing options come from ``config.json`` (the
``ModelArgs`` field names the converted checkpoint carries, architecture.py:
42-93, or the Hugging Face names of the source release).
"""

from __future__ import annotations

import glob
import json
import os

import torch

from .moe import MoELayer, MoEWeights, WfUnsupported

# ModelArgs field -> the Hugging Face name of the same setting
_HF_NAMES = {
    "dim": "hidden_size", "moe_inter_dim": "moe_intermediate_size", "n_routed_experts": "n_routed_experts",
    "n_activated_experts": "num_experts_per_tok", "n_hash_layers": "num_hash_layers",
    "score_func": "scoring_func", "route_scale": "routed_scaling_factor", "swiglu_limit": "swiglu_limit",
    "vocab_size": "vocab_size",
}


def model_args(d):
    """The MoE-relevant ``ModelArgs`` fields of the checkpoint directory ``d``."""
    with open(os.path.join(d, "config.json")) as f:
        cfg = json.load(f)
    out = {}
    for key, hf in _HF_NAMES.items():
        if key in cfg:
            out[key] = cfg[key]
        elif hf in cfg:
            out[key] = cfg[hf]
    out.setdefault("n_hash_layers", 0)
    out.setdefault("swiglu_limit", 0.0)
    out.setdefault("route_scale", 1.0)
    qc = cfg.get("quantization_config") or {}
    out["scale_fmt"] = cfg.get("scale_fmt", qc.get("scale_fmt", "ue8m0"))
    missing = [k for k in ("dim", "moe_inter_dim", "n_routed_experts", "n_activated_experts", "score_func")
               if k not in out]
    if missing:
        raise ValueError(f"{d}/config.json lacks {missing}")
    return out


class TensorIndex:
    """Which ``model*-mp*.safetensors`` file holds each tensor name (the lookup of
    partition.tensor_locations, partition.py:69-85), with the files opened once."""

    def __init__(self, d):
        from safetensors import safe_open

        files = sorted(glob.glob(os.path.join(d, "model*-mp*.safetensors")))
        if not files:
            raise FileNotFoundError(f"no model*-mp*.safetensors in {d!r} (a converted checkpoint)")
        self._open = {}
        self.where = {}
        for f in files:
            h = safe_open(f, framework="pt", device="cpu")
            self._open[f] = h
            for n in h.keys():
                self.where[n] = f

    def __contains__(self, name):
        return name in self.where

    def get(self, name):
        if name not in self.where:
            raise KeyError(f"tensor {name!r} not in the checkpoint")
        return self._open[self.where[name]].get_tensor(name)


def _u8(t):
    return t.contiguous().view(torch.uint8)


def read_layer(d, layer_id, rank=0, world=1, device="cpu", index=None):
    """``(MoEWeights, MoELayer keyword arguments)`` of MoE layer ``layer_id`` of the
    checkpoint in ``d``, for expert shard ``rank`` of ``world`` (architecture.py:749-756),
    with every tensor on ``device``."""
    args = model_args(d)
    idx = index or TensorIndex(d)
    D, I, E = args["dim"], args["moe_inter_dim"], args["n_routed_experts"]
    if E % world:
        raise ValueError(f"{E} experts do not divide over {world} ranks")
    El = E // world
    lo = rank * El
    pre = f"layers.{layer_id}.ffn."
    dev = torch.device(device)
    if idx.get(f"{pre}experts.{lo}.w1.weight").dtype != torch.float4_e2m1fn_x2:
        raise WfUnsupported("routed experts are not FP4")
    w13 = torch.empty(El, 2 * I, D // 2, dtype=torch.uint8, device=dev)
    w13_s = torch.empty(El, 2 * I, D // 32, dtype=torch.uint8, device=dev)
    w2 = torch.empty(El, D, I // 2, dtype=torch.uint8, device=dev)
    w2_s = torch.empty(El, D, I // 32, dtype=torch.uint8, device=dev)
    for j in range(El):
        ep = f"{pre}experts.{lo + j}."
        w13[j, :I].copy_(_u8(idx.get(ep + "w1.weight")))
        w13[j, I:].copy_(_u8(idx.get(ep + "w3.weight")))
        w13_s[j, :I].copy_(_u8(idx.get(ep + "w1.scale")))
        w13_s[j, I:].copy_(_u8(idx.get(ep + "w3.scale")))
        w2[j].copy_(_u8(idx.get(ep + "w2.weight")))
        w2_s[j].copy_(_u8(idx.get(ep + "w2.scale")))
    sp = f"{pre}shared_experts."
    if idx.get(sp + "w1.weight").dtype != torch.float8_e4m3fn:
        raise WfUnsupported("shared expert is not FP8")

    def scale(name):
        s = idx.get(name)
        return (s.float() if s.dtype == torch.float32 else _u8(s)).contiguous()

    shared_w13 = torch.cat([_u8(idx.get(sp + "w1.weight")), _u8(idx.get(sp + "w3.weight"))]).to(dev)
    shared_s13 = torch.cat([scale(sp + "w1.scale"), scale(sp + "w3.scale")]).to(dev)
    hash_layer = layer_id < int(args["n_hash_layers"])
    gate_w = idx.get(pre + "gate.weight").to(torch.bfloat16).to(dev)
    gate_b = None if hash_layer else idx.get(pre + "gate.bias").float().to(dev)
    tid2eid = idx.get(pre + "gate.tid2eid").to(torch.int32).to(dev) if hash_layer else None
    weights = MoEWeights(gate_w=gate_w, gate_b=gate_b, tid2eid=tid2eid, w13=w13, w13_s=w13_s, w2=w2, w2_s=w2_s,
                         shared_w13=shared_w13, shared_s13=shared_s13,
                         shared_w2=_u8(idx.get(sp + "w2.weight")).to(dev), shared_s2=scale(sp + "w2.scale").to(dev))
    kwargs = dict(dim=D, inter_dim=I, n_experts=E, topk=int(args["n_activated_experts"]),
                  score_func=args["score_func"], route_scale=float(args["route_scale"]),
                  swiglu_limit=float(args["swiglu_limit"]), hash_layer=hash_layer,
                  vocab=int(tid2eid.size(0)) if hash_layer else 0, ue8m0=args["scale_fmt"] is not None,
                  n_local_experts=El, expert_offset=lo)
    return weights, kwargs


def load_layer(d, layer_id, rank=0, world=1, max_tokens=64, device=None, index=None):
    """A ready ``MoELayer`` for MoE layer ``layer_id`` of the converted checkpoint ``d``,
    its bank read straight onto ``device`` (the current CUDA device by default)."""
    dev = device or torch.device("cuda", torch.cuda.current_device())
    weights, kwargs = read_layer(d, layer_id, rank=rank, world=world, device=dev, index=index)
    return MoELayer(weights, max_tokens=max_tokens, **kwargs)


def load_layers(d, layer_ids, rank=0, world=1, max_tokens=64, device=None):
    """``{layer_id: MoELayer}`` for a stage's layers, the files opened once."""
    index = TensorIndex(d)
    return {li: load_layer(d, li, rank, world, max_tokens, device, index) for li in layer_ids}
