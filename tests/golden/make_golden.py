"""Generate the golden vectors in this folder from the REFERENCE's own CPU path.

Usage::

    python tests/golden/make_golden.py --reference <path to the WANferenz checkout>

The reference is imported as the package ``wanferenz`` with its torch CPU
operator backend (``V4_KERNELS=cpu``: wanferenz/kernels/torch_ops.py:197-240)
and its model file loaded the way its own grouped-MoE smoke does
(``_load_model_module``, wanferenz/kernels/fp4_grouped.py:432-455): world size
1, FP8 default dtype for the shared expert, ``scale_fmt="ue8m0"`` and e8m0
activation scales.  No expert-dispatch plugin is installed, so ``MoE.forward``
is the plain reference loop (architecture.py:777-794).

Every weight is regenerated from ``oracle.fixtures`` (seeded bf16 sources), then
quantized by the REFERENCE's quantizers (``torch_ops.fp4_act_quant``,
``fp4_grouped._fp8_block_quant``).  The golden files store, per case:

* the layer spec and the token batch's seed;
* sha256 digests of the reference-quantized weight bytes (so the oracle's
  quantizer restatement can be pinned bit-exactly without storing weights);
* the reference's outputs: layer output ``y`` (bf16 bits), router weights,
  router indices and router logits (fp32).

Operator-level cases (``act_quant``, ``fp4_act_quant``, ``fp8_gemm``,
``fp4_gemm``) store their outputs the same way.
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import fixtures as F  # noqa: E402
from oracle import moe_oracle as O  # noqa: E402

# Layer cases: name -> (spec, T values).  Small "mini" shapes cover each
# routing / activation option; cfg1 and cfg2 are BASELINE configs 1 and 2;
# cfg2_batch is config 2 at the benchmark's 16 tokens and cfg4 is BASELINE
# config 4 (64 tokens, Zipf(1.2) expert popularity: experts with more than 16
# tokens, i.e. several token groups of one expert).
LAYER_CASES = {
    "mini_sigmoid": (F.LayerSpec(D=256, I=128, E=16, topk=4, score_func="sigmoid",
                                 route_scale=1.5, seed=11), (1, 5)),
    "mini_sqrtsoftplus_clamp": (F.LayerSpec(D=256, I=256, E=16, topk=4, score_func="sqrtsoftplus",
                                            route_scale=2.5, swiglu_limit=10.0, w_std=0.5,
                                            seed=12), (3,)),
    "mini_softmax": (F.LayerSpec(D=384, I=128, E=8, topk=2, score_func="softmax",
                                 route_scale=1.0, seed=13), (4,)),
    "mini_hash_dups": (F.LayerSpec(D=256, I=128, E=16, topk=6, score_func="sqrtsoftplus",
                                   route_scale=1.5, swiglu_limit=10.0, hash_layer=True,
                                   hash_pattern=(3, 3, 7, 3, 12, 7), seed=14), (2,)),
    "mini_hash_random": (F.LayerSpec(D=256, I=128, E=16, topk=6, score_func="sqrtsoftplus",
                                     route_scale=1.5, hash_layer=True, seed=15), (6,)),
    "mini_fp32scale": (F.LayerSpec(D=256, I=128, E=16, topk=4, score_func="sigmoid",
                                   route_scale=1.5, ue8m0=False, seed=16), (3,)),
    "cfg1": (F.CONFIG1, (1, 8)),
    "cfg2": (F.CONFIG2, (1, 4)),
    "cfg2_batch": (F.CONFIG2, (16,)),
    "cfg4": (F.CONFIG4, (64,)),
}


def _load_reference(path):
    os.environ["V4_KERNELS"] = "cpu"
    os.environ["V4_MOE_DECODE"] = "0"
    os.environ["V4_MOE_GROUPED"] = "0"
    os.environ["PYTHONDONTWRITEBYTECODE"] = "1"
    sys.dont_write_bytecode = True
    sys.path.insert(0, path)
    import torch
    import wanferenz.kernels.fp4_grouped as fp4_grouped

    mod = fp4_grouped._load_model_module()
    return torch, mod, fp4_grouped


def _bf16_tensor(torch, u16):
    return torch.from_numpy(np.ascontiguousarray(u16).view(np.int16)).view(torch.bfloat16)


def _u8(t):
    import torch
    return t.contiguous().view(torch.uint8).numpy().copy()


def make_layer_case(torch, mod, fp4_grouped, name, spec, T_values, out):
    from wanferenz.kernels.reference import fp4_act_quant

    mod.scale_fmt = "ue8m0" if spec.ue8m0 else None
    mod.scale_dtype = torch.float8_e8m0fnu if spec.ue8m0 else torch.float32
    layer = F.SyntheticLayer(spec)
    args = mod.ModelArgs(dim=spec.D, moe_inter_dim=spec.I, n_routed_experts=spec.E,
                         n_activated_experts=spec.topk, n_shared_experts=1,
                         n_hash_layers=1 if spec.hash_layer else 0, score_func=spec.score_func,
                         route_scale=spec.route_scale, swiglu_limit=spec.swiglu_limit,
                         expert_dtype="fp4", vocab_size=spec.vocab)
    with mod.set_dtype(torch.bfloat16):
        moe = mod.MoE(0, args)
    with torch.no_grad():
        moe.gate.weight.data.copy_(_bf16_tensor(torch, layer.gate_w_bf16))
        if spec.hash_layer:
            moe.gate.tid2eid.data.copy_(torch.from_numpy(layer.tid2eid))
        else:
            moe.gate.bias.data.copy_(torch.from_numpy(layer.gate_b))
        sh_hash = []
        for lin, src in zip((moe.shared_experts.w1, moe.shared_experts.w3, moe.shared_experts.w2),
                            layer.shared_bf16()):
            w, s = fp4_grouped._fp8_block_quant(_bf16_tensor(torch, src), 128)
            lin.weight.data.copy_(w)
            lin.scale.data.copy_(s)
            sh_hash += [_u8(w), _u8(s)]
    filled = {}
    for T in T_values:
        x16, ids = layer.activations(T)
        x = _bf16_tensor(torch, x16).view(1, T, spec.D)
        tid = torch.from_numpy(ids).view(1, T)
        with torch.no_grad():
            weights, indices = moe.gate(x.view(-1, spec.D), tid.flatten())
            logits = torch.nn.functional.linear(x.view(-1, spec.D).float(), moe.gate.weight.float())
            for e in sorted(set(indices.flatten().tolist())):
                if e in filled:
                    continue
                ex = moe.experts[e]
                digest = []
                for lin, src in zip((ex.w1, ex.w3, ex.w2), layer.expert_bf16(e)):
                    w, s = fp4_act_quant(_bf16_tensor(torch, src), 32)
                    lin.weight.data.copy_(w)
                    lin.scale.data.copy_(s)
                    digest += [_u8(w), _u8(s)]
                filled[e] = F.sha256(*digest)
            y = moe(x, tid)
        key = f"{name}_T{T}"
        out[key] = dict(
            spec=json.dumps(spec.as_dict()), T=np.int64(T),
            y=y.view(-1, spec.D).view(torch.int16).numpy().view(np.uint16).copy(),
            weights=weights.float().numpy().copy(),
            indices=indices.long().numpy().copy(),
            logits=logits.numpy().copy(),
            expert_ids=np.array(sorted(filled), np.int64),
            expert_sha=np.array([filled[e] for e in sorted(filled)]),
            shared_sha=np.array(F.sha256(*sh_hash)),
        )
        print(f"{key}: experts touched so far {len(filled)}", flush=True)


def make_op_cases(torch, out):
    from wanferenz.kernels import reference as R
    import wanferenz.kernels.fp4_grouped as fp4_grouped

    x16 = F.normal_bf16((101, 0), (8, 512), 1.0)
    x = _bf16_tensor(torch, x16)
    for fmt, sd, tag in (("ue8m0", torch.float8_e8m0fnu, "ue8m0"), (None, torch.float32, "fp32")):
        q, s = R.act_quant(x, 128, fmt, sd)
        out[f"op_act_quant_{tag}"] = dict(q=_u8(q), s=(_u8(s) if sd != torch.float32 else s.numpy().copy()))
    w16 = F.normal_bf16((102, 0), (64, 256), 0.02)
    wq, ws = R.fp4_act_quant(_bf16_tensor(torch, w16), 32)
    out["op_fp4_act_quant"] = dict(q=_u8(wq), s=_u8(ws))
    # fp8_gemm: e8m0 weight scales (model path) and fp32 weight scales
    a16 = F.normal_bf16((103, 0), (4, 512), 1.0)
    a = _bf16_tensor(torch, a16)
    b16 = F.normal_bf16((104, 0), (256, 512), 0.02)
    bq, bs = fp4_grouped._fp8_block_quant(_bf16_tensor(torch, b16), 128)
    aq, as_ = R.act_quant(a, 128, "ue8m0", torch.float8_e8m0fnu)
    c = R.fp8_gemm(aq, as_, bq, bs, torch.float8_e8m0fnu)
    out["op_fp8_gemm_e8m0"] = dict(c=c.view(torch.int16).numpy().view(np.uint16).copy(),
                                   bq_sha=np.array(F.sha256(_u8(bq), _u8(bs))))
    bs32 = (bs.float() * 1.25).contiguous()
    aq32, as32 = R.act_quant(a, 128, None, torch.float32)
    c32 = R.fp8_gemm(aq32, as32, bq, bs32, torch.float32)
    out["op_fp8_gemm_fp32"] = dict(c=c32.view(torch.int16).numpy().view(np.uint16).copy())
    w2_16 = F.normal_bf16((105, 0), (256, 512), 0.02)
    w2q, w2s = R.fp4_act_quant(_bf16_tensor(torch, w2_16), 32)
    c4 = R.fp4_gemm(aq, as_, w2q, w2s, torch.float8_e8m0fnu)
    out["op_fp4_gemm"] = dict(c=c4.view(torch.int16).numpy().view(np.uint16).copy())


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--reference", required=True, help="path of the WANferenz checkout")
    ap.add_argument("--only", default="", help="comma-separated case names")
    a = ap.parse_args()
    torch, mod, fp4_grouped = _load_reference(a.reference)
    torch.set_num_threads(os.cpu_count())
    only = set(filter(None, a.only.split(",")))
    ops = {}
    if not only or "ops" in only:
        make_op_cases(torch, ops)
        np.savez_compressed(os.path.join(HERE, "ops.npz"),
                            **{f"{k}/{f}": v for k, d in ops.items() for f, v in d.items()})
    for name, (spec, Ts) in LAYER_CASES.items():
        if only and name not in only:
            continue
        out = {}
        make_layer_case(torch, mod, fp4_grouped, name, spec, Ts, out)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"),
                            **{f"{k}/{f}": v for k, d in out.items() for f, v in d.items()})


if __name__ == "__main__":
    main()
