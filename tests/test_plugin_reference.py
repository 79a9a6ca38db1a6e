"""The layer plugin against the reference's own ``MoE`` module, on the host (no GPU).

The reference model file is loaded the way its grouped-MoE smoke loads it
(``fp4_grouped._load_model_module``, wanferenz/kernels/fp4_grouped.py:432-455,
torch CPU operators), in a spawned child process so its global settings (default
dtype, ``sys.modules['wanferenz']``) stay out of this one.  The child builds real
``MoE`` layers (architecture.py:744-775) with FP4 routed experts and an FP8
shared expert quantized by the reference's own quantizers, and runs the host
half of the plugin on them:

* ``bank_from_module(preserve=False)``: bank shapes and bytes, the experts'
  parameters rebound as views into the bank (the reference's forward still gives
  the same output through them), and the configuration fields read from the
  module (top-k, score function, route scale, SwiGLU limit, hash routing and its
  vocabulary, the expert shard of rank 1 of 2);
* ``checkpoint.read_layer``: a converted checkpoint holding the module (its
  state_dict under ``layers.{L}.ffn.``, ``config.json`` from ``ModelArgs``) reads
  into the same bank bytes and configuration as the module relayout;
* the reference's CUDA-graph capture gate (graphs/decoder.py:249-272) and lever
  audit (serving/controls.py:38-68) on a module with the plugin installed: the
  chain starts with the grouped marker, the bank is found, and the probe step
  counts one ``_grouped_steps`` with no decline.  The device step is replaced by
  the reference forward here, since no GPU is present.

The reference checkout is found through ``WANFERENZ_REFERENCE`` or as the
``reference`` directory beside this repository; the test skips without it.
"""

import os

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _reference_dir():
    for cand in (os.environ.get("WANFERENZ_REFERENCE"), os.path.join(os.path.dirname(ROOT), "reference")):
        if cand and os.path.isfile(os.path.join(cand, "wanferenz", "model", "architecture.py")):
            return cand
    return None


REF = _reference_dir()
pytestmark = pytest.mark.skipif(REF is None, reason="reference checkout not found")


def _build_moe(mod, torch, spec, layer_id):
    """A reference MoE whose weights are the fixture's, quantized by the reference."""
    import wanferenz.kernels.fp4_grouped as fp4_grouped
    from wanferenz.kernels.reference import fp4_act_quant

    from oracle import fixtures as F

    def bf16(u16):
        return torch.from_numpy(np.ascontiguousarray(u16).view(np.int16)).view(torch.bfloat16)

    layer = F.SyntheticLayer(spec)
    args = mod.ModelArgs(dim=spec.D, moe_inter_dim=spec.I, n_routed_experts=spec.E,
                         n_activated_experts=spec.topk, n_shared_experts=1,
                         n_hash_layers=1 if spec.hash_layer else 0, score_func=spec.score_func,
                         route_scale=spec.route_scale, swiglu_limit=spec.swiglu_limit,
                         expert_dtype="fp4", vocab_size=spec.vocab)
    with mod.set_dtype(torch.bfloat16):
        moe = mod.MoE(layer_id, args)
    with torch.no_grad():
        moe.gate.weight.data.copy_(bf16(layer.gate_w_bf16))
        if spec.hash_layer:
            moe.gate.tid2eid.data.copy_(torch.from_numpy(layer.tid2eid))
        else:
            moe.gate.bias.data.copy_(torch.from_numpy(layer.gate_b))
        for lin, src in zip((moe.shared_experts.w1, moe.shared_experts.w3, moe.shared_experts.w2),
                            layer.shared_bf16()):
            w, s = fp4_grouped._fp8_block_quant(bf16(src), 128)
            lin.weight.data.copy_(w)
            lin.scale.data.copy_(s)
        for e in range(moe.experts_start_idx, moe.experts_end_idx):
            for lin, src in zip((moe.experts[e].w1, moe.experts[e].w3, moe.experts[e].w2), layer.expert_bf16(e)):
                w, s = fp4_act_quant(bf16(src), 32)
                lin.weight.data.copy_(w)
                lin.scale.data.copy_(s)
    return moe, layer


def _child(ref_dir, q):
    """Runs in a spawned process: every check, results (or the failure) to ``q``."""
    import sys
    import traceback

    try:
        os.environ.update(V4_KERNELS="cpu", V4_MOE_DECODE="0", V4_MOE_GROUPED="0", PYTHONDONTWRITEBYTECODE="1")
        sys.dont_write_bytecode = True
        sys.path.insert(0, ref_dir)
        sys.path.insert(0, ROOT)
        import torch
        import wanferenz.kernels.fp4_grouped as fp4_grouped

        import wanferenz_b200.moe as b200
        from oracle import fixtures as F

        mod = fp4_grouped._load_model_module()
        out = {}
        specs = {
            "sigmoid": (F.LayerSpec(D=256, I=128, E=16, topk=4, score_func="sigmoid", route_scale=1.5,
                                    seed=81), 5, 1, 0),
            "hash": (F.LayerSpec(D=256, I=128, E=16, topk=6, score_func="sqrtsoftplus", route_scale=2.5,
                                 swiglu_limit=10.0, hash_layer=True, vocab=64, seed=82), 5, 0, 0),
            "rank1of2": (F.LayerSpec(D=256, I=128, E=16, topk=4, score_func="softmax", route_scale=1.0,
                                     seed=83), 3, 1, 1),
        }
        import dataclasses
        import json
        import tempfile

        import safetensors.torch as ST

        from wanferenz_b200 import checkpoint

        for name, (spec, T, layer_id, rank) in specs.items():
            mod.world_size, mod.rank = (2, rank) if name == "rank1of2" else (1, 0)
            moe, layer = _build_moe(mod, torch, spec, layer_id)
            lo, hi = moe.experts_start_idx, moe.experts_end_idx
            # a converted checkpoint holding this layer, under the names a stage's
            # load reads (layers.{L}.ffn.*; partition.py:759-801, chain.py:2105-2117)
            ckpt = tempfile.mkdtemp(prefix="wf_ckpt_")
            state = {f"layers.{layer_id}.ffn.{k}": v.detach().clone().contiguous()
                     for k, v in moe.state_dict().items()}
            ST.save_file(state, os.path.join(ckpt, "model00000-mp1.safetensors"))
            margs = mod.ModelArgs(dim=spec.D, moe_inter_dim=spec.I, n_routed_experts=spec.E,
                                  n_activated_experts=spec.topk, n_shared_experts=1,
                                  n_hash_layers=1 if spec.hash_layer else 0, score_func=spec.score_func,
                                  route_scale=spec.route_scale, swiglu_limit=spec.swiglu_limit,
                                  expert_dtype="fp4", vocab_size=spec.vocab)
            with open(os.path.join(ckpt, "config.json"), "w") as fh:
                json.dump(dataclasses.asdict(margs), fh)
            cw, ckw = checkpoint.read_layer(ckpt, layer_id, rank=mod.rank, world=mod.world_size, device="cpu")
            before = {e: [getattr(moe.experts[e], k).weight.view(torch.uint8).clone() for k in ("w1", "w3", "w2")]
                      for e in range(lo, hi)}
            x16, ids = layer.activations(T)
            x = torch.from_numpy(x16.view(np.int16)).view(torch.bfloat16).view(1, T, spec.D)
            tid = torch.from_numpy(ids).view(1, T)
            if mod.world_size == 1:
                with torch.no_grad():
                    y0 = mod.MoE.forward(moe, x, tid).clone()
            w, kw = b200.bank_from_module(moe, mod, preserve=False)
            r = {"kw": kw, "shapes": {f: tuple(getattr(w, f).shape) for f in
                                      ("w13", "w13_s", "w2", "w2_s", "shared_w13", "shared_s13",
                                       "shared_w2", "shared_s2", "gate_w")},
                 "tid2eid": None if w.tid2eid is None else tuple(w.tid2eid.shape),
                 "gate_b": w.gate_b is not None}
            views = True
            same = True
            for j, e in enumerate(range(lo, hi)):
                ex = moe.experts[e]
                I = spec.I
                views &= ex.w1.weight.data_ptr() == w.w13[j].data_ptr()
                views &= ex.w3.weight.data_ptr() == w.w13[j, I:].data_ptr()
                views &= ex.w2.weight.data_ptr() == w.w2[j].data_ptr()
                views &= ex.w1.scale.data_ptr() == w.w13_s[j].data_ptr()
                views &= ex.w2.scale.data_ptr() == w.w2_s[j].data_ptr()
                same &= bool(torch.equal(w.w13[j, :I], before[e][0]) and torch.equal(w.w13[j, I:], before[e][1])
                             and torch.equal(w.w2[j], before[e][2]))
            r["views"], r["bytes_kept"] = bool(views), bool(same)
            fields = ("gate_w", "gate_b", "tid2eid", "w13", "w13_s", "w2", "w2_s", "shared_w13", "shared_s13",
                      "shared_w2", "shared_s2")
            r["checkpoint_bank_equal"] = all(
                (getattr(cw, f) is None and getattr(w, f) is None) or
                (getattr(cw, f) is not None and getattr(w, f) is not None and
                 torch.equal(getattr(cw, f).view(torch.uint8) if getattr(cw, f).dtype != torch.float32 else getattr(cw, f),
                             getattr(w, f).view(torch.uint8) if getattr(w, f).dtype != torch.float32 else getattr(w, f)))
                for f in fields)
            r["checkpoint_kwargs_equal"] = ckw == kw
            if mod.world_size == 1:
                with torch.no_grad():
                    y1 = mod.MoE.forward(moe, x, tid)
                r["forward_unchanged"] = bool(torch.equal(y0, y1))
            out[name] = r
        # the reference's graph-capture gate on a module with the plugin installed
        mod.world_size, mod.rank = 1, 0
        import wanferenz.graphs.decoder as decoder
        import wanferenz.serving.controls as controls

        spec, T, layer_id, _ = specs["sigmoid"]
        moe, layer = _build_moe(mod, torch, spec, layer_id)
        ref_forward = mod.MoE.forward
        torch.cuda.is_available = lambda: True  # install() checks for a device; no kernel runs here
        assert b200.install(mod)
        out["chain"] = controls.moe_chain(mod)
        out["grouped_at_one_token"] = decoder.grouped_at_one_token(mod)
        w, _ = b200.bank_from_module(moe, mod, preserve=False)
        moe._grouped_bank = {"w13": w.w13, "w13_s": w.w13_s, "w2": w.w2, "w2_s": w.w2_s}
        moe._wf_layer = object()  # a built layer; its device step is replaced below
        b200._b200_step = lambda self, layer, x, ids: ref_forward(self, x, ids.view(x.shape[:-1]))
        L = type("Block", (), {})()
        L.ffn = moe
        ids = torch.zeros(1, 1, dtype=torch.int64)
        out["refusal"] = decoder._moe_refusal(L, torch.device("cpu"), torch.bfloat16, ids, mod)
        out["steps_after_probe"] = getattr(moe, "_grouped_steps", 0)
        moe._grouped_bank = None
        out["refusal_without_bank"] = decoder._moe_refusal(L, torch.device("cpu"), torch.bfloat16, ids, mod)
        b200.uninstall(mod)
        # the drafter's MoE layers (decoding/expert_bank.py:167-196): instance-level
        # forward on a load-time bank, the drafter's own tallies
        import types as _types

        spec, T, layer_id, _ = specs["sigmoid"]
        dmoe, dlayer = _build_moe(mod, torch, spec, layer_id)
        dstail = _types.SimpleNamespace(mtp=[_types.SimpleNamespace(ffn=dmoe), _types.SimpleNamespace(ffn=None)])

        def host_layer(moe, m, preserve=True, max_tokens=64):
            w, _ = b200.bank_from_module(moe, m, preserve=preserve)
            return _types.SimpleNamespace(weights=w)

        b200._layer_from_module = host_layer  # the device upload needs a GPU
        out["drafter_took"] = b200.install_drafter(dstail, mod=mod)
        x16, ids = dlayer.activations(3)
        xd = torch.from_numpy(x16.view(np.int16)).view(torch.bfloat16).view(1, 3, spec.D)
        with torch.no_grad():
            y_draft = dmoe.forward(xd, torch.from_numpy(ids).view(1, 3))
            y_ref = mod.MoE.forward(dmoe, xd, torch.from_numpy(ids).view(1, 3))
        out["drafter_patched"] = isinstance(dmoe.forward, _types.MethodType) and getattr(
            dmoe.forward.__func__, "_wf_b200", False)
        out["drafter_steps"] = getattr(dmoe, "_draft_steps", 0)
        out["drafter_same"] = bool(torch.equal(y_draft, y_ref))
        out["drafter_bank"] = sorted((dmoe._grouped_bank or {}).keys())
        q.put(("ok", out))
    except Exception:
        q.put(("error", traceback.format_exc()))


@pytest.fixture(scope="module")
def results():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_child, args=(REF, q))
    p.start()
    status, out = q.get(timeout=600)
    p.join(timeout=60)
    assert status == "ok", out
    return out


def test_bank_from_reference_module(results):
    for name in ("sigmoid", "hash", "rank1of2"):
        r = results[name]
        El = 8 if name == "rank1of2" else 16
        assert r["shapes"]["w13"] == (El, 256, 128)
        assert r["shapes"]["w13_s"] == (El, 256, 8)
        assert r["shapes"]["w2"] == (El, 256, 64)
        assert r["shapes"]["w2_s"] == (El, 256, 4)
        assert r["shapes"]["shared_w13"] == (256, 256)
        assert r["shapes"]["shared_s13"] == (2, 2) and r["shapes"]["shared_s2"] == (2, 1)
        assert r["shapes"]["gate_w"] == (16, 256)
        assert r["views"], f"{name}: expert parameters are not views into the bank"
        assert r["bytes_kept"], f"{name}: the bank does not hold the experts' bytes"
        if name != "rank1of2":
            assert r["forward_unchanged"], f"{name}: the reference forward changed after the relayout"


def test_checkpoint_loader_matches_module_bank(results):
    """wanferenz_b200.checkpoint reads a converted checkpoint of the reference's module
    (its state_dict under layers.{L}.ffn., config.json from ModelArgs) straight into
    the same bank bytes and configuration as the module relayout."""
    for name in ("sigmoid", "hash", "rank1of2"):
        assert results[name]["checkpoint_bank_equal"], name
        assert results[name]["checkpoint_kwargs_equal"], name


def test_drafter_layers_patched(results):
    """install_drafter patches each drafter MoE instance (a block without an ffn is
    skipped), gives it a load-time bank under the reference's keys and counts its
    steps in the drafter's tally; the device step is replaced by the reference
    forward here, so the output equals the reference's."""
    assert results["drafter_took"] == 1
    assert results["drafter_patched"]
    assert results["drafter_steps"] == 1
    assert results["drafter_same"]
    assert results["drafter_bank"] == ["w13", "w13_s", "w2", "w2_s"]


def test_config_fields_read_from_reference_module(results):
    kw = results["sigmoid"]["kw"]
    assert (kw["topk"], kw["score_func"], kw["route_scale"], kw["swiglu_limit"]) == (4, "sigmoid", 1.5, 0.0)
    assert (kw["hash_layer"], kw["vocab"], kw["ue8m0"]) == (False, 0, True)
    assert (kw["n_local_experts"], kw["expert_offset"], kw["n_experts"]) == (16, 0, 16)
    assert results["sigmoid"]["gate_b"] and results["sigmoid"]["tid2eid"] is None
    kw = results["hash"]["kw"]
    assert (kw["topk"], kw["score_func"], kw["route_scale"], kw["swiglu_limit"]) == (6, "sqrtsoftplus", 2.5, 10.0)
    assert (kw["hash_layer"], kw["vocab"]) == (True, 64)
    assert results["hash"]["tid2eid"] == (64, 6) and not results["hash"]["gate_b"]
    kw = results["rank1of2"]["kw"]
    assert (kw["n_local_experts"], kw["expert_offset"], kw["score_func"]) == (8, 8, "softmax")


def test_reference_graph_gate_admits_the_plugin(results):
    assert results["chain"][0] == "grouped", results["chain"]
    assert results["grouped_at_one_token"]
    assert results["refusal"] is None, results["refusal"]
    assert results["steps_after_probe"] == 0  # the probe restores the counter it read
    assert "no load-time expert bank" in (results["refusal_without_bank"] or "")
