"""The CPU oracle against the reference's own outputs (tests/golden, made by make_golden.py).

Pins the oracle before it is trusted as the checker of the CUDA path:
* its quantizers reproduce the reference-quantized weight bytes (sha256);
* its layer output, router weights and indices match the reference's.
"""

import numpy as np
import pytest

from oracle import fixtures as F
from oracle import moe_oracle as O
from tests import golden_util as G

MINI = G.LAYER_FILES[:6]


def _cases(names):
    for name in names:
        for key, case in G.load(name).items():
            yield pytest.param(name, key, id=key)


def _check_case(name, key, touched_only=True):
    case = G.load(name)[key]
    spec = G.spec_of(case)
    layer = F.SyntheticLayer(spec)
    T = int(case["T"])
    x16, ids = layer.activations(T)
    x = O.bf16_to_f32(x16)
    idx_ref = case["indices"]
    used = set(int(e) for e in np.unique(idx_ref))
    for e, sha in zip(case["expert_ids"], case["expert_sha"]):
        if touched_only and int(e) not in used:
            continue
        assert F.sha256(*layer.expert(int(e))) == str(sha), f"expert {e} quantization differs"
    assert F.sha256(*layer.shared()) == str(case["shared_sha"]), "shared expert quantization differs"
    y, w, idx = O.moe_forward(x, layer.params(), ids)
    y_ref = O.bf16_to_f32(case["y"])
    # indices: bit-exact except where the k/k+1 gap is within fp32 summation noise
    _, _, biased = O.gate(x, layer.gate_w, layer.gate_b, spec.topk, spec.score_func,
                          spec.route_scale, layer.tid2eid, ids)
    margin = O.topk_margin(biased, spec.topk) if not spec.hash_layer else np.full(T, np.inf)
    tie = margin < 1e-6
    np.testing.assert_array_equal(idx[~tie], idx_ref[~tie])
    np.testing.assert_allclose(w[~tie], case["weights"][~tie], rtol=1e-6, atol=1e-7)
    # the oracle restates the reference step by step: outputs are bit-identical here
    assert np.array_equal(y[~tie], y_ref[~tie])


@pytest.mark.parametrize("name,key", list(_cases(MINI)))
def test_oracle_matches_reference_mini(name, key):
    _check_case(name, key)


def test_oracle_matches_reference_cfg1_t1():
    _check_case("cfg1", "cfg1_T1")


@pytest.mark.slow
@pytest.mark.parametrize("name,key", [("cfg1", "cfg1_T8"), ("cfg2", "cfg2_T1"), ("cfg2", "cfg2_T4")])
def test_oracle_matches_reference_full_size(name, key):
    _check_case(name, key)


def test_oracle_operator_goldens():
    ops = G.load("ops")
    x = O.bf16_to_f32(F.normal_bf16((101, 0), (8, 512), 1.0))
    q, s = O.act_quant(x, 128, ue8m0=True)
    assert np.array_equal(O.e4m3_encode(q), ops["op_act_quant_ue8m0"]["q"])
    assert np.array_equal(O.e8m0_encode(s), ops["op_act_quant_ue8m0"]["s"])
    q, s = O.act_quant(x, 128, ue8m0=False)
    assert np.array_equal(O.e4m3_encode(q), ops["op_act_quant_fp32"]["q"])
    assert np.array_equal(s, ops["op_act_quant_fp32"]["s"])
    w = O.bf16_to_f32(F.normal_bf16((102, 0), (64, 256), 0.02))
    wq, ws = O.fp4_act_quant(w)
    assert np.array_equal(wq, ops["op_fp4_act_quant"]["q"])
    assert np.array_equal(ws, ops["op_fp4_act_quant"]["s"])
    a = O.bf16_to_f32(F.normal_bf16((103, 0), (4, 512), 1.0))
    b = O.bf16_to_f32(F.normal_bf16((104, 0), (256, 512), 0.02))
    bq, bs = O.fp8_block_quant(b)
    assert F.sha256(bq, bs) == str(ops["op_fp8_gemm_e8m0"]["bq_sha"])
    aq, as_ = O.act_quant(a, 128, True)
    c = O.fp8_gemm(aq, as_, bq, bs)
    assert np.array_equal(O.f32_to_bf16(c), ops["op_fp8_gemm_e8m0"]["c"])
    bs32 = (O.e8m0_decode(bs) * np.float32(1.25)).astype(np.float32)
    aq32, as32 = O.act_quant(a, 128, False)
    c32 = O.fp8_gemm(aq32, as32, bq, bs32)
    ref = O.bf16_to_f32(ops["op_fp8_gemm_fp32"]["c"])
    np.testing.assert_allclose(c32, ref, rtol=8e-3, atol=1e-6)
    w2 = O.bf16_to_f32(F.normal_bf16((105, 0), (256, 512), 0.02))
    w2q, w2s = O.fp4_act_quant(w2)
    c4 = O.fp4_gemm(aq, as_, w2q, w2s)
    assert np.array_equal(O.f32_to_bf16(c4), ops["op_fp4_gemm"]["c"])


@pytest.mark.parametrize("name,key", [("cfg2_batch", "cfg2_batch_T16"), ("cfg4", "cfg4_T64")])
def test_oracle_router_matches_reference_full_batch(name, key):
    """The full-batch golden cases (the benchmark's 16 tokens; config 4's 64 tokens
    with Zipf popularity): the oracle's router (gate bias recipe included) gives the
    reference's logits, indices and weights.  Their layer outputs are checked on the
    GPU against the reference's, on weights pinned to the reference's bytes."""
    case = G.load(name)[key]
    spec = G.spec_of(case)
    layer = F.SyntheticLayer(spec)
    x16, ids = layer.activations(int(case["T"]))
    x = O.bf16_to_f32(x16)
    logits, _ = O.gate_scores(x, layer.gate_w, spec.score_func)
    np.testing.assert_allclose(logits, case["logits"], rtol=0, atol=2e-6)
    w, idx, biased = O.gate(x, layer.gate_w, layer.gate_b, spec.topk, spec.score_func, spec.route_scale)
    tie = O.topk_margin(biased, spec.topk) < 1e-6
    assert tie.sum() <= max(1, len(tie) // 64)
    np.testing.assert_array_equal(idx[~tie], case["indices"][~tie])
    np.testing.assert_allclose(w[~tie], case["weights"][~tie], rtol=1e-6, atol=1e-7)


def test_config4_golden_has_multi_group_experts():
    """The config-4 golden case exercises experts with more than 16 tokens (several
    16-token groups of one expert, i.e. B-operand reloads at K = 4096 / 2048) and
    many experts with none."""
    case = G.load("cfg4")["cfg4_T64"]
    counts = np.bincount(case["indices"].ravel(), minlength=256)
    assert (counts > 16).sum() >= 2 and counts.max() > 32
    assert (counts == 0).sum() > 128


def test_planted_mistake_is_caught():
    """A deliberately wrong oracle (bias dropped) must disagree with the golden indices."""
    case = G.load("mini_sigmoid")["mini_sigmoid_T5"]
    spec = G.spec_of(case)
    layer = F.SyntheticLayer(spec)
    x16, ids = layer.activations(int(case["T"]))
    w, idx, _ = O.gate(O.bf16_to_f32(x16), layer.gate_w, None, spec.topk, spec.score_func,
                       spec.route_scale)
    assert not np.array_equal(idx, case["indices"]) or not np.allclose(w, case["weights"])
