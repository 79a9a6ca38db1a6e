"""The torch CPU restatement that the bench times as the reference's CPU path
(``oracle/torch_port.py``) against the reference's own outputs (tests/golden)
and the numpy oracle.

Its router indices must match the reference's (rows whose k/k+1 biased-score
gap is within fp32 summation noise excepted) and its layer outputs must meet
the layer tolerance; it uses the same torch ops as the reference, so on most
cases they are bit-identical.
"""

import numpy as np
import pytest

from oracle import fixtures as F
from oracle import moe_oracle as O
from oracle import torch_port as P
from tests import golden_util as G


def _cases(names):
    for name in names:
        for key in G.load(name):
            yield pytest.param(name, key, id=key)


@pytest.mark.parametrize("name,key", list(_cases(G.LAYER_FILES[:6])) + [pytest.param("cfg1", "cfg1_T1", id="cfg1_T1")])
def test_torch_port_matches_reference(name, key):
    case = G.load(name)[key]
    spec = G.spec_of(case)
    layer = F.SyntheticLayer(spec)
    T = int(case["T"])
    x16, ids = layer.activations(T)
    x = O.bf16_to_f32(x16)
    y = P.moe_forward(x, layer.params(), ids).numpy()
    w, idx = P.gate(P._t(x), layer.params(), ids)
    _, _, biased = O.gate(x, layer.gate_w, layer.gate_b, spec.topk, spec.score_func,
                          spec.route_scale, layer.tid2eid, ids)
    tie = (O.topk_margin(biased, spec.topk) < 1e-6) if not spec.hash_layer else np.zeros(T, bool)
    np.testing.assert_array_equal(idx.numpy()[~tie], case["indices"][~tie])
    np.testing.assert_allclose(w.numpy()[~tie], case["weights"][~tie], rtol=1e-5, atol=1e-7)
    y_ref = O.bf16_to_f32(case["y"])[~tie]
    d = np.abs(y[~tie] - y_ref)
    assert d.mean() <= 2e-3
    assert (d / np.maximum(np.abs(y_ref), 0.01 * np.sqrt((y_ref ** 2).mean()))).max() <= 1e-2


def test_torch_port_quantizers_match_oracle():
    x = O.bf16_to_f32(F.normal_bf16((101, 0), (8, 512), 1.0))
    for ue8m0 in (True, False):
        q, s = P.act_quant(P._t(x), 128, ue8m0)
        qo, so = O.act_quant(x, 128, ue8m0)
        assert np.array_equal(q.numpy(), qo) and np.array_equal(s.numpy(), so)
    w = O.bf16_to_f32(F.normal_bf16((102, 0), (64, 256), 0.02))
    wq, ws = O.fp4_act_quant(w)
    assert np.array_equal(P.dequant_fp4(wq, ws).numpy(), O.dequant_fp4(wq, ws))
    b = O.bf16_to_f32(F.normal_bf16((104, 0), (256, 512), 0.02))
    bq, bs = O.fp8_block_quant(b)
    assert np.array_equal(P.dequant_fp8(bq, bs).numpy(), O.dequant_fp8(bq, bs))
