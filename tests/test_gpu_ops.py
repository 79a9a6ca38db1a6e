"""Parity of the CUDA operators (reference operator API) with the reference / oracle."""

import numpy as np
import pytest
import torch

from oracle import fixtures as F
from oracle import moe_oracle as O
from tests import golden_util as G
from tests import gpu_util as U

pytestmark = pytest.mark.gpu


def _ops():
    from wanferenz_b200 import ops
    return ops


@pytest.fixture(params=["tcgen05", "mma_sync"])
def engine(request, monkeypatch):
    """Dense GEMMs run on the tcgen05 kernel when shapes allow; WF_DISABLE_TC selects the other one."""
    monkeypatch.setenv("WF_DISABLE_TC", "1" if request.param == "mma_sync" else "0")
    return request.param


def test_act_quant_bit_exact():
    ops = _ops()
    g = G.load("ops")
    x = U.bf16_tensor(F.normal_bf16((101, 0), (8, 512), 1.0))
    q, s = ops.act_quant(x, 128, "ue8m0", torch.float8_e8m0fnu)
    assert np.array_equal(q.view(torch.uint8).cpu().numpy(), g["op_act_quant_ue8m0"]["q"])
    assert np.array_equal(s.view(torch.uint8).cpu().numpy(), g["op_act_quant_ue8m0"]["s"])
    q, s = ops.act_quant(x, 128, None, torch.float32)
    assert np.array_equal(q.view(torch.uint8).cpu().numpy(), g["op_act_quant_fp32"]["q"])
    assert np.array_equal(s.cpu().numpy(), g["op_act_quant_fp32"]["s"])


@pytest.mark.parametrize("shape,std", [((64, 256), 0.02), ((300, 4096), 1.0), ((17, 2048), 1e-3)])
def test_fp4_act_quant_bit_exact(shape, std):
    ops = _ops()
    w16 = F.normal_bf16((102, shape[0]), shape, std)
    q, s = ops.fp4_act_quant(U.bf16_tensor(w16))
    q_ref, s_ref = O.fp4_act_quant(O.bf16_to_f32(w16))
    assert np.array_equal(q.view(torch.uint8).cpu().numpy(), q_ref)
    assert np.array_equal(s.view(torch.uint8).cpu().numpy(), s_ref)


def test_fp8_gemm_golden(engine):
    ops = _ops()
    g = G.load("ops")
    a = U.bf16_tensor(F.normal_bf16((103, 0), (4, 512), 1.0))
    b = O.bf16_to_f32(F.normal_bf16((104, 0), (256, 512), 0.02))
    bq, bs = O.fp8_block_quant(b)
    bq_t = U.u8_tensor(bq).view(torch.float8_e4m3fn)
    bs_t = U.u8_tensor(bs).view(torch.float8_e8m0fnu)
    aq, as_ = ops.act_quant(a, 128, "ue8m0", torch.float8_e8m0fnu)
    c = ops.fp8_gemm(aq, as_, bq_t, bs_t, torch.float8_e8m0fnu)
    U.assert_layer_close(U.to_f32(c), O.bf16_to_f32(g["op_fp8_gemm_e8m0"]["c"]), "fp8 e8m0")
    bs32 = torch.from_numpy((O.e8m0_decode(bs) * np.float32(1.25)).astype(np.float32)).cuda()
    aq32, as32 = ops.act_quant(a, 128, None, torch.float32)
    c32 = ops.fp8_gemm(aq32, as32, bq_t, bs32, torch.float32)
    U.assert_layer_close(U.to_f32(c32), O.bf16_to_f32(g["op_fp8_gemm_fp32"]["c"]), "fp8 f32")


def test_fp4_gemm_golden(engine):
    ops = _ops()
    g = G.load("ops")
    a = U.bf16_tensor(F.normal_bf16((103, 0), (4, 512), 1.0))
    w = O.bf16_to_f32(F.normal_bf16((105, 0), (256, 512), 0.02))
    wq, ws = O.fp4_act_quant(w)
    aq, as_ = ops.act_quant(a, 128, "ue8m0", torch.float8_e8m0fnu)
    c = ops.fp4_gemm(aq, as_, U.u8_tensor(wq).view(torch.float4_e2m1fn_x2),
                     U.u8_tensor(ws).view(torch.float8_e8m0fnu), torch.float8_e8m0fnu)
    U.assert_layer_close(U.to_f32(c), O.bf16_to_f32(g["op_fp4_gemm"]["c"]), "fp4")


@pytest.mark.parametrize("M,N,K", [(1, 4096, 4096), (2, 12288, 4096), (16, 4096, 4096), (5, 1024, 4096),
                                   (3, 512, 2048), (9, 2048, 1024), (4, 4096, 16384), (16, 1024, 8192),
                                   (8, 129280, 4096), (1, 32768, 1024),
                                   # the attention's dense projections (fp8_vector.py:505-513)
                                   (1, 512, 4096), (16, 32768, 1024), (4, 4096, 8192), (1, 8192, 1024)])
@pytest.mark.parametrize("scale", ["e8m0", "f32"])
def test_fp8_gemm_vs_oracle(M, N, K, scale, engine):
    """BASELINE config 3 shapes and the attention projections of fp8_vector.py:505-513
    (fp32 or e8m0 weight scales per 128x128)."""
    ops = _ops()
    a16 = F.normal_bf16((201, M, N, K), (M, K), 1.0)
    rng = F.rng(202, N, K)
    bq = O.e4m3_encode(O.e4m3_round(np.clip(rng.standard_normal((N, K), dtype=np.float32) * 40, -448, 448)))
    if scale == "e8m0":
        bs = rng.integers(118, 125, size=(N // 128, K // 128)).astype(np.uint8)
        bs_t = U.u8_tensor(bs).view(torch.float8_e8m0fnu)
    else:
        bs = (rng.random((N // 128, K // 128), dtype=np.float32) * 1e-3 + 1e-4).astype(np.float32)
        bs_t = torch.from_numpy(bs).cuda()
    ue = scale == "e8m0"
    aq, as_ = ops.act_quant(U.bf16_tensor(a16), 128, "ue8m0" if ue else None,
                            torch.float8_e8m0fnu if ue else torch.float32)
    c = ops.fp8_gemm(aq, as_, U.u8_tensor(bq).view(torch.float8_e4m3fn), bs_t)
    aq_o, as_o = O.act_quant(O.bf16_to_f32(a16), 128, ue)
    c_ref = O.fp8_gemm(aq_o, as_o, bq, bs)
    U.assert_layer_close(U.to_f32(c), c_ref, f"fp8 {M}x{N}x{K}")


@pytest.mark.parametrize("M,N,K", [(1, 4096, 4096), (3, 4096, 8192), (12, 2048, 2048)])
def test_fp4_gemm_vs_oracle(M, N, K, engine):
    """fp4_gemm (torch_ops.py:102-108), including split-K (K > 4096)."""
    ops = _ops()
    a16 = F.normal_bf16((211, M, N, K), (M, K), 1.0)
    rng = F.rng(212, N, K)
    wq = rng.integers(0, 256, size=(N, K // 2)).astype(np.uint8)
    ws = rng.integers(116, 126, size=(N, K // 32)).astype(np.uint8)
    aq, as_ = ops.act_quant(U.bf16_tensor(a16), 128, "ue8m0", torch.float8_e8m0fnu)
    c = ops.fp4_gemm(aq, as_, U.u8_tensor(wq).view(torch.float4_e2m1fn_x2),
                     U.u8_tensor(ws).view(torch.float8_e8m0fnu))
    aq_o, as_o = O.act_quant(O.bf16_to_f32(a16), 128, True)
    U.assert_layer_close(U.to_f32(c), O.fp4_gemm(aq_o, as_o, wq, ws), f"fp4 {M}x{N}x{K}")


def test_grouped_fp4_gemm_vs_oracle():
    """grouped_fp4_gemm (fp4_grouped.py:96-128): slot g uses weights g."""
    ops = _ops()
    G_, N, K = 6, 4096, 4096
    a16 = F.normal_bf16((301,), (G_, K), 1.0)
    aq, as_ = ops.act_quant(U.bf16_tensor(a16), 128, "ue8m0", torch.float8_e8m0fnu)
    aq_o, as_o = O.act_quant(O.bf16_to_f32(a16), 128, True)
    ws, ss, refs = [], [], []
    for gi in range(G_):
        w = O.bf16_to_f32(F.normal_bf16((302, gi), (N, K), 0.02))
        wq, wsc = O.fp4_act_quant(w)
        ws.append(wq); ss.append(wsc)
        refs.append(O.fp4_gemm(aq_o[gi:gi + 1], as_o[gi:gi + 1], wq, wsc))
    c = ops.grouped_fp4_gemm(aq, as_, U.u8_tensor(np.stack(ws)).view(torch.float4_e2m1fn_x2),
                             U.u8_tensor(np.stack(ss)).view(torch.float8_e8m0fnu))
    U.assert_layer_close(U.to_f32(c), np.concatenate(refs), "grouped")
