"""The C-ABI library loads on any host and exports what include/wfb200.h declares.

No compute calls here: these run without a GPU.
"""

import ctypes
import os
import re

import pytest

from wanferenz_b200 import _lib as L

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    src = open(os.path.join(ROOT, "include", "wfb200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(wf_[a-z0-9_]+)\s*\(", src)))


def test_header_matches_binding_list():
    assert _declared() == sorted(L.EXPORTS)


def test_library_exports_every_declared_symbol():
    lib = L.load()
    for name in _declared():
        assert hasattr(lib, name), name


def _cfg(**kw):
    base = dict(dim=4096, inter_dim=2048, n_experts=256, n_local_experts=256, expert_offset=0,
                topk=6, score_func=1, hash_layer=0, ue8m0=1, max_tokens=64, vocab=0,
                route_scale=1.5, swiglu_limit=0.0)
    base.update(kw)
    return L.MoeConfig(**base)


def test_workspace_size_and_config_validation():
    lib = L.load()
    ok = lib.wf_moe_workspace_bytes(ctypes.byref(_cfg()))
    assert ok > 0
    # workspace holds h (T*k*I bf16) and o (T*k*D bf16) at least
    assert ok >= 64 * 6 * (2048 + 4096) * 2
    bad = [dict(dim=4000), dict(inter_dim=0), dict(n_experts=1024), dict(topk=9),
           dict(expert_offset=200, n_local_experts=100), dict(max_tokens=0), dict(score_func=7),
           dict(dim=8192), dict(hash_layer=1, vocab=0)]
    for kw in bad:
        assert lib.wf_moe_workspace_bytes(ctypes.byref(_cfg(**kw))) == 0, kw
        assert lib.wf_last_error().decode(), kw


def test_null_arguments_fail_with_status():
    lib = L.load()
    rc = lib.wf_moe_forward(ctypes.byref(_cfg()), None, None, None, 1, None, None, None, None,
                            None, 0, None)
    assert rc == L.WF_E_ARG
    assert lib.wf_act_quant(None, 1, 128, 128, 1, None, None, 1, None) == L.WF_E_ARG
    assert lib.wf_fp8_gemm(None, None, 0, None, None, 0, 1, 16, 128, None, None, 0, None) == L.WF_E_ARG


def test_shape_errors_before_any_launch():
    lib = L.load()
    p = ctypes.c_void_p(16)  # never dereferenced: shape checks come first
    assert lib.wf_act_quant(p, 2, 100, 128, 1, p, p, 1, None) == L.WF_E_SHAPE
    assert lib.wf_fp4_act_quant(p, 2, 48, p, p, None) == L.WF_E_SHAPE
    assert lib.wf_fp8_gemm(p, p, 0, p, p, 0, 1, 16, 100, p, p, 256, None) == L.WF_E_SHAPE
    assert lib.wf_fp8_gemm(p, p, 5, p, p, 0, 1, 16, 128, p, p, 256, None) == L.WF_E_DTYPE


def test_expert_parallel_entry_points_validate_before_launch():
    lib = L.load()
    p = ctypes.c_void_p(16)  # never dereferenced: every check below precedes any launch
    w = L.MoeWeights()
    for f in ("w13", "w13_s", "w2", "w2_s", "shared_w13", "shared_s13", "shared_w2", "shared_s2", "gate_w"):
        setattr(w, f, 16)
    cfg = ctypes.byref(_cfg())
    # routing and output are required
    assert lib.wf_moe_forward_ep(cfg, ctypes.byref(w), p, 4, None, p, 0, 4, p, p, 1 << 40, None) == L.WF_E_ARG
    # the shared-expert window must lie inside the batch
    for r0, n in ((-1, 1), (0, 5), (3, 2), (0, -1)):
        assert lib.wf_moe_forward_ep(cfg, ctypes.byref(w), p, 4, p, p, r0, n, p, p, 1 << 40, None) == L.WF_E_SHAPE
    assert lib.wf_moe_to_bf16(None, 8, p, None) == L.WF_E_ARG
    assert lib.wf_moe_to_bf16(p, 0, p, None) == L.WF_E_SHAPE
    assert lib.wf_moe_sum_ranks(p, 0, 8, p, None) == L.WF_E_SHAPE       # no ranks
    assert lib.wf_moe_sum_ranks(p, 2, 6, p, None) == L.WF_E_SHAPE       # n not a multiple of 4
    assert lib.wf_moe_sum_ranks(ctypes.c_void_p(24), 2, 8, p, None) == L.WF_E_ARG  # parts misaligned
