"""The allocation-free forward (wf_moe_forward_noalloc), through the C ABI.

Some callers cannot hand the layer a workspace: their device memory belongs to
another allocator that has nothing to give out at call time, or they may not
call the CUDA allocator while serving (cudaMalloc can synchronize the whole
device).  For them the layer runs on the library's own module-scope scratch.
These tests check, on two consecutive calls each time:

* the output against the oracle (fixture experts) and against wf_moe_forward
  with a caller-provided workspace, within the layer tolerance the other tests
  use, with identical router indices and weights;
* the largest batch the static scratch holds at the V4-Flash shapes (48
  tokens), bit-identical to wf_moe_forward on the same (mma.sync) engine, and
  that the next size is rejected before anything runs;
* that an out-of-range token id on a hash layer is reported through
  wf_moe_read_error_noalloc (the kernel clamps the id; only the flag is set),
  and that reading clears it.

The file sorts last so a failure here leaves every other test already run.
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import fixtures as F
from oracle import moe_oracle as O
from tests import gpu_util as U

pytestmark = pytest.mark.gpu


def _noalloc(lib, layer, x, ids, T):
    from wanferenz_b200 import _lib as L

    y = torch.empty(T, layer.dim, dtype=torch.bfloat16, device="cuda")
    rw = torch.empty(T, layer.topk, dtype=torch.float32, device="cuda")
    ri = torch.empty(T, layer.topk, dtype=torch.int64, device="cuda")
    rc = lib.wf_moe_forward_noalloc(ctypes.byref(layer.cfg), ctypes.byref(layer.wstruct), L.ptr(x),
                                    L.ptr(ids), T, L.ptr(y), L.ptr(rw), L.ptr(ri), L.stream_ptr())
    L.check(rc, "wf_moe_forward_noalloc")
    return y, rw, ri


def test_noalloc_matches_oracle_and_workspace_forward_twice():
    from wanferenz_b200 import _lib as L

    spec = F.LayerSpec(D=512, I=256, E=16, topk=4, score_func="sqrtsoftplus", route_scale=1.5,
                       swiglu_limit=10.0, seed=61)
    syn = F.SyntheticLayer(spec)
    T = 5
    x16, ids = syn.activations(T, draw=2)
    xf = O.bf16_to_f32(x16)
    y_or, w_or, i_or = O.moe_forward(xf, syn.params(), ids)
    y_or32, _, _ = O.moe_forward(xf, syn.params(), ids, acc=np.float32)
    layer = U.device_layer(syn, np.unique(i_or), max_tokens=8)
    x = U.bf16_tensor(x16)
    y_ws, w_ws, i_ws = layer.forward(x, routing=True)
    lib = L.load()
    for call in range(2):
        y, rw, ri = _noalloc(lib, layer, x, None, T)
        torch.cuda.synchronize()
        L.check(lib.wf_moe_read_error_noalloc(L.stream_ptr()), "wf_moe_read_error_noalloc")
        assert torch.equal(ri, i_ws), f"call {call}: router indices differ from wf_moe_forward"
        assert torch.equal(rw, w_ws), f"call {call}: router weights differ from wf_moe_forward"
        np.testing.assert_array_equal(ri.cpu().numpy(), i_or)
        U.assert_layer_close_envelope(U.to_f32(y), y_or, y_or32, f"noalloc call {call} vs oracle")
        U.assert_layer_close(U.to_f32(y), U.to_f32(y_ws), f"noalloc call {call} vs workspace forward")


def test_noalloc_largest_batch_at_v4_flash_shapes(monkeypatch):
    """T = 48 fits the 4 MiB scratch at hidden 4096 / inter 2048 / 256 experts, T = 49 does
    not.  The allocation-free path runs the mma.sync engine; wf_moe_forward on that
    engine (WF_DISABLE_TC=1) gives bit-identical outputs."""
    from wanferenz_b200 import _lib as L

    syn = F.SyntheticLayer(F.CONFIG2)
    T = 48
    x16, _ = syn.activations(T, draw=4)
    layer = U.quant_layer(syn, max_tokens=T, seed=5)  # N(0, 0.02) experts, quantized
    x = U.bf16_tensor(x16)
    monkeypatch.setenv("WF_DISABLE_TC", "1")
    y_ws, w_ws, i_ws = layer.forward(x, routing=True)
    lib = L.load()
    for call in range(2):
        y, rw, ri = _noalloc(lib, layer, x, None, T)
        torch.cuda.synchronize()
        L.check(lib.wf_moe_read_error_noalloc(L.stream_ptr()), "wf_moe_read_error_noalloc")
        assert torch.equal(ri, i_ws) and torch.equal(rw, w_ws), f"call {call}: routing differs"
        assert torch.equal(y, y_ws), f"T=48 call {call}: output differs from wf_moe_forward on the same engine"
    y = torch.empty(T + 1, layer.dim, dtype=torch.bfloat16, device="cuda")
    x1 = torch.cat([x, x[:1]])
    rc = lib.wf_moe_forward_noalloc(ctypes.byref(layer.cfg), ctypes.byref(layer.wstruct), L.ptr(x1), 0,
                                    T + 1, L.ptr(y), 0, 0, L.stream_ptr())
    assert rc == L.WF_E_SHAPE
    assert "static scratch" in lib.wf_last_error().decode()


def test_noalloc_rejects_oversized_batches_before_any_launch():
    from wanferenz_b200 import _lib as L

    lib = L.load()
    cfg = L.MoeConfig(dim=4096, inter_dim=2048, n_experts=256, n_local_experts=256, expert_offset=0,
                      topk=6, score_func=1, hash_layer=0, ue8m0=1, max_tokens=256, vocab=0,
                      route_scale=1.5, swiglu_limit=0.0)
    w = L.MoeWeights()
    rc = lib.wf_moe_forward_noalloc(ctypes.byref(cfg), ctypes.byref(w), ctypes.c_void_p(16), 0, 256,
                                    ctypes.c_void_p(16), 0, 0, L.stream_ptr())
    assert rc == L.WF_E_SHAPE
    assert "static scratch" in lib.wf_last_error().decode()


def test_noalloc_reports_out_of_range_token_id():
    """A hash layer given a token id outside its vocabulary: the router clamps the id
    (no out-of-bounds read) and sets the id flag, which wf_moe_read_error_noalloc
    reports once and clears."""
    from wanferenz_b200 import _lib as L

    spec = F.LayerSpec(D=256, I=128, E=16, topk=6, score_func="sqrtsoftplus", route_scale=1.5,
                       hash_layer=True, vocab=64, seed=62)
    syn = F.SyntheticLayer(spec)
    T = 4
    x16, ids = syn.activations(T)
    layer = U.device_layer(syn, list(range(spec.E)), max_tokens=8)
    x = U.bf16_tensor(x16)
    lib = L.load()
    ok_ids = torch.from_numpy(ids).cuda()
    for call in range(2):
        _noalloc(lib, layer, x, ok_ids, T)
        assert lib.wf_moe_read_error_noalloc(L.stream_ptr()) == L.WF_OK
    bad_ids = ok_ids.clone()
    bad_ids[2] = spec.vocab + 5
    _noalloc(lib, layer, x, bad_ids, T)
    assert lib.wf_moe_read_error_noalloc(L.stream_ptr()) == L.WF_E_EXPERT_ID
    assert lib.wf_moe_read_error_noalloc(L.stream_ptr()) == L.WF_OK  # read-and-clear
    y, _, ri = _noalloc(lib, layer, x, ok_ids, T)
    assert lib.wf_moe_read_error_noalloc(L.stream_ptr()) == L.WF_OK
    y_ref, _, i_ref = O.moe_forward(O.bf16_to_f32(x16), syn.params(), ids)
    np.testing.assert_array_equal(ri.cpu().numpy(), i_ref)
    U.assert_layer_close(U.to_f32(y), y_ref, "after the error was read")
