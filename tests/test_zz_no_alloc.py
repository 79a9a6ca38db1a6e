"""The allocation-free forward (wf_moe_forward_noalloc) against the regular one.

For callers that cannot allocate device memory (their memory belongs to
another allocator, or they may not call the CUDA allocator while serving),
the layer can run on the library's own module-scope scratch.  This checks,
through the C ABI, that two consecutive calls of that entry point give the
same output as wf_moe_forward with a caller-provided workspace, within the
layer tolerance the other tests use.  The file sorts last so a failure here
leaves every other test already run.
"""

import ctypes

import pytest
import torch

from oracle import fixtures as F
from tests import gpu_util as U

pytestmark = pytest.mark.gpu

CASES = [
    (F.LayerSpec(D=512, I=256, E=16, topk=4, score_func="sqrtsoftplus", route_scale=1.5,
                 swiglu_limit=10.0, seed=61), 5),
    (F.CONFIG1, 8),
]


@pytest.mark.parametrize("spec,T", CASES, ids=["mini", "config1"])
def test_noalloc_matches_workspace_forward_twice(spec, T):
    from wanferenz_b200 import _lib as L

    syn = F.SyntheticLayer(spec)
    x16, _ = syn.activations(T, draw=2)
    layer = U.device_layer(syn, [], max_tokens=max(T, 8))  # experts: seeded random FP4 bytes
    x = U.bf16_tensor(x16)
    y_ref, w_ref, i_ref = layer.forward(x, routing=True)
    lib = L.load()
    for call in range(2):
        y = torch.empty_like(y_ref)
        rw = torch.empty_like(w_ref)
        ri = torch.empty_like(i_ref)
        rc = lib.wf_moe_forward_noalloc(ctypes.byref(layer.cfg), ctypes.byref(layer.wstruct), L.ptr(x),
                                        0, T, L.ptr(y), L.ptr(rw), L.ptr(ri), L.stream_ptr())
        L.check(rc, "wf_moe_forward_noalloc")
        torch.cuda.synchronize()
        assert torch.equal(ri, i_ref), f"call {call}: router indices differ"
        U.assert_layer_close(U.to_f32(y), U.to_f32(y_ref), f"noalloc call {call}")


def test_noalloc_rejects_oversized_batches():
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
