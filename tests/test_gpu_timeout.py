"""Failure detection on the GPU without a GPU fault: a device wait that runs out.

Every wait of the layer kernels on another role's progress is bounded.  The
test lowers that bound (``wf_set_wait_limit``) to a few hundred SM cycles, far
below the microseconds a weight stage or an operand takes to arrive, so some
wait runs out.  The kernels must then wind down (the drains of their own
copies and MMAs keep the long bound), set WF_E_TIMEOUT in the workspace's
error word, and leave the context usable: with the default bound restored
and the workspace re-zeroed, the next forward is correct.
"""

import numpy as np
import pytest
import torch

from oracle import fixtures as F
from oracle import moe_oracle as O
from tests import gpu_util as U

pytestmark = pytest.mark.gpu

SPEC = F.LayerSpec(D=512, I=256, E=16, topk=4, score_func="sigmoid", route_scale=1.5, seed=71)


@pytest.fixture(params=["fused", "tcgen05", "mma_sync"])
def engine(request, monkeypatch):
    monkeypatch.setenv("WF_DISABLE_TC", "1" if request.param == "mma_sync" else "0")
    monkeypatch.setenv("WF_FUSED", "1" if request.param == "fused" else "0")
    return request.param


def test_short_wait_limit_reports_timeout_and_context_recovers(engine):
    from wanferenz_b200 import _lib as L
    from wanferenz_b200.moe import MoELayer  # noqa: F401  (loads the library)

    lib = L.load()
    syn = F.SyntheticLayer(SPEC)
    T = 8
    x16, ids = syn.activations(T, draw=1)
    y_ref, _, i_ref = O.moe_forward(O.bf16_to_f32(x16), syn.params(), ids)
    layer = U.device_layer(syn, np.unique(i_ref), max_tokens=16)
    x = U.bf16_tensor(x16)
    try:
        L.check(lib.wf_set_wait_limit(200), "wf_set_wait_limit")
        layer.forward(x)
        torch.cuda.synchronize()
        rc = lib.wf_moe_read_error(L.ptr(layer.workspace), layer.workspace.numel(), L.stream_ptr())
    finally:
        lib.wf_set_wait_limit(0)
    assert rc == L.WF_E_TIMEOUT, f"expected a timed-out wait, got status {rc}"
    # the context is intact: default bound, fresh workspace, correct output
    layer.workspace.zero_()
    y, _, ri = layer.forward(x, routing=True)
    torch.cuda.synchronize()
    layer.read_error()
    np.testing.assert_array_equal(ri.cpu().numpy(), i_ref)
    U.assert_layer_close(U.to_f32(y), y_ref, f"{engine} after a timeout")
