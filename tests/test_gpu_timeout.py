"""Failure detection on the GPU without a GPU fault: a device wait that runs out.

Every wait of the layer kernels on another role's progress is bounded.  The
test lowers that bound (``wf_set_wait_limit``) to a few hundred SM cycles, far
below the microseconds a weight stage or an operand takes to arrive.  The
layer has the BASELINE config-1 shape, so every CTA streams many more weight
stages than its ring holds: some role must wait for a refill, and that wait
runs out.  The kernels must then wind down (the drains of their own copies and
MMAs keep the long bound), set WF_E_TIMEOUT in the workspace's error word, and
leave the context usable: with the default bound restored and the workspace
re-zeroed, the next forward is bit-identical to a forward run before the
timeout.
"""

import pytest
import torch

from oracle import fixtures as F
from tests import gpu_util as U

pytestmark = pytest.mark.gpu


@pytest.fixture(params=["fused", "tcgen05", "mma_sync"])
def engine(request, monkeypatch):
    monkeypatch.setenv("WF_DISABLE_TC", "1" if request.param == "mma_sync" else "0")
    monkeypatch.setenv("WF_FUSED", "1" if request.param == "fused" else "0")
    return request.param


def test_short_wait_limit_reports_timeout_and_context_recovers(engine):
    from wanferenz_b200 import _lib as L
    from wanferenz_b200.moe import MoELayer  # noqa: F401  (loads the library)

    lib = L.load()
    syn = F.SyntheticLayer(F.CONFIG1)
    T = 8
    x16, _ = syn.activations(T, draw=1)
    layer = U.device_layer(syn, [], max_tokens=16)  # routed experts: random FP4 bytes
    x = U.bf16_tensor(x16)
    y0, w0, i0 = layer.forward(x, routing=True)
    torch.cuda.synchronize()
    layer.read_error()
    assert torch.isfinite(y0.float()).all()
    try:
        L.check(lib.wf_set_wait_limit(200), "wf_set_wait_limit")
        layer.forward(x)
        torch.cuda.synchronize()
        rc = lib.wf_moe_read_error(L.ptr(layer.workspace), layer.workspace.numel(), L.stream_ptr())
    finally:
        lib.wf_set_wait_limit(0)
    assert rc == L.WF_E_TIMEOUT, f"{engine}: expected a timed-out wait, got status {rc}"
    # the context is intact: default bound, fresh workspace, the same output as before
    layer.workspace.zero_()
    y, w, i = layer.forward(x, routing=True)
    torch.cuda.synchronize()
    layer.read_error()
    assert torch.equal(i, i0) and torch.equal(w, w0), f"{engine}: routing differs after a timeout"
    assert torch.equal(y, y0), f"{engine}: output differs after a timeout"
