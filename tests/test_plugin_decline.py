"""The layer plugin's decline convention, on the host (no GPU needed).

The reference plugins never raise for a configuration they do not cover: they
count the reason and call the forward they replaced (fp4_grouped.py:256-262,
339-351).  ``wanferenz_b200.moe.b200_forward`` does the same for
``WfUnsupported`` configurations, here a MoE whose routed experts are bf16.
"""

import types

import torch

import wanferenz_b200.moe as b200


def _bf16_moe():
    lin = lambda: types.SimpleNamespace(weight=torch.zeros(4, 4, dtype=torch.bfloat16))  # noqa: E731
    expert = types.SimpleNamespace(w1=lin(), w2=lin(), w3=lin())
    return types.SimpleNamespace(experts=[expert, expert], experts_start_idx=0, experts_end_idx=2, dim=4)


def test_unsupported_layer_declines_to_the_replaced_forward(monkeypatch):
    calls = []

    def ref_forward(self, x, input_ids):
        calls.append((self, x, input_ids))
        return x + 1

    monkeypatch.setattr(b200, "_REF_FORWARD", ref_forward)
    moe = _bf16_moe()
    x = torch.zeros(1, 1, 4)
    ids = torch.zeros(1, 1, dtype=torch.int64)
    for step in (1, 2):
        y = b200.b200_forward(moe, x, ids)
        assert torch.equal(y, x + 1)
        assert moe._grouped_declined == {"routed experts are not FP4": step}
    assert len(calls) == 2 and calls[0][0] is moe
    assert moe._wf_layer is False  # the bank is not rebuilt on every step
    assert getattr(moe, "_grouped_steps", 0) == 0


def test_install_without_cuda_raises_instead_of_falling_back(monkeypatch):
    monkeypatch.setattr(torch.cuda, "is_available", lambda: False)
    mod = types.SimpleNamespace(MoE=type("MoE", (), {"forward": lambda self, x, ids: x}))
    try:
        b200.install(mod)
    except RuntimeError as e:
        assert "no CUDA device" in str(e)
    else:
        raise AssertionError("install must refuse without a CUDA device")
    assert not getattr(mod.MoE.forward, "_wf_b200", False)
