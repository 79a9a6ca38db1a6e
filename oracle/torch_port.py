"""Timed CPU baseline: the reference's MoE layer restated with torch CPU ops.

TEST INFRASTRUCTURE, not product code.  ``bench.py``'s CPU legs
(``cpu_baseline`` and ``--impl reference``) time this module, and
``tests/test_torch_port.py`` checks it against the numpy oracle
(``oracle/moe_oracle.py``), which is pinned bit-exactly to the reference's
golden vectors.  The reference's own CPU path is torch
(``wanferenz/kernels/torch_ops.py`` under ``wanferenz/model/architecture.py``):
its dequantization and matrix products run as vectorized, multi-threaded
torch ops with fp32 BLAS.  This restatement follows the same algorithm with
the same kind of ops, so the host-core timing reflects how the reference
runs, which the numpy oracle's single-threaded elementwise code does not
(~8x slower on config 2).

Inputs use the numpy oracle's parameter layout (``moe_oracle.moe_forward``):
routed experts as a callable ``e -> (w1, w1_s, w3, w3_s, w2, w2_s)`` of packed
E2M1 / e8m0 bytes, the shared expert as e4m3 / e8m0 bytes.
"""

from __future__ import annotations

import numpy as np
import torch

FP8_MAX = 448.0
_E2M1 = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                      -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], dtype=torch.float32)


def _t(a):
    return a if isinstance(a, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(a))


def _e8m0(b):
    """e8m0 bytes -> float32 powers of two."""
    return torch.ldexp(torch.ones(b.shape, dtype=torch.float32), _t(b).to(torch.int32) - 127)


def _pow2_at_or_above(x):
    """The power of two at or above ``x`` (``_round_scale``, torch_ops.py:17-21)."""
    mant, exp = torch.frexp(x)
    exp = torch.where(mant == 0.5, exp - 1, exp)
    return torch.ldexp(torch.ones_like(x), exp)


def act_quant(x, block=128, ue8m0=True):
    """``act_quant`` (torch_ops.py:33-49): E4M3 values (as float32) and per-block scales."""
    k = x.shape[-1]
    z = x.reshape(*x.shape[:-1], k // block, block)
    amax = z.abs().amax(-1, keepdim=True).clamp_min(1e-4)
    x_scaled = amax * torch.tensor(1.0 / FP8_MAX, dtype=torch.float32)
    s = _pow2_at_or_above(x_scaled) if ue8m0 else x_scaled
    q = (z / s).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn).to(torch.float32)
    return q.reshape(x.shape), s[..., 0]


def dequant_fp4(w, w_s, block=32):
    """Packed E2M1 ``[N, K/2]`` + e8m0 ``[N, K/32]`` -> float32 ``[N, K]`` (torch_ops.py:82-90)."""
    u = _t(w).to(torch.int64)
    v = torch.stack([_E2M1[u & 15], _E2M1[u >> 4]], -1).reshape(u.shape[0], -1)
    return v * _e8m0(w_s).repeat_interleave(block, -1)


def dequant_fp8(w, w_s, block=128):
    """e4m3 ``[N, K]`` + block scales ``[N/128, K/128]`` (e8m0 bytes or float32) -> float32."""
    v = _t(w).view(torch.float8_e4m3fn).to(torch.float32)
    s = _t(w_s)
    s = s.to(torch.float32) if s.dtype == torch.float32 else _e8m0(s)
    s = s.repeat_interleave(block, 0).repeat_interleave(block, 1)[: v.shape[0], : v.shape[1]]
    return v * s


def _linear(x, w_deq, ue8m0, acc=torch.float32):
    """``linear`` on a quantized weight (architecture.py:121-134): act_quant, dequantized
    product in fp32 (``acc=torch.float64``: the exact sum, rounded to fp32), bf16 output."""
    q, s = act_quant(x, 128, ue8m0)
    a = q * s.repeat_interleave(128, -1)
    return (a.to(acc) @ w_deq.to(acc).T).to(torch.float32).to(torch.bfloat16).to(torch.float32)


def _expert(x, w1, w3, w2, weights, limit, ue8m0, acc=torch.float32):
    """``Expert.forward`` (architecture.py:721-741) on dequantized weights."""
    g = _linear(x, w1, ue8m0, acc)
    u = _linear(x, w3, ue8m0, acc)
    if limit > 0:
        u = u.clamp(-limit, limit)
        g = g.clamp(max=limit)
    h = torch.nn.functional.silu(g) * u
    if weights is not None:
        h = weights * h
    return _linear(h.to(torch.bfloat16).to(torch.float32), w2, ue8m0, acc)


def gate(x, p, input_ids=None, acc=torch.float32):
    """``Gate.forward`` (architecture.py:696-718): (weights [T, k], indices [T, k])."""
    logits = (x.to(acc) @ _t(p["gate_w"]).to(acc).T).to(torch.float32)
    sf = p["score_func"]
    if sf == "softmax":
        scores = logits.softmax(-1)
    elif sf == "sigmoid":
        scores = logits.sigmoid()
    else:
        scores = torch.nn.functional.softplus(logits).sqrt()
    biased = scores + _t(p["gate_b"]).to(torch.float32) if p.get("gate_b") is not None else scores
    if p.get("tid2eid") is not None:
        indices = _t(p["tid2eid"]).to(torch.int64)[_t(input_ids).to(torch.int64)]
    else:
        indices = biased.topk(p["topk"], dim=-1).indices
    w = scores.gather(1, indices)
    if sf != "softmax":
        w = w / w.sum(-1, keepdim=True)
    return w * p["route_scale"], indices


def moe_forward(x, p, input_ids=None, acc=torch.float32, routing=None):
    """``MoE.forward`` (architecture.py:777-794): float32 ``x [T, D]`` (bf16-valued) ->
    bf16-valued float32 ``[T, D]``.  Local experts in ascending id; a token listing an
    expert twice keeps its last slot (index-put semantics).  ``acc=torch.float64``
    makes every matrix product the exact sum rounded to fp32 (the spread between the
    two shows where the reference's own summation order decides a rounding);
    ``routing=(weights, indices)`` replaces the gate."""
    x = _t(x).to(torch.float32)
    w, idx = (_t(routing[0]), _t(routing[1])) if routing is not None else gate(x, p, input_ids, acc)
    y = torch.zeros_like(x)
    ue8m0, limit = p["ue8m0"], p["swiglu_limit"]
    for e in torch.unique(idx).tolist():
        rows, slots = torch.nonzero(idx == e, as_tuple=True)
        keep = {}
        for r, s in zip(rows.tolist(), slots.tolist()):
            keep[r] = s
        toks = torch.tensor(sorted(keep), dtype=torch.int64)
        sl = torch.tensor([keep[t] for t in toks.tolist()], dtype=torch.int64)
        w1, w1_s, w3, w3_s, w2, w2_s = p["experts"](e)
        out = _expert(x[toks], dequant_fp4(w1, w1_s), dequant_fp4(w3, w3_s), dequant_fp4(w2, w2_s),
                      w[toks, sl][:, None], limit, ue8m0, acc)
        y[toks] += out
    s1, s1_s, s3, s3_s, s2, s2_s = p["shared"]
    y = y + _expert(x, dequant_fp8(s1, s1_s), dequant_fp8(s3, s3_s), dequant_fp8(s2, s2_s), None, limit, ue8m0,
                    acc)
    return y.to(torch.bfloat16).to(torch.float32)
