"""Operator API of ``wanferenz.kernels.reference`` on the B200 kernels.

Same names, arguments and return values as the reference's operators
(wanferenz/kernels/reference.py and its CPU twin wanferenz/kernels/torch_ops.py),
so ``architecture.linear()`` can bind them unchanged:

* ``act_quant(x, block_size=128, scale_fmt=None, scale_dtype=torch.float32, inplace=False)``
* ``fp4_act_quant(x, block_size=32, inplace=False)``
* ``fp8_gemm(a, a_s, b, b_s, scale_dtype=torch.float32)``
* ``fp4_gemm(a, a_s, b, b_s, scale_dtype=torch.float32)``
* ``grouped_fp4_gemm(a, a_s, w, w_s, scale_dtype=torch.float32)`` (fp4_grouped.py:96-128)

All tensors must be CUDA tensors; there is no CPU path.  Outputs are bf16,
as the reference's are under the model's bf16 default dtype.
"""

from __future__ import annotations

import torch

from . import _lib as L

_GEMM_WS = {}


def _need_cuda(*ts):
    for t in ts:
        if not t.is_cuda:
            raise ValueError("wanferenz_b200 operators run on CUDA tensors only")


def _kind(s: torch.Tensor) -> int:
    if s.dtype == torch.float32:
        return L.WF_SCALE_F32
    if s.dtype == torch.float8_e8m0fnu:
        return L.WF_SCALE_E8M0
    raise TypeError(f"unsupported scale dtype {s.dtype}")


def _u8(t: torch.Tensor) -> torch.Tensor:
    return t.contiguous().view(torch.uint8)


def _gemm_ws(device, m, n, k) -> torch.Tensor:
    """Per-device workspace, grown to the largest (M, N, K) seen; zero-filled when allocated
    (its split-K counters return to zero after every call)."""
    need = L.load().wf_gemm_workspace_bytes(m, n, k)
    if need == 0:
        raise ValueError(f"unsupported GEMM shape M={m} N={n} K={k}")
    key = (device.type, device.index)
    ws = _GEMM_WS.get(key)
    if ws is None or ws.numel() < need:
        ws = _GEMM_WS[key] = torch.zeros(need, dtype=torch.uint8, device=device)
    return ws


def act_quant(x, block_size=128, scale_fmt=None, scale_dtype=torch.float32, inplace=False):
    """Per-``block_size`` E4M3 quantization (torch_ops.py:33-49; reference.py:117-146)."""
    _need_cuda(x)
    lib = L.load()
    z = x.contiguous()
    if z.dtype != torch.bfloat16:
        raise TypeError("act_quant expects bf16 input")
    n = z.size(-1)
    if n % block_size:
        raise ValueError(f"last dim {n} is not a multiple of {block_size}")
    m = z.numel() // n
    y = torch.empty(z.shape, dtype=torch.float8_e4m3fn, device=z.device)
    s = torch.empty(*z.shape[:-1], n // block_size, dtype=scale_dtype, device=z.device)
    L.check(lib.wf_act_quant(L.ptr(z), m, n, block_size, int(scale_fmt is not None), L.ptr(y),
                             L.ptr(s), _kind(s), L.stream_ptr()), "wf_act_quant")
    if inplace:
        deq = y.float() * s.float().repeat_interleave(block_size, -1)
        x.copy_(deq.to(x.dtype))
        return x
    return y, s


def fp4_act_quant(x, block_size=32, inplace=False):
    """Per-32 E2M1 quantization with UE8M0 scales (torch_ops.py:61-74; reference.py:212-232)."""
    _need_cuda(x)
    if block_size != 32:
        raise ValueError("fp4_act_quant supports block_size=32 only")
    lib = L.load()
    z = x.contiguous()
    n = z.size(-1)
    m = z.numel() // n
    q = torch.empty(*z.shape[:-1], n // 2, dtype=torch.uint8, device=z.device)
    s = torch.empty(*z.shape[:-1], n // 32, dtype=torch.uint8, device=z.device)
    L.check(lib.wf_fp4_act_quant(L.ptr(z), m, n, L.ptr(q), L.ptr(s), L.stream_ptr()),
            "wf_fp4_act_quant")
    q = q.view(torch.float4_e2m1fn_x2)
    s = s.view(torch.float8_e8m0fnu)
    if inplace:
        from . import moe as _moe

        x.copy_(_moe.dequant_fp4(q, s).to(x.dtype))
        return x
    return q, s


def _out(a, n):
    return torch.empty(*a.shape[:-1], n, dtype=torch.bfloat16, device=a.device)


def fp8_gemm(a, a_s, b, b_s, scale_dtype=torch.float32):
    """``C = (a*a_s) @ (b*b_s)^T`` for E4M3 ``a [.., K]``, ``b [N, K]`` with 128x128 weight blocks."""
    _need_cuda(a, a_s, b, b_s)
    lib = L.load()
    k, n = a.size(-1), b.size(0)
    m = a.numel() // k
    c = _out(a, n)
    ws = _gemm_ws(a.device, m, n, k)
    L.check(lib.wf_fp8_gemm(L.ptr(_u8(a)), L.ptr(a_s.contiguous()), _kind(a_s), L.ptr(_u8(b)),
                            L.ptr(b_s.contiguous()), _kind(b_s), m, n, k, L.ptr(c), L.ptr(ws),
                            ws.numel(), L.stream_ptr()), "wf_fp8_gemm")
    return c


def fp4_gemm(a, a_s, b, b_s, scale_dtype=torch.float32):
    """``C = (a*a_s) @ (unpack(b)*b_s)^T`` for E4M3 ``a [.., K]`` and packed E2M1 ``b [N, K/2]``."""
    _need_cuda(a, a_s, b, b_s)
    lib = L.load()
    k, n = a.size(-1), b.size(0)
    m = a.numel() // k
    c = _out(a, n)
    ws = _gemm_ws(a.device, m, n, k)
    L.check(lib.wf_fp4_gemm(L.ptr(_u8(a)), L.ptr(a_s.contiguous()), _kind(a_s), L.ptr(_u8(b)),
                            L.ptr(_u8(b_s)), m, n, k, L.ptr(c), L.ptr(ws), ws.numel(),
                            L.stream_ptr()), "wf_fp4_gemm")
    return c


def grouped_fp4_gemm(a, a_s, w, w_s, scale_dtype=torch.float32):
    """Slot ``g`` multiplies ``a[g]`` by its own FP4 weights ``w[g]`` (fp4_grouped.py:96-128)."""
    _need_cuda(a, a_s, w, w_s)
    lib = L.load()
    g, k = a.shape
    n = w.size(1)
    c = torch.empty(g, n, dtype=torch.bfloat16, device=a.device)
    ws = _gemm_ws(a.device, g, n, k)
    L.check(lib.wf_grouped_fp4_gemm(L.ptr(_u8(a)), L.ptr(a_s.contiguous()), _kind(a_s),
                                    L.ptr(_u8(w)), L.ptr(_u8(w_s)), g, n, k, L.ptr(c), L.ptr(ws),
                                    ws.numel(), L.stream_ptr()), "wf_grouped_fp4_gemm")
    return c


OPERATORS = {
    "act_quant": act_quant,
    "fp4_act_quant": fp4_act_quant,
    "fp8_gemm": fp8_gemm,
    "fp4_gemm": fp4_gemm,
}
