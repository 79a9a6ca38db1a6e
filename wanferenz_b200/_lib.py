"""ctypes binding of ``libwfb200.so`` (the C ABI in ``include/wfb200.h``).

Loading fails loudly: there is no Python or CPU implementation behind these
symbols.
"""

from __future__ import annotations

import ctypes
import os

from . import _build

WF_OK = 0
WF_E_SHAPE, WF_E_DTYPE, WF_E_EXPERT_ID, WF_E_TIMEOUT, WF_E_CUDA, WF_E_RANGE, WF_E_ARG = (
    -1, -2, -3, -4, -5, -6, -7)
WF_SCALE_F32, WF_SCALE_E8M0 = 0, 1
WF_SCORE = {"softmax": 0, "sigmoid": 1, "sqrtsoftplus": 2}

# every symbol include/wfb200.h declares
EXPORTS = (
    "wf_last_error", "wf_device_sm_count", "wf_moe_workspace_bytes", "wf_moe_forward",
    "wf_moe_forward_timed",
    "wf_moe_finish", "wf_moe_route", "wf_moe_read_error", "wf_act_quant", "wf_fp4_act_quant",
    "wf_fp8_gemm", "wf_fp4_gemm", "wf_grouped_fp4_gemm", "wf_gemm_workspace_bytes",
    "wf_fp4_scales_in_range", "wf_moe_forward_noalloc", "wf_moe_forward_ep", "wf_moe_to_bf16",
    "wf_moe_sum_ranks", "wf_moe_read_error_noalloc", "wf_set_wait_limit",
    "wf_launch_count", "wf_ep_buffer_bytes", "wf_ep_alloc", "wf_ep_free", "wf_ipc_get_handle",
    "wf_ipc_open_handle", "wf_ipc_close_handle", "wf_moe_forward_ep_p2p",
)


class WfError(RuntimeError):
    """A wfb200 entry point returned a non-zero status."""

    def __init__(self, code, fn, msg):
        super().__init__(f"{fn} failed with status {code}: {msg}")
        self.code = code


class MoeConfig(ctypes.Structure):
    _fields_ = [
        ("dim", ctypes.c_int32), ("inter_dim", ctypes.c_int32), ("n_experts", ctypes.c_int32),
        ("n_local_experts", ctypes.c_int32), ("expert_offset", ctypes.c_int32),
        ("topk", ctypes.c_int32), ("score_func", ctypes.c_int32), ("hash_layer", ctypes.c_int32),
        ("ue8m0", ctypes.c_int32), ("max_tokens", ctypes.c_int32), ("vocab", ctypes.c_int64),
        ("route_scale", ctypes.c_float), ("swiglu_limit", ctypes.c_float),
    ]


class MoeWeights(ctypes.Structure):
    _fields_ = [
        ("gate_w", ctypes.c_void_p), ("gate_bias", ctypes.c_void_p), ("tid2eid", ctypes.c_void_p),
        ("w13", ctypes.c_void_p), ("w13_s", ctypes.c_void_p), ("w2", ctypes.c_void_p),
        ("w2_s", ctypes.c_void_p), ("shared_w13", ctypes.c_void_p), ("shared_s13", ctypes.c_void_p),
        ("shared_w2", ctypes.c_void_p), ("shared_s2", ctypes.c_void_p),
        ("shared_scale_kind", ctypes.c_int32),
    ]


_LIB = None
P = ctypes.c_void_p
I32, I64, SZ = ctypes.c_int32, ctypes.c_int64, ctypes.c_size_t


def _declare(lib):
    sig = {
        "wf_last_error": (ctypes.c_char_p, []),
        "wf_device_sm_count": (ctypes.c_int, []),
        "wf_moe_workspace_bytes": (SZ, [ctypes.POINTER(MoeConfig)]),
        "wf_moe_forward": (ctypes.c_int, [ctypes.POINTER(MoeConfig), ctypes.POINTER(MoeWeights), P, P,
                                          I32, P, P, P, P, P, SZ, P]),
        "wf_moe_forward_timed": (ctypes.c_int, [ctypes.POINTER(MoeConfig), ctypes.POINTER(MoeWeights),
                                                P, P, I32, P, P, P, P, P, SZ, P,
                                                ctypes.POINTER(ctypes.c_void_p)]),
        "wf_moe_finish": (ctypes.c_int, [ctypes.POINTER(MoeConfig), P, I32, I32, P, P, SZ, P]),
        "wf_moe_forward_ep": (ctypes.c_int, [ctypes.POINTER(MoeConfig), ctypes.POINTER(MoeWeights), P, I32,
                                             P, P, I32, I32, P, P, SZ, P]),
        "wf_moe_to_bf16": (ctypes.c_int, [P, I64, P, P]),
        "wf_moe_sum_ranks": (ctypes.c_int, [P, I32, I64, P, P]),
        "wf_moe_route": (ctypes.c_int, [ctypes.POINTER(MoeConfig), ctypes.POINTER(MoeWeights), P, P,
                                        I32, P, P, P, SZ, P]),
        "wf_moe_read_error": (ctypes.c_int, [P, SZ, P]),
        "wf_act_quant": (ctypes.c_int, [P, I64, I64, I32, I32, P, P, I32, P]),
        "wf_fp4_act_quant": (ctypes.c_int, [P, I64, I64, P, P, P]),
        "wf_fp8_gemm": (ctypes.c_int, [P, P, I32, P, P, I32, I64, I64, I64, P, P, SZ, P]),
        "wf_fp4_gemm": (ctypes.c_int, [P, P, I32, P, P, I64, I64, I64, P, P, SZ, P]),
        "wf_grouped_fp4_gemm": (ctypes.c_int, [P, P, I32, P, P, I64, I64, I64, P, P, SZ, P]),
        "wf_gemm_workspace_bytes": (SZ, [I64, I64, I64]),
        "wf_fp4_scales_in_range": (ctypes.c_int, [P, I64, P]),
        "wf_moe_forward_noalloc": (ctypes.c_int, [ctypes.POINTER(MoeConfig), ctypes.POINTER(MoeWeights),
                                                  P, P, I32, P, P, P, P]),
        "wf_moe_read_error_noalloc": (ctypes.c_int, [P]),
        "wf_set_wait_limit": (ctypes.c_int, [I64]),
        "wf_launch_count": (ctypes.c_uint64, []),
        "wf_ep_buffer_bytes": (SZ, [ctypes.POINTER(MoeConfig), I32]),
        "wf_ep_alloc": (ctypes.c_int, [SZ, ctypes.POINTER(ctypes.c_void_p)]),
        "wf_ep_free": (ctypes.c_int, [P]),
        "wf_ipc_get_handle": (ctypes.c_int, [P, P]),
        "wf_ipc_open_handle": (ctypes.c_int, [P, ctypes.POINTER(ctypes.c_void_p)]),
        "wf_ipc_close_handle": (ctypes.c_int, [P]),
        "wf_moe_forward_ep_p2p": (ctypes.c_int, [ctypes.POINTER(MoeConfig), ctypes.POINTER(MoeWeights), P, P,
                                                 I32, I32, I32, ctypes.POINTER(ctypes.c_void_p),
                                                 P, P, P, P, SZ, P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args


def lib_path() -> str:
    return _build.LIB


def load(build_if_missing: bool = True):
    """Loads (building first if needed) the CUDA library; raises if it cannot."""
    global _LIB
    if _LIB is not None:
        return _LIB
    path = _build.LIB
    if not os.path.exists(path):
        if not build_if_missing:
            raise ImportError(f"wanferenz_b200: CUDA library missing at {path}; run "
                              f"`python -m wanferenz_b200._build`")
        _build.build()
    lib = ctypes.CDLL(path)
    _declare(lib)
    _LIB = lib
    return lib


def check(code: int, fn: str):
    if code != WF_OK:
        msg = _LIB.wf_last_error().decode() if _LIB is not None else ""
        raise WfError(code, fn, msg)
    return code


def stream_ptr(stream=None) -> int:
    import torch

    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream)


def ptr(t) -> int:
    return 0 if t is None else int(t.data_ptr())
