"""CPU restatement (numpy) of WANferenz's decode-time quantized MoE layer.

TEST INFRASTRUCTURE ONLY.  This module is the parity checker for the CUDA
path in ``wanferenz_b200``: only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it.  The
product path never calls it and has no CPU fallback.

Every function restates one step of the reference's own CPU operator backend
(``wanferenz/kernels/torch_ops.py``) or model code
(``wanferenz/model/architecture.py``); each docstring cites the file:line it
follows.  Arrays use these conventions:

* bf16 tensors are carried as ``uint16`` bit patterns;
* e4m3 / e8m0 / packed-e2m1 tensors are carried as ``uint8`` bytes;
* all arithmetic the reference does in fp32 is done in ``float32`` here,
  except matrix products, which accumulate in ``acc`` (``float64`` by default,
  i.e. the correctly rounded fp32 value of the exact sum; ``float32`` mirrors
  the reference's sgemm cost for CPU-baseline timing).
"""

from __future__ import annotations

import numpy as np

FP8_MAX = np.float32(448.0)
FP4_MAX = np.float32(6.0)
FP8_MAX_INV = np.float32(1.0 / 448.0)
FP4_MAX_INV = np.float32(1.0 / 6.0)
E2M1_VALUES = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], np.float32)
E2M1_MID = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], np.float32)

SCORE_FUNCS = ("softmax", "sigmoid", "sqrtsoftplus")


# --------------------------------------------------------------------------
# scalar formats
# --------------------------------------------------------------------------

def bf16_to_f32(u16: np.ndarray) -> np.ndarray:
    """bf16 bit patterns -> float32 (exact)."""
    return (np.asarray(u16, np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(f: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns, round-to-nearest-even (torch ``.to(bfloat16)``)."""
    u = np.ascontiguousarray(f, np.float32).view(np.uint32)
    nan = np.isnan(f)
    r = ((u + np.uint32(0x7FFF) + ((u >> 16) & np.uint32(1))) >> 16).astype(np.uint16)
    if nan.any():
        r = np.where(nan, np.uint16(0x7FC0), r)
    return r


def round_bf16(f: np.ndarray) -> np.ndarray:
    """float32 value rounded through bf16 and back."""
    return bf16_to_f32(f32_to_bf16(f))


def e4m3_round(q: np.ndarray) -> np.ndarray:
    """Nearest e4m3fn value (ties to even) of float32 ``q`` already clamped to +-448.

    Restates torch's ``.to(torch.float8_e4m3fn)`` cast used by ``act_quant``
    (``wanferenz/kernels/torch_ops.py:48``).
    """
    q = np.asarray(q, np.float32)
    a = np.abs(q)
    _, e = np.frexp(a)
    step = np.maximum(e - 4, -9)  # 3 mantissa bits; subnormal step 2^-9
    r = np.ldexp(np.rint(np.ldexp(a, -step)), step).astype(np.float32)
    return np.copysign(r, q).astype(np.float32)


def e4m3_encode(v: np.ndarray) -> np.ndarray:
    """e4m3fn-representable float32 values -> bytes."""
    v = np.asarray(v, np.float32)
    a = np.abs(v)
    m, e = np.frexp(a)  # a = m * 2^e, m in [0.5, 1)
    normal = a >= np.float32(2.0 ** -6)
    ef = np.where(normal, e - 1 + 7, 0)
    mant = np.where(normal, np.ldexp(m, 4) - 8, np.ldexp(a, 9))
    code = (ef.astype(np.int64) << 3) | mant.astype(np.int64)
    code = np.where(a == 0, 0, code)
    sign = np.signbit(v).astype(np.int64) << 7
    return (code | sign).astype(np.uint8)


def e4m3_decode(b: np.ndarray) -> np.ndarray:
    """e4m3fn bytes -> float32 (0x7F / 0xFF decode to NaN)."""
    b = np.asarray(b, np.uint8).astype(np.int64)
    s = np.where(b & 0x80, -1.0, 1.0)
    ef = (b >> 3) & 0xF
    mf = b & 7
    val = np.where(ef == 0, mf * 2.0 ** -9, (8 + mf) * np.ldexp(1.0, ef - 10))
    val = np.where((b & 0x7F) == 0x7F, np.nan, val)
    return (s * val).astype(np.float32)


def e8m0_decode(b: np.ndarray) -> np.ndarray:
    """e8m0fnu bytes -> float32 powers of two (0xFF decodes to NaN)."""
    b = np.asarray(b, np.uint8).astype(np.int64)
    v = np.ldexp(np.float64(1.0), b - 127)
    v = np.where(b == 255, np.nan, v)
    return v.astype(np.float32)


def e8m0_encode(s: np.ndarray) -> np.ndarray:
    """Exact powers of two -> e8m0fnu bytes (torch ``.to(float8_e8m0fnu)`` on powers of two)."""
    s = np.asarray(s, np.float32)
    _, e = np.frexp(s)
    return (e - 1 + 127).astype(np.uint8)


# --------------------------------------------------------------------------
# quantizers
# --------------------------------------------------------------------------

def round_scale(amax: np.ndarray, max_inv: np.float32) -> np.ndarray:
    """``_round_scale`` (torch_ops.py:17-21): the power of two at or above ``amax * max_inv``."""
    x = (np.asarray(amax, np.float32) * np.float32(max_inv)).astype(np.float32)
    mant, exp = np.frexp(x)
    exp = np.where(mant == 0.5, exp - 1, exp)
    return np.ldexp(np.ones_like(x), exp).astype(np.float32)


def act_quant(x: np.ndarray, block: int = 128, ue8m0: bool = True):
    """``act_quant`` (torch_ops.py:33-49; TileLang twin reference.py:40-146).

    ``x`` float32 ``[..., K]`` (bf16-valued).  Returns ``(q, s)`` where ``q`` are
    the e4m3 values as float32 (same shape) and ``s`` the per-block float32
    scales ``[..., K/block]`` (powers of two when ``ue8m0``; ``amax/448``
    otherwise, as when the reference's ``scale_fmt`` is ``None``).
    """
    x = np.asarray(x, np.float32)
    k = x.shape[-1]
    assert k % block == 0, f"last dim {k} not a multiple of {block}"
    z = x.reshape(*x.shape[:-1], k // block, block)
    amax = np.maximum(np.abs(z).max(-1, keepdims=True), np.float32(1e-4))
    if ue8m0:
        s = round_scale(amax, FP8_MAX_INV)
    else:
        s = (amax * FP8_MAX_INV).astype(np.float32)
    q = np.clip((z / s).astype(np.float32), -FP8_MAX, FP8_MAX)
    q = e4m3_round(q)
    return q.reshape(x.shape), s[..., 0]


def _e2m1_codes(a: np.ndarray) -> np.ndarray:
    """``_e2m1`` (torch_ops.py:52-58): nearest E2M1 code of ``|q|``, ties to the even code."""
    lo = np.searchsorted(E2M1_MID, a, side="left")
    hi = np.searchsorted(E2M1_MID, a, side="right")
    return lo + ((hi != lo) & (lo % 2 == 1)).astype(lo.dtype)


def fp4_act_quant(x: np.ndarray, block: int = 32):
    """``fp4_act_quant`` (torch_ops.py:61-74; TileLang twin reference.py:149-232).

    ``x`` float32 ``[N, K]`` (bf16-valued) -> packed E2M1 bytes ``[N, K/2]`` (low
    nibble = even k) and e8m0 scale bytes ``[N, K/block]``.
    """
    x = np.asarray(x, np.float32)
    n, k = x.shape
    z = x.reshape(n, k // block, block)
    amax = np.maximum(np.abs(z).max(-1, keepdims=True), np.float32(6.0 * 2.0 ** -126))
    s = round_scale(amax, FP4_MAX_INV)
    q = np.clip((z / s).astype(np.float32), -FP4_MAX, FP4_MAX)
    code = _e2m1_codes(np.abs(q).ravel()).reshape(q.shape).astype(np.uint8)
    code = code | ((q < 0).astype(np.uint8) << 3)
    code = code.reshape(n, k)
    packed = (code[:, 0::2] | (code[:, 1::2] << 4)).astype(np.uint8)
    return packed, e8m0_encode(s[..., 0])


def fp8_block_quant(w: np.ndarray, block: int = 128):
    """``_fp8_block_quant`` (wanferenz/kernels/fp4_grouped.py:354-365).

    ``w`` float32 ``[N, K]`` -> e4m3 bytes ``[N, K]`` and e8m0 scale bytes
    ``[N/block, K/block]`` with scale ``2^ceil(log2(amax/448))``, amax floored at 1e-4.
    """
    w = np.asarray(w, np.float32)
    n, k = w.shape
    b = w.reshape(n // block, block, k // block, block)
    amax = np.maximum(np.abs(b).max(axis=(1, 3)), np.float32(1e-4))
    scale = np.power(np.float32(2.0), np.ceil(np.log2((amax / FP8_MAX).astype(np.float32)))).astype(np.float32)
    q = np.clip((b / scale[:, None, :, None]).astype(np.float32), -FP8_MAX, FP8_MAX)
    q = e4m3_round(q).reshape(n, k)
    return e4m3_encode(q), e8m0_encode(scale)


def unpack_fp4(packed: np.ndarray) -> np.ndarray:
    """``unpack_fp4`` (torch_ops.py:82-90): packed bytes ``[N, K/2]`` -> float32 values ``[N, K]``."""
    u = np.asarray(packed, np.uint8)
    table = np.concatenate([E2M1_VALUES, -E2M1_VALUES]).astype(np.float32)
    out = np.empty(u.shape[:-1] + (u.shape[-1] * 2,), np.float32)
    out[..., 0::2] = table[u & 0x0F]
    out[..., 1::2] = table[u >> 4]
    return out


# --------------------------------------------------------------------------
# GEMMs (dequantize, multiply, round to bf16)
# --------------------------------------------------------------------------

def _matmul_bf16(da: np.ndarray, db: np.ndarray, acc) -> np.ndarray:
    c = np.asarray(da, acc) @ np.asarray(db, acc).T
    return round_bf16(c.astype(np.float32))


def dequant_fp4(w: np.ndarray, w_s: np.ndarray, block: int = 32) -> np.ndarray:
    """Packed E2M1 weight ``[N, K/2]`` + e8m0 scales ``[N, K/32]`` -> float32 ``[N, K]``."""
    v = unpack_fp4(w)
    return (v * np.repeat(e8m0_decode(w_s), block, axis=-1)[:, : v.shape[-1]]).astype(np.float32)


def dequant_fp8(w: np.ndarray, w_s: np.ndarray, block: int = 128) -> np.ndarray:
    """e4m3 weight ``[N, K]`` + block scales ``[ceil(N/128), ceil(K/128)]`` (e8m0 bytes or float32)."""
    v = e4m3_decode(w)
    s = w_s if w_s.dtype == np.float32 else e8m0_decode(w_s)
    s = np.repeat(np.repeat(s, block, axis=0), block, axis=1)[: v.shape[0], : v.shape[1]]
    return (v * s).astype(np.float32)


def fp4_gemm(a_q, a_s, w, w_s, acc=np.float64):
    """``fp4_gemm`` (torch_ops.py:102-108): ``(a_q*a_s) @ (unpack(w)*w_s)^T`` -> bf16-valued float32."""
    k = a_q.shape[-1]
    da = (a_q * np.repeat(a_s, 128, axis=-1)[..., :k]).astype(np.float32)
    return _matmul_bf16(da, dequant_fp4(w, w_s), acc)


def fp8_gemm(a_q, a_s, w, w_s, acc=np.float64):
    """``fp8_gemm`` (torch_ops.py:93-99): ``(a_q*a_s) @ (w*w_s)^T`` -> bf16-valued float32."""
    k = a_q.shape[-1]
    da = (a_q * np.repeat(a_s, 128, axis=-1)[..., :k]).astype(np.float32)
    return _matmul_bf16(da, dequant_fp8(w, w_s), acc)


# --------------------------------------------------------------------------
# the layer
# --------------------------------------------------------------------------

def _sigmoid(x):
    return (np.float32(1.0) / (np.float32(1.0) + np.exp(-x))).astype(np.float32)


def _softplus(x):
    # torch F.softplus(beta=1, threshold=20)
    return np.where(x > 20, x, np.log1p(np.exp(np.minimum(x, 20)))).astype(np.float32)


def gate_scores(x, gate_w, score_func, acc=np.float64):
    """Scores of ``Gate.forward`` (architecture.py:699-705) before bias and top-k.

    ``x`` float32 ``[T, D]``; ``gate_w`` float32 ``[E, D]`` (bf16-valued).
    Returns ``(logits, scores)`` float32 ``[T, E]``.
    """
    logits = (np.asarray(x, acc) @ np.asarray(gate_w, acc).T).astype(np.float32)
    if score_func == "softmax":
        m = logits.max(-1, keepdims=True)
        e = np.exp(logits - m).astype(np.float32)
        scores = (e / e.sum(-1, keepdims=True, dtype=np.float32)).astype(np.float32)
    elif score_func == "sigmoid":
        scores = _sigmoid(logits)
    elif score_func == "sqrtsoftplus":
        scores = np.sqrt(_softplus(logits)).astype(np.float32)
    else:
        raise ValueError(score_func)
    return logits, scores


def gate(x, gate_w, bias, topk, score_func, route_scale, tid2eid=None, input_ids=None, acc=np.float64):
    """``Gate.forward`` (architecture.py:696-718).

    Returns ``(weights float32 [T,k], indices int64 [T,k], biased_scores float32 [T,E])``.
    Indices are ordered by descending biased score (torch ``topk``); equal
    scores keep the lower expert id first.  Hash layers (``tid2eid`` given)
    take ``tid2eid[input_ids]`` (architecture.py:710-711).
    """
    _, scores = gate_scores(x, gate_w, score_func, acc)
    original = scores
    biased = scores + bias.astype(np.float32) if bias is not None else scores
    biased = biased.astype(np.float32)
    if tid2eid is not None:
        indices = np.asarray(tid2eid)[np.asarray(input_ids)].astype(np.int64)
    else:
        order = np.argsort(-biased, axis=-1, kind="stable")
        indices = order[:, :topk].astype(np.int64)
    weights = np.take_along_axis(original, indices, axis=1).astype(np.float32)
    if score_func != "softmax":
        weights = (weights / weights.sum(-1, keepdims=True, dtype=np.float32)).astype(np.float32)
    weights = (weights * np.float32(route_scale)).astype(np.float32)
    return weights, indices, biased


def topk_margin(biased: np.ndarray, topk: int) -> np.ndarray:
    """Per token, the gap between the k-th and (k+1)-th biased score.

    A gap within a few fp32 ulps means a CPU fp32 sgemm and any other
    summation order may legitimately disagree on the expert set.
    """
    s = -np.sort(-biased, axis=-1)
    if s.shape[-1] <= topk:
        return np.full(s.shape[0], np.inf, np.float32)
    return (s[:, topk - 1] - s[:, topk]).astype(np.float32)


def _silu(g):
    # exp(-g) overflows to inf for g < -88: g / inf = -0, silu's limit
    with np.errstate(over="ignore"):
        return (g / (np.float32(1.0) + np.exp(-g))).astype(np.float32)


def expert_fp4(x, w1, w1_s, w3, w3_s, w2, w2_s, weights=None, swiglu_limit=0.0, ue8m0=True, acc=np.float64):
    """``Expert.forward`` (architecture.py:728-741) on FP4 weights via ``linear`` (121-134).

    ``x`` float32 ``[t, D]`` bf16-valued; ``weights`` float32 ``[t, 1]`` or None.
    Returns bf16-valued float32 ``[t, D]``.
    """
    xq, xs = act_quant(x, 128, ue8m0)
    g = fp4_gemm(xq, xs, w1, w1_s, acc)
    u = fp4_gemm(xq, xs, w3, w3_s, acc)
    h = _swiglu(g, u, weights, swiglu_limit)
    hq, hs = act_quant(h, 128, ue8m0)
    return fp4_gemm(hq, hs, w2, w2_s, acc)


def expert_fp8(x, w1, w1_s, w3, w3_s, w2, w2_s, weights=None, swiglu_limit=0.0, ue8m0=True, acc=np.float64):
    """``Expert.forward`` (architecture.py:728-741) on FP8 block-scaled weights (the shared expert)."""
    xq, xs = act_quant(x, 128, ue8m0)
    g = fp8_gemm(xq, xs, w1, w1_s, acc)
    u = fp8_gemm(xq, xs, w3, w3_s, acc)
    h = _swiglu(g, u, weights, swiglu_limit)
    hq, hs = act_quant(h, 128, ue8m0)
    return fp8_gemm(hq, hs, w2, w2_s, acc)


def _swiglu(g, u, weights, limit):
    """architecture.py:733-741: clamp, ``silu(gate) * up``, ``* weights``, round to bf16."""
    g = g.astype(np.float32)
    u = u.astype(np.float32)
    if limit > 0:
        lim = np.float32(limit)
        u = np.clip(u, -lim, lim)
        g = np.minimum(g, lim)
    h = (_silu(g) * u).astype(np.float32)
    if weights is not None:
        h = (np.asarray(weights, np.float32) * h).astype(np.float32)
    return round_bf16(h)


def moe_forward(x, params, input_ids=None, expert_range=None, acc=np.float64, return_partial=False,
                routing=None):
    """``MoE.forward`` (architecture.py:777-794).

    ``x`` float32 ``[T, D]`` bf16-valued.  ``params`` is a dict:

    * ``gate_w`` float32 [E, D], ``gate_b`` float32 [E] or None, ``tid2eid`` int [V, k] or None
    * ``experts``: callable ``e -> (w1, w1_s, w3, w3_s, w2, w2_s)`` bytes (packed E2M1 + e8m0)
    * ``shared``: tuple ``(w1, w1_s, w3, w3_s, w2, w2_s)`` (e4m3 + e8m0 bytes)
    * ``topk``, ``score_func``, ``route_scale``, ``swiglu_limit``, ``ue8m0``

    The routed sum runs over local experts in ascending id (785-790); a token
    that lists an expert twice (hash layers) keeps one contribution, the one
    of its last slot (index-put semantics, fp4_grouped.py:265-268).
    ``expert_range=(lo, hi)`` restricts to one expert-parallel shard (749-756);
    with ``return_partial`` the fp32 routed partial sum is returned before the
    all-reduce and shared expert (791-793).  ``routing=(weights, indices)``
    replaces the gate with a routing computed elsewhere (the expert-parallel
    split routes each token once, on the rank that owns it).
    Returns ``(y bf16-valued float32 [T, D], weights, indices)``.
    """
    T, D = x.shape
    if routing is not None:
        weights = np.asarray(routing[0], np.float32)
        indices = np.asarray(routing[1], np.int64)
    else:
        weights, indices, _ = gate(
            x, params["gate_w"], params.get("gate_b"), params["topk"], params["score_func"],
            params["route_scale"], params.get("tid2eid"), input_ids, acc)
    E = params["gate_w"].shape[0]
    lo, hi = expert_range if expert_range is not None else (0, E)
    y = np.zeros((T, D), np.float32)
    for e in range(lo, hi):
        rows, slots = np.nonzero(indices == e)
        if rows.size == 0:
            continue
        # keep the last slot of each duplicated token (index-put: last write wins)
        keep = {}
        for r, s in zip(rows.tolist(), slots.tolist()):
            keep[r] = s
        toks = np.array(sorted(keep), np.int64)
        sl = np.array([keep[t] for t in toks.tolist()], np.int64)
        out = expert_fp4(x[toks], *params["experts"](e), weights=weights[toks, sl][:, None],
                         swiglu_limit=params["swiglu_limit"], ue8m0=params["ue8m0"], acc=acc)
        y[toks] = (y[toks] + out).astype(np.float32)
    if return_partial:
        return y, weights, indices
    sh = expert_fp8(x, *params["shared"], weights=None, swiglu_limit=params["swiglu_limit"],
                    ue8m0=params["ue8m0"], acc=acc)
    y = (y + sh).astype(np.float32)
    return round_bf16(y), weights, indices


def finish_partial(y_partial, x, params, acc=np.float64):
    """Ends an expert-parallel forward: ``y += shared(x)`` then bf16 (architecture.py:793-794)."""
    sh = expert_fp8(x, *params["shared"], weights=None, swiglu_limit=params["swiglu_limit"],
                    ue8m0=params["ue8m0"], acc=acc)
    return round_bf16((y_partial + sh).astype(np.float32))
