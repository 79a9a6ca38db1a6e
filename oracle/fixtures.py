"""Seeded synthetic MoE layers shared by the golden-vector generator and the tests.

TEST INFRASTRUCTURE ONLY (see ``oracle/moe_oracle.py``).

The reference builds its fixtures from N(0, 0.02) bf16 weights quantized with
its own quantizers (``build_real_dims_moe``, wanferenz/kernels/fp4_grouped.py:368-408;
``real_dims_args`` 411-425).  This module follows that recipe with a
platform-independent generator (numpy PCG64 seeded by a tuple), so that every
tensor can be regenerated bit-exactly, one expert at a time, on any machine:

* gate weight ``[E, D]`` N(0, 0.02) bf16; bias ``[E]`` N(0, bias_std) fp32;
* routed expert ``e``: w1, w3 ``[I, D]`` and w2 ``[D, I]`` N(0, 0.02) bf16 ->
  ``fp4_act_quant`` (packed E2M1 + e8m0 per 32 along K);
* shared expert: w1, w3 ``[I, D]``, w2 ``[D, I]`` N(0, 0.02) bf16 ->
  ``fp8_block_quant`` (e4m3 + e8m0 per 128x128);
* activations ``[T, D]`` N(0, 1) bf16;
* optional Zipf expert popularity: over a seeded
  permutation giving each expert a popularity rank r in 1..E, the gate bias
  gets ``zipf_beta * log(r ** -zipf)`` added, so expert popularity falls off
  like a Zipf(zipf) law (many experts get no token, a few get more than 16).
"""

from __future__ import annotations

import dataclasses
import hashlib

import numpy as np

from . import moe_oracle as O

TAG_GATE_W, TAG_GATE_B, TAG_W1, TAG_W3, TAG_W2 = 1, 2, 3, 4, 5
TAG_SW1, TAG_SW3, TAG_SW2, TAG_X, TAG_TID2EID, TAG_IDS = 6, 7, 8, 9, 10, 11
TAG_ZIPF = 12


def rng(*key: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(np.random.SeedSequence([int(k) for k in key])))


def normal_bf16(key, shape, std) -> np.ndarray:
    """N(0, std) rounded to bf16, as uint16 bit patterns."""
    f = rng(*key).standard_normal(size=shape, dtype=np.float32) * np.float32(std)
    return O.f32_to_bf16(f.astype(np.float32))


def sha256(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


@dataclasses.dataclass(frozen=True)
class LayerSpec:
    """One MoE layer's shapes and routing options (ModelArgs fields, architecture.py:42-93)."""

    D: int
    I: int
    E: int
    topk: int = 6
    score_func: str = "sigmoid"
    route_scale: float = 1.5
    swiglu_limit: float = 0.0
    hash_layer: bool = False
    vocab: int = 512
    bias_std: float = 0.01
    w_std: float = 0.02
    seed: int = 0
    ue8m0: bool = True
    hash_pattern: tuple = ()
    zipf: float = 0.0        # Zipf exponent of the expert popularity bias (0: uniform routing)
    zipf_beta: float = 0.08  # bias scale of the Zipf recipe

    def as_dict(self):
        return dataclasses.asdict(self)


# BASELINE.json configs 1 and 2 (config 2 at the real V4-Flash shapes)
CONFIG1 = LayerSpec(D=2048, I=1024, E=64, topk=6, score_func="sigmoid", route_scale=1.5)
CONFIG2 = LayerSpec(D=4096, I=2048, E=256, topk=6, score_func="sigmoid", route_scale=1.5)
# the config-2 layer with Zipf(1.2) expert popularity
CONFIG4 = LayerSpec(D=4096, I=2048, E=256, topk=6, score_func="sigmoid", route_scale=1.5, zipf=1.2)


def zipf_bias(seed: int, E: int, s: float, beta: float) -> np.ndarray:
    """``beta * log(rank_e ** -s)`` for a seeded popularity rank ``rank_e`` in 1..E."""
    perm = rng(seed, TAG_ZIPF).permutation(E)
    rank = np.empty(E, np.float32)
    rank[perm] = np.arange(1, E + 1, dtype=np.float32)
    return (np.float32(beta) * np.log(rank ** np.float32(-s))).astype(np.float32)


class SyntheticLayer:
    """Lazily generated weights of one layer (bf16 sources and quantized bytes)."""

    def __init__(self, spec: LayerSpec):
        self.spec = spec
        s = spec
        self.gate_w_bf16 = normal_bf16((s.seed, TAG_GATE_W), (s.E, s.D), 0.02)
        self.gate_w = O.bf16_to_f32(self.gate_w_bf16)
        if s.hash_layer:
            self.gate_b = None
            self.tid2eid = rng(s.seed, TAG_TID2EID).integers(0, s.E, size=(s.vocab, s.topk)).astype(np.int32)
            if s.hash_pattern:
                # every token lists the same experts, duplicates included
                # (the reference's own hash-routing case, fp4_grouped.py:471-474)
                self.tid2eid[:] = np.asarray(s.hash_pattern, np.int32)
        else:
            self.gate_b = (rng(s.seed, TAG_GATE_B).standard_normal(s.E, dtype=np.float32)
                           * np.float32(s.bias_std)).astype(np.float32)
            if s.zipf:
                self.gate_b = (self.gate_b + zipf_bias(s.seed, s.E, s.zipf, s.zipf_beta)).astype(np.float32)
            self.tid2eid = None
        self._experts = {}
        self._shared = None

    # -- raw bf16 sources -------------------------------------------------
    @staticmethod
    def _sources(s: LayerSpec, e: int):
        return (normal_bf16((s.seed, TAG_W1, e), (s.I, s.D), s.w_std),
                normal_bf16((s.seed, TAG_W3, e), (s.I, s.D), s.w_std),
                normal_bf16((s.seed, TAG_W2, e), (s.D, s.I), s.w_std))

    def expert_bf16(self, e):
        return self._sources(self.spec, e)

    def shared_bf16(self):
        s = self.spec
        return (normal_bf16((s.seed, TAG_SW1), (s.I, s.D), s.w_std),
                normal_bf16((s.seed, TAG_SW3), (s.I, s.D), s.w_std),
                normal_bf16((s.seed, TAG_SW2), (s.D, s.I), s.w_std))

    # -- quantized ---------------------------------------------------------
    def expert(self, e):
        """(w1, w1_s, w3, w3_s, w2, w2_s) packed E2M1 + e8m0 bytes."""
        if e not in self._experts:
            out = []
            for w in self.expert_bf16(e):
                out.extend(O.fp4_act_quant(O.bf16_to_f32(w), 32))
            self._experts[e] = tuple(out)
        return self._experts[e]

    def shared(self):
        """(w1, w1_s, w3, w3_s, w2, w2_s) e4m3 + e8m0 bytes."""
        if self._shared is None:
            out = []
            for w in self.shared_bf16():
                out.extend(O.fp8_block_quant(O.bf16_to_f32(w), 128))
            self._shared = tuple(out)
        return self._shared

    def activations(self, T, draw=0):
        s = self.spec
        x = normal_bf16((s.seed, TAG_X, T, draw), (T, s.D), 1.0)
        ids = rng(s.seed, TAG_IDS, T, draw).integers(0, s.vocab, size=(T,)).astype(np.int64)
        return x, ids

    def params(self):
        s = self.spec
        return dict(gate_w=self.gate_w, gate_b=self.gate_b, tid2eid=self.tid2eid,
                    experts=self.expert, shared=self.shared(), topk=s.topk,
                    score_func=s.score_func, route_scale=s.route_scale,
                    swiglu_limit=s.swiglu_limit, ue8m0=s.ue8m0)
