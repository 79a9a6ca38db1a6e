"""Parity of the CUDA MoE layer (through the C ABI) with the reference.

Golden cases compare with the reference's own outputs (tests/golden); the
other cases compare with the oracle, which is pinned bit-exactly to the
reference by tests/test_oracle_golden.py.  Router indices must be bit-exact
(rows whose k/k+1 biased-score gap is below 1e-6 are reported and skipped);
bf16 outputs must meet the tolerance in ``gpu_util.assert_layer_close``.
"""

import numpy as np
import pytest
import torch

from oracle import fixtures as F
from oracle import moe_oracle as O
from tests import golden_util as G
from tests import gpu_util as U

pytestmark = pytest.mark.gpu


def _golden_cases():
    for name in G.LAYER_FILES:
        for key in G.load(name):
            yield pytest.param(name, key, id=key)


_LAYERS = {}
_SYN = {}


def _syn(spec):
    if spec not in _SYN:
        _SYN[spec] = F.SyntheticLayer(spec)
    return _SYN[spec]


def _layer(spec, touched, **kw):
    """Device layers are cached (a few at a time) so both engines reuse one upload."""
    key = (spec, tuple(sorted(int(e) for e in touched)),
           tuple(sorted((k, v) for k, v in kw.items() if k not in ("expert_sha", "shared_sha"))))
    if key not in _LAYERS:
        while len(_LAYERS) >= 3:
            _LAYERS.pop(next(iter(_LAYERS)))
        torch.cuda.empty_cache()
        _LAYERS[key] = U.device_layer(_syn(spec), touched, **kw)
    return _LAYERS[key]


@pytest.fixture(params=["fused", "tcgen05", "mma_sync"])
def engine(request, monkeypatch):
    """Every layer engine: the three-launch tcgen05 one (default where scales are
    e8m0), the single-launch tcgen05 layer (WF_FUSED=1) and the mma.sync one."""
    monkeypatch.setenv("WF_DISABLE_TC", "1" if request.param == "mma_sync" else "0")
    monkeypatch.setenv("WF_FUSED", "1" if request.param == "fused" else "0")
    return request.param


@pytest.mark.parametrize("name,key", list(_golden_cases()))
def test_layer_matches_reference_golden(name, key, engine):
    """Every token of every golden case (up to config 4's 64 tokens with Zipf routing)
    against the reference's own outputs, on weights whose quantized bytes are checked
    against the reference's (sha256)."""
    case = G.load(name)[key]
    spec = G.spec_of(case)
    T = int(case["T"])
    syn = _syn(spec)
    x16, ids = syn.activations(T)
    touched = np.unique(case["indices"])
    sha = {int(e): str(h) for e, h in zip(case["expert_ids"], case["expert_sha"])}
    dl = _layer(spec, touched, max_tokens=max(64, T), expert_sha=sha, shared_sha=str(case["shared_sha"]))
    x = U.bf16_tensor(x16)
    y, rw, ri = dl.forward(x, torch.from_numpy(ids).cuda(), routing=True)
    torch.cuda.synchronize()
    dl.read_error()
    tie = U.near_tie_rows_from_logits(case["logits"], syn, what=f"{key} {engine}")
    np.testing.assert_array_equal(ri.cpu().numpy()[~tie], case["indices"][~tie])
    np.testing.assert_allclose(rw.cpu().numpy()[~tie], case["weights"][~tie], rtol=2e-6, atol=1e-7)
    keep = np.nonzero(~tie)[0]
    terms = U.layer_token_terms(dl, O.bf16_to_f32(x16)[keep], case["weights"][keep], case["indices"][keep])
    U.assert_layer_close_requant(U.to_f32(y)[keep], O.bf16_to_f32(case["y"])[keep], terms, f"{key} {engine}",
                                 ue8m0=spec.ue8m0, limit=spec.swiglu_limit)


ORACLE_SPECS = [
    F.LayerSpec(D=256, I=128, E=16, topk=4, score_func="sigmoid", route_scale=1.5, seed=21),
    F.LayerSpec(D=512, I=256, E=32, topk=6, score_func="sqrtsoftplus", route_scale=2.5,
                swiglu_limit=10.0, w_std=0.3, seed=22),
    F.LayerSpec(D=256, I=128, E=8, topk=2, score_func="softmax", route_scale=1.0, seed=23),
    F.LayerSpec(D=256, I=256, E=16, topk=6, score_func="sqrtsoftplus", hash_layer=True, seed=24),
    F.LayerSpec(D=256, I=128, E=16, topk=4, score_func="sigmoid", ue8m0=False, seed=25),
    F.CONFIG1,
]


@pytest.mark.parametrize("spec", ORACLE_SPECS, ids=lambda s: f"D{s.D}_E{s.E}_{s.score_func}_h{int(s.hash_layer)}_u{int(s.ue8m0)}")
@pytest.mark.parametrize("T", [1, 3, 8, 13, 40])
def test_layer_matches_oracle(spec, T, engine):
    if spec is F.CONFIG1 and T > 13:
        pytest.skip("oracle time")
    syn = _syn(spec)
    x16, ids = syn.activations(T, draw=7)
    x = O.bf16_to_f32(x16)
    y_ref, w_ref, i_ref = O.moe_forward(x, syn.params(), ids)
    y_ref32, _, _ = O.moe_forward(x, syn.params(), ids, acc=np.float32)
    dl = _layer(spec, np.unique(i_ref))
    y, rw, ri = dl.forward(U.bf16_tensor(x16), torch.from_numpy(ids).cuda(), routing=True)
    torch.cuda.synchronize()
    dl.read_error()
    tie = U.near_tie_rows(x, syn)
    np.testing.assert_array_equal(ri.cpu().numpy()[~tie], i_ref[~tie])
    U.assert_layer_close_envelope(U.to_f32(y)[~tie], y_ref[~tie], y_ref32[~tie], f"T={T}")


_PORT_REF = {}


@pytest.mark.parametrize("spec", [F.CONFIG2, F.CONFIG4], ids=["uniform", "zipf"])
def test_prefill_256_tokens_against_torch_port(spec, engine):
    """A config-5-sized layer step: 256 tokens at the V4-Flash shapes, uniform and
    Zipf(1.2) routing, every token against the torch CPU restatement of the
    reference's path (oracle/torch_port.py, pinned to the reference's golden
    vectors), evaluated with exact matrix sums.  Every routed expert is N(0, 0.02)
    quantized to FP4 (the reference's weight recipe); the shared expert is the
    fixture's."""
    import os

    from oracle import torch_port as P

    syn = _syn(spec)
    T = 256
    x16, _ = syn.activations(T, draw=9)
    xf = O.bf16_to_f32(x16)
    key = (spec, T)
    if key not in _PORT_REF:
        _LAYERS.clear()
        torch.cuda.empty_cache()
        dl = U.quant_layer(syn, max_tokens=T, seed=17)
        torch.set_num_threads(os.cpu_count() or 1)
        w, I = dl.weights, spec.I

        def experts(e):
            return tuple(t.cpu().numpy() for t in (w.w13[e, :I], w.w13_s[e, :I], w.w13[e, I:], w.w13_s[e, I:],
                                                   w.w2[e], w.w2_s[e]))

        p = syn.params()
        p["experts"] = experts
        wr, ir = P.gate(P._t(xf), p)
        y64 = P.moe_forward(xf, p, acc=torch.float64, routing=(wr, ir)).numpy()
        _PORT_REF[key] = (dl, y64, wr.numpy(), ir.numpy())
    dl, y_ref, w_ref, i_ref = _PORT_REF[key]
    counts = np.bincount(i_ref.ravel(), minlength=spec.E)
    if spec.zipf:
        assert counts.max() > 32, "Zipf routing should give experts several token groups"
    y, rw, ri = dl.forward(U.bf16_tensor(x16), routing=True)
    torch.cuda.synchronize()
    dl.read_error()
    tie = U.near_tie_rows(xf, syn, what=f"T=256 {'zipf' if spec.zipf else 'uniform'} {engine}")
    np.testing.assert_array_equal(ri.cpu().numpy()[~tie], i_ref[~tie])
    np.testing.assert_allclose(rw.cpu().numpy()[~tie], w_ref[~tie], rtol=1e-5, atol=1e-7)
    keep = np.nonzero(~tie)[0]
    terms = U.layer_token_terms(dl, xf[keep], w_ref[keep], i_ref[keep])
    U.assert_layer_close_requant(U.to_f32(y)[keep], y_ref[keep], terms, f"T=256 {engine}")


def test_checkpoint_loader_layer_matches_fixture_layer(tmp_path):
    """A layer loaded by wanferenz_b200.checkpoint from a converted checkpoint (the
    reference's tensor names and dtypes, conversion.py:55-82) gives bit-identical
    outputs to the same weights uploaded directly."""
    import dataclasses
    import json

    import safetensors.torch as ST

    from wanferenz_b200 import checkpoint

    spec = F.LayerSpec(D=512, I=256, E=16, topk=6, score_func="sqrtsoftplus", route_scale=1.5,
                       swiglu_limit=10.0, hash_layer=True, vocab=64, seed=91)
    syn = _syn(spec)
    L_ID = 0  # a hash layer (layer_id < n_hash_layers)
    dl = U.device_layer(syn, list(range(spec.E)))
    w = dl.weights
    I = spec.I
    pre = f"layers.{L_ID}.ffn."
    st = {pre + "gate.weight": w.gate_w.cpu(), pre + "gate.tid2eid": w.tid2eid.cpu()}
    for e in range(spec.E):
        for name, t, dt in (("w1.weight", w.w13[e, :I], torch.float4_e2m1fn_x2),
                            ("w3.weight", w.w13[e, I:], torch.float4_e2m1fn_x2),
                            ("w2.weight", w.w2[e], torch.float4_e2m1fn_x2),
                            ("w1.scale", w.w13_s[e, :I], torch.float8_e8m0fnu),
                            ("w3.scale", w.w13_s[e, I:], torch.float8_e8m0fnu),
                            ("w2.scale", w.w2_s[e], torch.float8_e8m0fnu)):
            st[f"{pre}experts.{e}.{name}"] = t.cpu().contiguous().view(dt)
    for name, t, dt in (("w1.weight", w.shared_w13[:I], torch.float8_e4m3fn),
                        ("w3.weight", w.shared_w13[I:], torch.float8_e4m3fn),
                        ("w2.weight", w.shared_w2, torch.float8_e4m3fn),
                        ("w1.scale", w.shared_s13[:I // 128], torch.float8_e8m0fnu),
                        ("w3.scale", w.shared_s13[I // 128:], torch.float8_e8m0fnu),
                        ("w2.scale", w.shared_s2, torch.float8_e8m0fnu)):
        st[f"{pre}shared_experts.{name}"] = t.cpu().contiguous().view(dt)
    ST.save_file(st, str(tmp_path / "model00000-mp1.safetensors"))
    cfg = dict(dim=spec.D, moe_inter_dim=I, n_routed_experts=spec.E, n_activated_experts=spec.topk,
               n_hash_layers=1, score_func=spec.score_func, route_scale=spec.route_scale,
               swiglu_limit=spec.swiglu_limit, vocab_size=spec.vocab, scale_fmt="ue8m0")
    (tmp_path / "config.json").write_text(json.dumps(cfg))
    cl = checkpoint.load_layer(str(tmp_path), L_ID, max_tokens=64)
    x16, ids = syn.activations(9, draw=4)
    x = U.bf16_tensor(x16)
    tid = torch.from_numpy(ids).cuda()
    assert torch.equal(cl.forward(x, tid), dl.forward(x, tid))
    torch.cuda.synchronize()
    cl.read_error()


def _stand_in_moe(dl, spec):
    """A module with the reference MoE's attributes (architecture.py:744-775), holding a
    device layer's weights, for the plugin entry points on a GPU box without the reference."""
    import types

    w, I = dl.weights, spec.I

    def lin(weight, scale, dt, sdt):
        return types.SimpleNamespace(weight=weight.clone().view(dt), scale=scale.clone().view(sdt))

    f4, e8 = torch.float4_e2m1fn_x2, torch.float8_e8m0fnu
    experts = [types.SimpleNamespace(w1=lin(w.w13[e, :I], w.w13_s[e, :I], f4, e8),
                                     w3=lin(w.w13[e, I:], w.w13_s[e, I:], f4, e8),
                                     w2=lin(w.w2[e], w.w2_s[e], f4, e8), swiglu_limit=spec.swiglu_limit)
               for e in range(spec.E)]
    nb = I // 128
    shared = types.SimpleNamespace(w1=lin(w.shared_w13[:I], w.shared_s13[:nb], torch.float8_e4m3fn, e8),
                                   w3=lin(w.shared_w13[I:], w.shared_s13[nb:], torch.float8_e4m3fn, e8),
                                   w2=lin(w.shared_w2, w.shared_s2, torch.float8_e4m3fn, e8))
    gate = types.SimpleNamespace(weight=w.gate_w, bias=w.gate_b, tid2eid=w.tid2eid, hash=spec.hash_layer,
                                 topk=spec.topk, score_func=spec.score_func, route_scale=spec.route_scale)
    return types.SimpleNamespace(experts=experts, shared_experts=shared, gate=gate, dim=spec.D,
                                 n_routed_experts=spec.E, experts_start_idx=0, experts_end_idx=spec.E)


def test_drafter_install_runs_the_layer():
    """install_drafter (decoding/expert_bank.py:167-196) on a drafter block: the patched
    instance forward is the B200 layer forward (bit-identical) and counts its steps."""
    import types

    import wanferenz_b200.moe as b200

    spec = F.LayerSpec(D=512, I=256, E=16, topk=6, score_func="sigmoid", route_scale=1.5, seed=92)
    syn = _syn(spec)
    dl = U.device_layer(syn, list(range(spec.E)))
    moe = _stand_in_moe(dl, spec)
    dstail = types.SimpleNamespace(mtp=[types.SimpleNamespace(ffn=moe)])
    assert b200.install_drafter(dstail, mod=types.SimpleNamespace(world_size=1, scale_fmt="ue8m0")) == 1
    x16, ids = syn.activations(5, draw=3)
    x = U.bf16_tensor(x16)
    y = moe.forward(x.view(1, 5, spec.D), torch.from_numpy(ids).cuda().view(1, 5))
    assert torch.equal(y.view(5, spec.D), dl.forward(x))
    assert moe._draft_steps == 1 and sorted(moe._grouped_bank) == ["w13", "w13_s", "w2", "w2_s"]


def test_hash_duplicates_keep_one_contribution():
    """tid2eid rows like [3,3,7,3,12,7]: each expert contributes once (fp4_grouped.py:265-268)."""
    spec = F.LayerSpec(D=256, I=128, E=16, topk=6, score_func="sqrtsoftplus", hash_layer=True,
                       hash_pattern=(3, 3, 7, 3, 12, 7), swiglu_limit=10.0, seed=31)
    syn = _syn(spec)
    x16, ids = syn.activations(5)
    y_ref, _, i_ref = O.moe_forward(O.bf16_to_f32(x16), syn.params(), ids)
    dl = _layer(spec, np.unique(i_ref))
    y, _, ri = dl.forward(U.bf16_tensor(x16), torch.from_numpy(ids).cuda(), routing=True)
    np.testing.assert_array_equal(ri.cpu().numpy(), i_ref)
    U.assert_layer_close(U.to_f32(y), y_ref, "hash dups")


def test_batch_consistency_config2(engine):
    """Full V4-Flash size: tokens alone and inside batches of 16 / 40 each meet the layer
    tolerance against the oracle (the K split of the expert GEMMs follows the batch's work
    list, so the fp32 summation order may differ between batches), and a repeated call is
    bit-identical."""
    spec = F.CONFIG2
    syn = _syn(spec)
    x16, ids = syn.activations(40, draw=3)
    n = 3
    xf = O.bf16_to_f32(x16[:n])
    y_ref, _, i_ref = O.moe_forward(xf, syn.params(), ids[:n])
    y_ref32, _, _ = O.moe_forward(xf, syn.params(), ids[:n], acc=np.float32)
    dl = _layer(spec, np.unique(i_ref))
    x = U.bf16_tensor(x16)
    y_all = dl.forward(x)
    y16 = dl.forward(x[:16])
    singles = torch.cat([dl.forward(x[t:t + 1]) for t in range(n)])
    y16b = dl.forward(x[:16])
    torch.cuda.synchronize()
    dl.read_error()
    assert torch.equal(y16, y16b)
    for y, what in ((singles, "singles"), (y16[:n], "batch 16"), (y_all[:n], "batch 40")):
        U.assert_layer_close_envelope(U.to_f32(y), y_ref, y_ref32, what)


@pytest.mark.parametrize("spec", [F.CONFIG1, ORACLE_SPECS[1]], ids=["config1", "D512"])
def test_repeated_calls_bit_identical(spec, engine):
    """30 calls on one layer give bit-identical outputs: the stream-K split, the
    issuer order and every fixed-order sum are deterministic, and a pipeline race
    (a stage read before its copy landed) shows up as a differing call."""
    syn = _syn(spec)
    dl = _layer(spec, list(range(spec.E)))
    for T in (8, 13):
        x16, _ = syn.activations(T, draw=5)
        x = U.bf16_tensor(x16)
        ys = [dl.forward(x).clone() for _ in range(30)]
        torch.cuda.synchronize()
        dl.read_error()
        bad = [i for i in range(1, len(ys)) if not torch.equal(ys[i], ys[0])]
        assert not bad, f"T={T}: calls {bad[:5]} differ from the first"


def test_expert_parallel_partials_match_oracle():
    """Two expert shards, summed partials + shared (architecture.py:785-793) vs the oracle."""
    spec = F.LayerSpec(D=512, I=256, E=16, topk=4, score_func="sigmoid", route_scale=1.5, seed=41)
    syn = _syn(spec)
    T = 7
    x16, ids = syn.activations(T)
    x = O.bf16_to_f32(x16)
    p0, _, idx = O.moe_forward(x, syn.params(), ids, expert_range=(0, 8), return_partial=True)
    p1, _, _ = O.moe_forward(x, syn.params(), ids, expert_range=(8, 16), return_partial=True)
    y_ref = O.finish_partial((p0 + p1).astype(np.float32), x, syn.params())
    touched = np.unique(idx)
    d0 = U.device_layer(syn, touched, expert_range=(0, 8))
    d1 = U.device_layer(syn, touched, expert_range=(8, 16))
    xt = U.bf16_tensor(x16)
    q0 = d0.forward(xt, partial=True)
    q1 = d1.forward(xt, partial=True)
    y = d0.finish(q0 + q1)
    np.testing.assert_allclose(q0.cpu().numpy(), p0, rtol=1e-2, atol=2e-3)
    U.assert_layer_close(U.to_f32(y), y_ref, "ep2")


@pytest.mark.parametrize("T", [1, 5, 16])
def test_token_owner_split_matches_oracle(T, engine):
    """The expert-parallel forward of ``ep_forward`` with two ranks emulated on one GPU.

    Each rank routes its own T tokens (wf_moe_route); each expert shard runs on
    the gathered 2T tokens with that routing and the shared expert on its own
    rank's rows (wf_moe_forward_ep); a rank's rows of the summed partials, cast
    to bf16, must equal the single-layer oracle (architecture.py:777-794).
    """
    spec = F.LayerSpec(D=512, I=256, E=16, topk=4, score_func="sqrtsoftplus", route_scale=1.5,
                       swiglu_limit=10.0, seed=43)
    syn = _syn(spec)
    x16, ids = syn.activations(2 * T, draw=3)
    x = O.bf16_to_f32(x16)
    y_ref, w_ref, i_ref = O.moe_forward(x, syn.params(), ids)
    y_ref32, _, _ = O.moe_forward(x, syn.params(), ids, acc=np.float32)
    touched = np.unique(i_ref)
    shards = [U.device_layer(syn, touched, expert_range=(0, 8)),
              U.device_layer(syn, touched, expert_range=(8, 16))]
    xt = U.bf16_tensor(x16)
    idt = torch.from_numpy(ids).cuda()
    own = [shards[r].route(xt[r * T:(r + 1) * T], idt[r * T:(r + 1) * T]) for r in range(2)]
    wg = torch.cat([o[0] for o in own])
    ig = torch.cat([o[1] for o in own])
    parts = [d.forward_ep(xt, wg, ig, shared_rows=(r * T, T)) for r, d in enumerate(shards)]
    y = shards[0].to_bf16(parts[0] + parts[1])
    torch.cuda.synchronize()
    for d in shards:
        d.read_error()
    tie = U.near_tie_rows(x, syn)
    np.testing.assert_array_equal(ig.cpu().numpy()[~tie], i_ref[~tie])
    np.testing.assert_allclose(wg.cpu().numpy()[~tie], w_ref[~tie], rtol=2e-6, atol=1e-7)
    U.assert_layer_close_envelope(U.to_f32(y)[~tie], y_ref[~tie], y_ref32[~tie], f"split T={T}")
    # the given routing is used as is: the oracle's, on every row; shared rows of this shard only
    p0, _, _ = O.moe_forward(x, syn.params(), None, expert_range=(0, 8), return_partial=True,
                             routing=(w_ref, i_ref))
    sh = O.expert_fp8(x[:T], *syn.shared(), weights=None, swiglu_limit=spec.swiglu_limit, ue8m0=spec.ue8m0)
    p0[:T] += sh
    q0 = shards[0].forward_ep(xt, torch.from_numpy(w_ref).cuda(), torch.from_numpy(i_ref).cuda(), (0, T))
    np.testing.assert_allclose(q0.cpu().numpy(), p0, rtol=1e-2, atol=2e-3)


def test_forward_ep_rejects_out_of_range_expert():
    spec = F.LayerSpec(D=256, I=128, E=16, topk=2, score_func="sigmoid", route_scale=1.0, seed=44)
    syn = _syn(spec)
    x16, _ = syn.activations(3)
    d = U.device_layer(syn, [], expert_range=(0, 8))
    w = torch.full((3, 2), 0.5, device="cuda")
    idx = torch.tensor([[0, 1], [2, 16], [3, 4]], dtype=torch.int64, device="cuda")
    d.forward_ep(U.bf16_tensor(x16), w, idx)
    with pytest.raises(Exception):
        d.read_error()
    ok = torch.tensor([[0, 9], [2, 15], [3, 4]], dtype=torch.int64, device="cuda")
    d.forward_ep(U.bf16_tensor(x16), w, ok)
    d.read_error()


@pytest.mark.parametrize("shared_rows", [(0, 0), (1, 2)])
def test_forward_ep_shard_without_tokens(shared_rows, engine):
    """A shard none of whose experts is routed to: zero rows, plus the shared
    expert's rows when the window holds any."""
    spec = F.LayerSpec(D=256, I=128, E=16, topk=2, score_func="sigmoid", route_scale=1.0, seed=45)
    syn = _syn(spec)
    x16, _ = syn.activations(4)
    d = U.device_layer(syn, [], expert_range=(8, 16))
    w = torch.rand(4, 2, device="cuda")
    idx = torch.tensor([[0, 1], [2, 3], [7, 4], [5, 6]], dtype=torch.int64, device="cuda")
    q = d.forward_ep(U.bf16_tensor(x16), w, idx, shared_rows)
    torch.cuda.synchronize()
    d.read_error()
    r0, n = shared_rows
    rest = torch.cat([q[:r0], q[r0 + n:]])
    assert torch.count_nonzero(rest).item() == 0
    if n:
        sh = O.expert_fp8(O.bf16_to_f32(x16)[r0:r0 + n], *syn.shared(), weights=None,
                          swiglu_limit=spec.swiglu_limit, ue8m0=spec.ue8m0)
        U.assert_layer_close(q[r0:r0 + n].cpu().numpy(), sh, "shared rows")


@pytest.mark.parametrize("P", [1, 2, 8])
def test_sum_ranks_is_ascending_rank_sum(P):
    """wf_moe_sum_ranks: left-to-right fp32 sum over ranks, then bf16 (bit-exact)."""
    from wanferenz_b200 import _lib as L

    lib = L.load()
    g = torch.Generator(device="cuda").manual_seed(P)
    parts = torch.randn(P, 5, 4096, device="cuda", generator=g) * torch.logspace(-3, 3, P, device="cuda")[:, None, None]
    acc = parts[0].clone()
    for p in range(1, P):
        acc = acc + parts[p]
    out = torch.empty(5, 4096, dtype=torch.bfloat16, device="cuda")
    L.check(lib.wf_moe_sum_ranks(L.ptr(parts), P, parts[0].numel(), L.ptr(out), L.stream_ptr()), "wf_moe_sum_ranks")
    assert torch.equal(out, acc.to(torch.bfloat16))


def test_to_bf16_rounds_to_nearest_even():
    from wanferenz_b200 import _lib as L

    lib = L.load()
    v = torch.tensor([1.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -2.5, 3.4e38, 1e-40], device="cuda")
    out = torch.empty(6, dtype=torch.bfloat16, device="cuda")
    L.check(lib.wf_moe_to_bf16(L.ptr(v), 6, L.ptr(out), L.stream_ptr()), "wf_moe_to_bf16")
    assert torch.equal(out, v.to(torch.bfloat16))


def test_shard_without_tokens_gives_zero_partial():
    spec = F.LayerSpec(D=256, I=128, E=16, topk=1, score_func="sigmoid", route_scale=1.0, seed=42)
    syn = _syn(spec)
    x16, ids = syn.activations(1)
    _, _, idx = O.moe_forward(O.bf16_to_f32(x16), syn.params(), ids, return_partial=True)
    e = int(idx[0, 0])
    lo = 0 if e >= 8 else 8
    d = U.device_layer(syn, [], expert_range=(lo, lo + 8))
    q = d.forward(U.bf16_tensor(x16), partial=True)
    assert torch.count_nonzero(q).item() == 0


def test_cuda_graph_replay_matches_eager():
    """forward allocates nothing and never syncs, so it replays from a CUDA graph."""
    spec = F.CONFIG1
    syn = _syn(spec)
    dl = _layer(spec, [])
    x16a, _ = syn.activations(4, draw=11)
    x16b, _ = syn.activations(4, draw=12)
    xa, xb = U.bf16_tensor(x16a), U.bf16_tensor(x16b)
    x_static = xa.clone()
    y_static = torch.empty(4, spec.D, dtype=torch.bfloat16, device="cuda")
    dl.forward(x_static, out=y_static)  # warm-up outside capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        dl.forward(x_static, out=y_static)
    x_static.copy_(xb)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(y_static, dl.forward(xb))
