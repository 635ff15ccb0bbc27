"""Pin the CPU oracle against vectors produced by the reference itself.

``tests/golden/make_golden.py`` ran the reference's ``_router_split_gap`` and
vLLM's CPU routing / MoE functions; these tests check that the oracle
restatements reproduce them exactly (integer state) or bit-for-bit / within
one fp32 ulp (floating point).
"""

import json
import os

import numpy as np
import pytest
import torch

from oracle import moe as omoe
from oracle import routing as orouting
from oracle.slot_policy import PROBATION, PROTECTED, SlotOverflow, SlotPolicyModel
from sluice_b200.offloader import max_waves_for, plan_ids_for, waves_pingpong

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _scenarios():
    with open(os.path.join(GOLDEN, "slot_traces.json")) as f:
        return json.load(f)["scenarios"]


def model_for(sc) -> SlotPolicyModel:
    m = SlotPolicyModel(sc["num_slots"], sc["local_of"], sc["local_n"],
                        protect_frac=sc["protect_frac"], fast_hit=sc["fast_hit"],
                        prefill_resident=sc["prefill_resident"], lfu=sc.get("lfu", False))
    if sc["pins"]:
        m.apply_pins(sc["pins"])
    return m


@pytest.mark.parametrize("sc", _scenarios(), ids=lambda s: s["name"])
def test_slot_policy_matches_reference_trace(sc):
    m = model_for(sc)
    assert m.protected_cap == sc["protected_cap"]
    payload = [-1] * m.num_slots
    for s in range(m.num_slots):
        if m.expert_in_slot[s] >= 0:
            payload[s] = m.expert_in_slot[s]
    for i, (ids, exp) in enumerate(zip(sc["steps"], sc["trace"])):
        if i == sc["overflow_step"]:
            with pytest.raises(SlotOverflow) as ei:
                m.gap(ids)
            for loc, slot in ei.value.fills:
                payload[slot] = loc
        else:
            for loc, slot in m.gap(ids):
                payload[slot] = loc
        assert m.expert_map == exp["expert_map"], (sc["name"], i)
        assert m.expert_in_slot == exp["expert_in_slot"], (sc["name"], i)
        assert m.segment_order(PROTECTED) == exp["protected"], (sc["name"], i)
        assert m.segment_order(PROBATION) == exp["probation"], (sc["name"], i)
        assert m.map_is_standing == exp["map_is_standing"]
        assert (m.gaps, m.misses, m.fast_hits) == (exp["gaps"], exp["misses"],
                                                    exp["fast_hits"])
        live = [payload[s] if m.expert_in_slot[s] >= 0 else -1
                for s in range(m.num_slots)]
        assert live == exp["slot_payload"], (sc["name"], i)
        if sc.get("lfu"):
            assert m.freq == exp["freq"], (sc["name"], i)


def test_golden_covers_edge_cases():
    names = {s["name"]: s for s in _scenarios()}
    assert names["overflow_s40"]["overflow_step"] >= 1
    assert names["prefill_resident"]["prefill_resident"]
    assert names["v2lite_pins"]["pinned_slots"]
    aging = names["v2lite_lfu_aging"]
    assert aging["lfu"] and len(aging["trace"]) > 256  # crosses one halving
    assert any(g < 0 or g >= 64 for st in names["v2lite_invalid_ids"]["steps"] for g in st)
    assert names["ep_rank1_of2"]["local_n"] < names["ep_rank1_of2"]["global_n"]


def _wave_scenarios():
    with open(os.path.join(GOLDEN, "wave_traces.json")) as f:
        return json.load(f)["scenarios"]


def replay_wave_step(m: SlotPolicyModel, step: dict):
    """One step of a wave trace through the oracle: the gap, or the classic
    hook's wave planning. Returns the waves (gap steps: None)."""
    if step["kind"] == "gap":
        try:
            m.gap(step["ids"])
        except SlotOverflow:
            pass
        return None
    return m.run_moe(step["ids"], step["topk"], step_signal(step))


def step_signal(step: dict):
    """An MLA decode count, or the non-MLA classifier's decode rows (None:
    metadata that does not describe the batch, i.e. the heuristic)."""
    if "decode_rows" in step:
        return step["decode_rows"]
    rows = step["decode_row_index"]
    return 0 if rows is None else rows


@pytest.mark.parametrize("sc", _wave_scenarios(), ids=lambda s: s["name"])
def test_wave_planning_matches_reference_run_moe(sc):
    """Steps beyond the envelope: the oracle's run_moe / _run_waves restatement
    against the reference's own classic hook (waves, fills, final state)."""
    sc = dict(sc, prefill_resident=False)
    m = model_for(sc)
    assert m.protected_cap == sc["protected_cap"]
    n_pinned = len(sc["pinned_slots"])
    # the product's wave-buffer bound and ping-pong claim hold on the
    # reference's own plans
    bound = max_waves_for(m.num_slots, m.local_n, m.protected_cap, n_pinned)
    pipelined = waves_pingpong(m.num_slots, m.protected_cap, n_pinned)
    for i, exp in enumerate(sc["trace"]):
        waves = replay_wave_step(m, exp)
        where = (sc["name"], i)
        if waves is not None:
            got = [{"map": [list(x) for x in w["map"]], "fills": [list(x) for x in w["fills"]]}
                   for w in waves]
            assert got == exp["waves"], where
            assert len(waves) <= bound, where
            # the per-step bound the host issues: at most min(L, pairs) experts
            T = len(exp["ids"]) // exp["topk"]
            step_bound = max_waves_for(m.num_slots, min(m.local_n, len(exp["ids"])),
                                       m.protected_cap, n_pinned,
                                       all_decode=exp.get("decode_rows") == T)
            assert len(waves) <= step_bound <= bound, where
            if len(waves) > 2 and pipelined:
                # ping-pong: consecutive waves use disjoint slots
                for a, b in zip(waves[1:], waves[2:]):
                    assert not {s for _, s in a["fills"]} & {s for _, s in b["fills"]}, where
        assert m.expert_map == exp["expert_map"], where
        assert m.expert_in_slot == exp["expert_in_slot"], where
        assert m.segment_order(PROTECTED) == exp["protected"], where
        assert m.segment_order(PROBATION) == exp["probation"], where
        assert m.map_is_standing == exp["map_is_standing"], where
        assert (m.gaps, m.misses, m.fast_hits) == (exp["gaps"], exp["misses"],
                                                    exp["fast_hits"]), where
        assert (m.scan_steps, m.scan_hits, m.scan_misses, m.scan_waves) == (
            exp["scan_steps"], exp["scan_hits"], exp["scan_misses"], exp["scan_waves"]), where
        if sc["lfu"]:
            assert m.freq == exp["freq"], where


@pytest.mark.parametrize("sc", [s for s in _wave_scenarios() if s["name"].startswith("nonmla")],
                         ids=lambda s: s["name"])
def test_decode_rows_anywhere_plan_as_a_prefix(sc):
    """The product plans the non-MLA classifier's scattered decode rows by
    handing the planner the ids with those rows first and their count
    (``plan_ids_for``); through the prefix semantics the device planner
    implements, that reproduces the reference's row-index classification."""
    sc = dict(sc, prefill_resident=False)
    m = model_for(sc)
    for i, step in enumerate(sc["trace"]):
        if step["kind"] == "gap":
            replay_wave_step(m, step)
        else:
            k = step["topk"]
            t = torch.tensor(step["ids"], dtype=torch.int32).view(-1, k)
            sig = step_signal(step)
            ids, d = plan_ids_for(t, sig if isinstance(sig, int) else torch.tensor(sig))
            assert isinstance(d, int)
            waves = m.run_moe(ids.flatten().tolist(), k, d)
            got = [{"map": [list(x) for x in w["map"]], "fills": [list(x) for x in w["fills"]]}
                   for w in waves]
            assert got == step["waves"], (sc["name"], i)
        assert m.expert_map == step["expert_map"], (sc["name"], i)
        assert m.segment_order(PROTECTED) == step["protected"], (sc["name"], i)
        assert m.segment_order(PROBATION) == step["probation"], (sc["name"], i)


def test_wave_golden_covers_edge_cases():
    names = {s["name"]: s for s in _wave_scenarios()}
    nw = lambda n: [len(r["waves"]) for r in names[n]["trace"] if r["kind"] == "moe"]
    assert max(nw("s8_frac09_one_slot_rotation")) > 8        # one-slot groups, not ping-pong
    assert not waves_pingpong(8, names["s8_frac09_one_slot_rotation"]["protected_cap"], 0)
    assert max(nw("v2lite_mixed")) >= 3 and max(nw("qwen3_s64_mixed")) >= 5
    assert nw("no_owned_ids") == [1]
    assert names["v2lite_pins_prefill"]["pinned_slots"] and names["v2lite_lfu_mixed"]["lfu"]
    assert {r.get("decode_rows") for r in names["v2lite_mixed_decode_rows"]["trace"]} >= {
        4, 16, -1}
    rows = [r["decode_row_index"] for r in names["nonmla_scattered_decode_rows"]["trace"]
            if "decode_row_index" in r]
    # a None step, a pure prefill, and decode rows that are not a prefix
    assert None in rows and [] in rows
    assert any(r and r != list(range(len(r))) for r in rows if r is not None)


def _routing_case(z, name):
    meta = z[f"{name}_meta"]
    T, H, E, k, renorm, G, TG, sig = (int(v) for v in meta)
    logits = torch.from_numpy(z[f"{name}_logits"]).view(torch.bfloat16)
    sb = torch.from_numpy(z[f"{name}_score_bias"]) if f"{name}_score_bias" in z else None
    scale = float(z[f"{name}_scale"][0])
    return logits, k, bool(renorm), G, TG, "sigmoid" if sig else "softmax", scale, sb


@pytest.mark.parametrize("name", ["v2lite", "qwen3", "v3"])
def test_routing_matches_vllm_grouped_topk(name):
    z = np.load(os.path.join(GOLDEN, "routing.npz"))
    logits, k, renorm, G, TG, sf, scale, sb = _routing_case(z, name)
    w, ids = orouting.grouped_topk(logits, k, renorm, G, TG, sf, scale, sb)
    ref_ids = torch.from_numpy(z[f"{name}_ids"])
    ref_w = torch.from_numpy(z[f"{name}_weights"])
    g = logits.float()
    sel = torch.softmax(g, -1) if sf == "softmax" else g.sigmoid()
    if sb is not None:
        sel = sel + sb.unsqueeze(0)
    ties = 0
    for t in range(ids.shape[0]):
        got = dict(zip(ids[t].tolist(), w[t].tolist()))
        exp = dict(zip(ref_ids[t].tolist(), ref_w[t].tolist()))
        if set(got) != set(exp):
            # only an exact tie on the k-th selection score may differ; the
            # reference's torch.topk leaves that choice unspecified
            kth = min(sel[t, e].item() for e in got)
            for e in set(got) ^ set(exp):
                assert sel[t, e].item() == kth, (name, t, e)
            ties += 1
            continue
        for e in exp:
            # renormalisation sums k fp32 values; the reference sums them in
            # torch.topk's unspecified order, so allow a few ulp
            assert got[e] == pytest.approx(exp[e], rel=1e-6, abs=0), (name, t, e)
    assert ties <= 2, ties
    # canonical order: weights (selection scores) non-increasing per token
    if sb is None:
        assert bool((w[:, :-1] >= w[:, 1:]).all())


def test_softmax_topk_equals_grouped_single_group():
    z = np.load(os.path.join(GOLDEN, "routing.npz"))
    logits, k, renorm, *_ = _routing_case(z, "qwen3")
    w1, i1 = orouting.softmax_topk(logits, k, renorm)
    w2, i2 = orouting.grouped_topk(logits, k, renorm)
    assert torch.equal(i1, i2) and torch.equal(w1, w2)


def test_moe_matches_vllm_cpu_fused_moe():
    z = np.load(os.path.join(GOLDEN, "moe.npz"))
    bf = lambda a: torch.from_numpy(a).view(torch.bfloat16)
    out = omoe.fused_experts(bf(z["hs"]), bf(z["w13"]), bf(z["w2"]),
                             torch.from_numpy(z["topk_weights"]),
                             torch.from_numpy(z["topk_ids"]),
                             torch.from_numpy(z["expert_map"]))
    assert torch.equal(out.view(torch.int16), torch.from_numpy(z["out"]))


def test_split_shared_is_the_same_mlp():
    g = torch.Generator().manual_seed(3)
    n, I, H = 2, 64, 32
    w13 = torch.randn(2 * n * I, H, generator=g, dtype=torch.float64)
    w2 = torch.randn(H, n * I, generator=g, dtype=torch.float64)
    x = torch.randn(5, H, generator=g, dtype=torch.float64)
    whole = omoe.expert_mlp(x, w13, w2)
    s13, s2 = omoe.split_shared(w13, w2, n)
    parts = sum(omoe.expert_mlp(x, s13[i], s2[i]) for i in range(n))
    assert torch.allclose(whole, parts, atol=1e-9)


def test_fp8_dequant_block_scale():
    w = torch.randn(256, 384).to(torch.float8_e4m3fn)
    s = torch.rand(2, 3) + 0.5
    d = omoe.dequant_block_fp8(w, s)
    assert torch.equal(d[:128, :128], w[:128, :128].float() * s[0, 0])
    assert torch.equal(d[128:, 256:], w[128:, 256:].float() * s[1, 2])


def test_fp8_group_quant_matches_vllm():
    """The oracle's per-token-group e4m3 quantisation against vLLM's own
    (torch-native twin of its CUDA op): scales agree to one fp32 ulp (vLLM
    divides amax by 448, the Triton path and this oracle multiply by 1/448),
    and the e4m3 codes agree except where that ulp moves a value across a
    rounding boundary."""
    z = np.load(os.path.join(GOLDEN, "fp8_quant.npz"))
    x = torch.from_numpy(z["x"]).to(torch.bfloat16)
    q, scale = omoe.quant_group_fp8(x)
    ref_s = torch.from_numpy(z["scale"])
    assert ((scale - ref_s).abs() / ref_s).max().item() <= 2.4e-7
    ref_q = torch.from_numpy(z["q"]).view(torch.float8_e4m3fn).float()
    flips = (q.float() != ref_q)
    assert flips.float().mean().item() < 5e-3
    # a flip is one e4m3 step: at most 1/8 relative to the larger neighbour
    d = (q.float() - ref_q).abs()[flips]
    m = torch.maximum(q.float().abs(), ref_q.abs())[flips]
    assert (d <= m / 8 + 1e-6).all()
