"""GPU parity of steps beyond the envelope (expert waves): the device wave
planner against the reference's own classic hook (``run_moe`` /
``_run_waves`` traces: every wave's map and fills, the state after the step,
the streamed slot contents), and whole layers stepped in waves against the
oracle (bf16 and fp8 experts, CUDA-graph replay)."""

import json
import os
from dataclasses import replace

import pytest
import torch

from oracle import moe as omoe
from oracle import routing as orouting
from oracle.slot_policy import SlotPolicyModel
from sluice_b200 import _lib, configs, ops, synth
from sluice_b200.layer import MoEDecodeStack, SluiceMoELayer
from sluice_b200.offloader import ExpertStreamOffloader
from test_moe_gpu import assert_moe_close
from test_slots_gpu import _payload_params

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _wave_scenarios():
    with open(os.path.join(GOLDEN, "wave_traces.json")) as f:
        return json.load(f)["scenarios"]


def _install(sc):
    off = ExpertStreamOffloader(sc["num_slots"], protect_frac=sc["protect_frac"],
                                fast_hit=sc["fast_hit"], lfu=sc["lfu"])
    w13, w2 = _payload_params(sc["local_n"])
    return off.install_layer(w13, w2, global_n=sc["global_n"], local_of=sc["local_of"],
                             pins=sc["pins"], device="cuda")


def _slot_payload(cache):
    return (cache.w13[:, 0, 0].float().cpu().tolist(),
            cache.w2[:, 0, 0].float().cpu().tolist())


@pytest.mark.parametrize("sc", _wave_scenarios(), ids=lambda s: s["name"])
def test_wave_planner_matches_reference_run_moe(sc):
    cache = _install(sc)
    assert cache.protected_cap == sc["protected_cap"]
    for i, exp in enumerate(sc["trace"]):
        where = (sc["name"], i)
        ids = torch.tensor(exp["ids"], dtype=torch.int32, device="cuda")
        if exp["kind"] == "gap":
            cache.gap(ids)
            torch.cuda.synchronize()
        else:
            if "decode_rows" in exp:
                signal = exp["decode_rows"]
            else:  # the non-MLA classifier's decode rows (None: heuristic)
                rows = exp["decode_row_index"]
                signal = 0 if rows is None else torch.tensor(rows, dtype=torch.long)
            cache.plan_waves(ids.view(-1, exp["topk"]), signal)
            torch.cuda.synchronize()
            assert cache.wave_header()["status"] == _lib.SL_OK, where
            plan = cache.wave_plan()
            assert len(plan) == len(exp["waves"]) <= cache.max_waves, where
            for k, (got, want) in enumerate(zip(plan, exp["waves"])):
                assert sorted(got["map"]) == sorted(tuple(x) for x in want["map"]), (where, k)
                assert got["fills"] == [tuple(x) for x in want["fills"]], (where, k)
                # stream this wave alone: its slots now hold its experts
                cache.stream_wave(k)
                torch.cuda.synchronize()
                w13, w2 = _slot_payload(cache)
                for loc, slot in got["fills"]:
                    assert w13[slot] == loc and w2[slot] == -loc - 1, (where, k, slot)
            if len(plan) < cache.max_waves:
                cache.stream_wave(cache.max_waves - 1)  # past the count: nothing
        snap = cache.snapshot()
        assert snap["header"]["status"] == _lib.SL_OK, where
        assert snap["expert_map"] == exp["expert_map"], where
        assert snap["expert_in_slot"] == exp["expert_in_slot"], where
        assert snap["protected"] == exp["protected"], where
        assert snap["probation"] == exp["probation"], where
        assert bool(snap["header"]["map_is_standing"]) == exp["map_is_standing"], where
        c = snap["counters"]
        assert (c["gaps"], c["misses"], c["fast_hits"]) == (
            exp["gaps"], exp["misses"], exp["fast_hits"]), where
        assert (c["scan_steps"], c["scan_hits"], c["scan_misses"], c["waves"]) == (
            exp["scan_steps"], exp["scan_hits"], exp["scan_misses"], exp["scan_waves"]), where
        w13, w2 = _slot_payload(cache)
        for s, loc in enumerate(exp["slot_payload"]):
            if loc >= 0:
                assert w13[s] == loc and w2[s] == -loc - 1, (where, s)
        if sc["lfu"]:
            assert snap["freq"] == exp["freq"], where


def _layer(cfg, slots, seed, fp8=False, beyond="waves", zipf_bias=0.0):
    """A layer whose router has no popularity skew by default, so prefill
    working sets exceed the slots and steps spill into several waves."""
    w13, w2 = synth.layer_weights(cfg, 0, seed=seed, device="cuda")
    gw, lb, sb = synth.gate_params(cfg, 0, seed=seed, device="cuda", zipf_bias=zipf_bias)
    sh13, sh2 = synth.shared_weights(cfg, 0, seed=seed, device="cuda")
    off = ExpertStreamOffloader(slots, protect_frac=0.5, fast_hit=True)
    kw, host = {}, {"w13": w13.cpu(), "w2": w2.cpu(), "sh13": sh13, "sh2": sh2}
    if fp8:
        q13, s13 = synth.quantize_block_fp8(w13)
        q2, s2 = synth.quantize_block_fp8(w2)
        qs13, ss13 = synth.quantize_block_fp8(sh13)
        qs2, ss2 = synth.quantize_block_fp8(sh2)
        cache = off.install_layer(q13, q2, device="cuda", w13_scale=s13, w2_scale=s2)
        kw = dict(shared_w13_scale=ss13, shared_w2_scale=ss2)
        host = {"w13": q13.cpu(), "w2": q2.cpu(), "s13": s13.cpu(), "s2": s2.cpu(),
                "sh13": qs13, "sh2": qs2, "ss13": ss13, "ss2": ss2}
        sh13, sh2 = qs13, qs2
    else:
        cache = off.install_layer(w13, w2, device="cuda")
    layer = SluiceMoELayer(cfg, ops.Router(cfg.routing, gw, lb, sb), cache, sh13, sh2,
                           beyond_envelope=beyond, **kw)
    return layer, cache, host, sb


def _reference(cfg, layer, x, host, sb, fp8):
    """The oracle's layer output on the kernel's own bf16 logits; every
    (token, expert) pair counts once, whatever wave computed it."""
    rc = cfg.routing
    logits = layer.last_logits.cpu()
    ow, oi = orouting.grouped_topk(logits, rc.topk, rc.renormalize, rc.num_expert_group,
                                   rc.topk_group, rc.scoring_func, 1.0,
                                   None if sb is None else sb.cpu())
    ti = layer.last_ids.cpu()
    for t in range(ti.shape[0]):
        assert set(ti[t].tolist()) == set(oi[t].tolist()), t
    wmap = [dict(zip(oi[t].tolist(), ow[t].tolist())) for t in range(ti.shape[0])]
    tw = torch.tensor([[wmap[t][e] for e in ti[t].tolist()] for t in range(ti.shape[0])])
    if fp8:
        routed = omoe.fused_experts(x, host["w13"], host["w2"], tw, ti, None, host["s13"],
                                    host["s2"])
        shared = omoe.shared_experts(x, host["sh13"][0].cpu(), host["sh2"][0].cpu(),
                                     host["ss13"][0].cpu(), host["ss2"][0].cpu())
    else:
        routed = omoe.fused_experts(x, host["w13"], host["w2"], tw, ti)
        sh13, sh2 = host["sh13"], host["sh2"]
        shared = None if sh13 is None else sum(
            omoe.expert_mlp(x, sh13[i].cpu(), sh2[i].cpu()).float()
            for i in range(sh13.shape[0])).to(torch.bfloat16)
    return omoe.layer_output(routed, shared, cfg.routed_scaling_factor), ti


def test_v2lite_layer_in_waves_matches_oracle():
    """V2-Lite, 48 slots (envelope 8 tokens): prefill-sized steps (ws
    heuristic, decode rows, forced scan) interleaved with decode steps; slot
    state after every step against the oracle, outputs within tolerance."""
    cfg = configs.V2_LITE
    layer, cache, host, sb = _layer(cfg, 48, seed=21)
    model = SlotPolicyModel(48, list(range(cfg.num_experts)), cfg.num_experts, 0.5, True)
    g = torch.Generator().manual_seed(22)
    # (tokens, decode signal): heuristic, decode steps, decode-row prefix,
    # forced scan, and all-decode steps (the tighter wave count)
    plan = [(64, 0), (8, None), (40, 4), (8, None), (8, None), (29, -1), (96, 0), (8, None),
            (48, 48), (8, None), (64, 64)]
    nwaves = []
    for step, (T, d) in enumerate(plan):
        x = torch.randn(T, cfg.hidden, generator=g).to(torch.bfloat16)
        out = layer(x.cuda(), decode_rows=d or 0)
        torch.cuda.synchronize()
        cache.check()
        ref, ti = _reference(cfg, layer, x, host, sb, False)
        if d is None:
            model.gap(ti.flatten().tolist())
        else:
            nwaves.append(len(model.run_moe(ti.flatten().tolist(), cfg.routing.topk, d)))
            assert cache.wave_header()["num_waves"] == nwaves[-1], step
        assert cache.expert_map.cpu().tolist() == model.expert_map, step
        assert cache.snapshot()["expert_in_slot"] == model.expert_in_slot, step
        assert_moe_close(out, ref)
    assert max(nwaves) >= 2  # the steps really ran in several waves
    c = cache.counters()
    assert c["waves"] == model.scan_waves and c["scan_misses"] == model.scan_misses


def test_fp8_v3_style_layer_in_waves_matches_oracle():
    """fp8 e4m3 experts with 128x128 block scales (weights and scales stream
    wave by wave), V3 routing, 16 slots: 24 tokens x top-8 is 3 envelopes."""
    cfg = replace(configs.DEEPSEEK_V3, hidden=1024, num_experts=32, moe_intermediate=512,
                  num_moe_layers=1)
    layer, cache, host, sb = _layer(cfg, 16, seed=23, fp8=True)
    assert layer.envelope == 2
    g = torch.Generator().manual_seed(24)
    for step, T in enumerate([24, 2, 12, 24]):
        x = torch.randn(T, cfg.hidden, generator=g).to(torch.bfloat16)
        out = layer(x.cuda())
        torch.cuda.synchronize()
        cache.check()
        ref, _ = _reference(cfg, layer, x, host, sb, True)
        assert_moe_close(out, ref, rtol=5e-2)
    assert cache.counters()["waves"] >= 4


def test_waves_and_chunks_agree():
    """The same prefill step through waves and through envelope chunks gives
    the same output within bf16 tolerance (both are the full MoE)."""
    cfg = configs.QWEN3_30B_A3B
    a, _, _, _ = _layer(cfg, 64, seed=25)
    b, _, _, _ = _layer(cfg, 64, seed=25, beyond="chunks")
    x = torch.randn(48, cfg.hidden, generator=torch.Generator().manual_seed(26))
    x = x.to(torch.bfloat16).cuda()
    oa, ob = a(x), b(x)
    torch.cuda.synchronize()
    a.cache.check()
    b.cache.check()
    assert a.cache.wave_header()["num_waves"] >= 2
    assert_moe_close(oa, ob)
    # waves stream each missing expert once; chunks re-stream across chunks
    assert a.cache.stats()["fills"] < b.cache.stats()["fills"]


def test_wave_step_graph_replay_equals_eager():
    """A step beyond the envelope captures in a CUDA graph (fixed wave count,
    empty waves exit on the device) and replays bit-identically."""
    cfg = configs.V2_LITE
    a = MoEDecodeStack(cfg, slots=48, seed=27, num_layers=2)
    b = MoEDecodeStack(cfg, slots=48, seed=27, num_layers=2)
    b.capture(tokens=24)
    a.step(torch.zeros(24, cfg.hidden, dtype=torch.bfloat16, device="cuda"))
    stream = synth.TokenStream(cfg.hidden, 24, seed=28)
    for _ in range(3):
        x = stream.next().cuda()
        ea = a.step(x)
        eb = b.replay(x)
        torch.cuda.synchronize()
        assert torch.equal(ea, eb)
    a.check()
    b.check()
    assert a.stats() == b.stats() and a.stats()["waves"] >= 6
