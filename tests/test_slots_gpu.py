"""GPU parity: the device slot planner and streamer vs the reference's own
gap traces (bit-exact expert map, slot owners, SLRU order, counters, and the
streamed slot contents)."""

import json
import os

import pytest
import torch

from oracle.slot_policy import PROBATION, PROTECTED, SlotOverflow, SlotPolicyModel
from sluice_b200 import _lib
from sluice_b200.offloader import ExpertStreamOffloader

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _scenarios():
    with open(os.path.join(GOLDEN, "slot_traces.json")) as f:
        return json.load(f)["scenarios"]


def _payload_params(local_n):
    """Tiny per-expert params whose elements encode the local expert id
    (exact in bf16 for ids below 256)."""
    assert local_n <= 255
    ids = torch.arange(local_n, dtype=torch.float32)
    w13 = ids.view(-1, 1, 1).expand(local_n, 2, 8).to(torch.bfloat16).contiguous()
    w2 = (-ids - 1).view(-1, 1, 1).expand(local_n, 8, 1).to(torch.bfloat16).contiguous()
    return w13, w2


def _install(sc, pin_file=None, packed=False):
    off = ExpertStreamOffloader(sc["num_slots"], protect_frac=sc["protect_frac"],
                                fast_hit=sc["fast_hit"],
                                no_static_full=sc["prefill_resident"],
                                lfu=sc.get("lfu", False), pin_file=pin_file,
                                packed_host_store=packed)
    w13, w2 = _payload_params(sc["local_n"])
    return off.install_layer(w13, w2, global_n=sc["global_n"], local_of=sc["local_of"],
                             pins=None if pin_file else sc["pins"], device="cuda")


def _pin_file_cases():
    """Scenarios with pins, replayed with the pins given as a SLUICE_PIN_FILE."""
    return [s for s in _scenarios() if s["pins"]]


@pytest.mark.parametrize("sc", _scenarios(), ids=lambda s: s["name"])
def test_planner_matches_reference_trace(sc):
    _check_trace(sc, _install(sc))


@pytest.mark.parametrize("sc", _pin_file_cases(), ids=lambda s: s["name"])
def test_pin_file_matches_reference_trace(sc, tmp_path):
    path = tmp_path / "pins.json"
    path.write_text(json.dumps({"layers": {"0": sc["pins"]}}))
    _check_trace(sc, _install(sc, pin_file=str(path)))


@pytest.mark.parametrize("name", ["v2lite_zipf_fasthit", "v3_ep4_rank2"])
def test_packed_host_store_streams_the_same_contents(name):
    """One host record per expert ([w13 | w2]) instead of one host array per
    parameter: same plan, same slot contents after every streamed fill."""
    sc = next(s for s in _scenarios() if s["name"] == name)
    _check_trace(sc, _install(sc, packed=True))


def _check_trace(sc, cache):
    assert cache.protected_cap == sc["protected_cap"]
    for i, (ids, exp) in enumerate(zip(sc["steps"], sc["trace"])):
        t = torch.tensor(ids, dtype=torch.int32, device="cuda")
        cache.gap(t)
        snap = cache.snapshot()
        status = snap["header"]["status"]
        if i == sc["overflow_step"]:
            assert status == _lib.SL_ERR_OVERFLOW
            with pytest.raises(_lib.SluiceError):
                cache.check()
        else:
            assert status == _lib.SL_OK, (sc["name"], i)
        assert snap["expert_map"] == exp["expert_map"], (sc["name"], i)
        assert snap["expert_in_slot"] == exp["expert_in_slot"], (sc["name"], i)
        assert snap["protected"] == exp["protected"], (sc["name"], i)
        assert snap["probation"] == exp["probation"], (sc["name"], i)
        assert bool(snap["header"]["map_is_standing"]) == exp["map_is_standing"]
        c = snap["counters"]
        assert (c["gaps"], c["misses"], c["fast_hits"]) == (exp["gaps"], exp["misses"],
                                                            exp["fast_hits"]), (sc["name"], i)
        # streamed contents: every occupied slot holds its expert's bytes
        w13 = cache.w13[:, 0, 0].float().cpu().tolist()
        w2 = cache.w2[:, 0, 0].float().cpu().tolist()
        for s, loc in enumerate(exp["slot_payload"]):
            if loc >= 0:
                assert w13[s] == loc and w2[s] == -loc - 1, (sc["name"], i, s)
        if sc.get("lfu"):
            assert snap["freq"] == exp["freq"], (sc["name"], i)


def test_planner_long_random_run_matches_oracle():
    """A long run past many evictions, FAST_HIT on, against the oracle."""
    g = torch.Generator().manual_seed(5)
    S, E, T, k = 40, 96, 6, 6
    sc = {"num_slots": S, "protect_frac": 0.5, "fast_hit": True, "prefill_resident": False,
          "local_n": E, "global_n": E, "local_of": list(range(E)), "pins": None}
    cache = _install(sc)
    m = SlotPolicyModel(S, list(range(E)), E, 0.5, True)
    hot = torch.randperm(E, generator=g)[:30]
    for step in range(300):
        if step % 3 == 0:
            ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)])
        else:
            ids = hot[torch.stack([torch.randperm(30, generator=g)[:k] for _ in range(T)])]
        ids = ids.to(torch.int32)
        cache.gap(ids.cuda())
        m.gap(ids.flatten().tolist())
        if step % 25 == 0 or step == 299:
            snap = cache.snapshot()
            assert snap["expert_map"] == m.expert_map, step
            assert snap["protected"] == m.segment_order(PROTECTED), step
            assert snap["probation"] == m.segment_order(PROBATION), step
    c = cache.counters()
    assert (c["gaps"], c["misses"], c["fast_hits"]) == (m.gaps, m.misses, m.fast_hits)


def test_clock_renumbering_keeps_lru_order():
    """Force the stamp clock near its limit; the order must survive renumbering."""
    S, E = 16, 32
    sc = {"num_slots": S, "protect_frac": 0.5, "fast_hit": False, "prefill_resident": False,
          "local_n": E, "global_n": E, "local_of": list(range(E)), "pins": None}
    cache = _install(sc)
    m = SlotPolicyModel(S, list(range(E)), E, 0.5, False)
    g = torch.Generator().manual_seed(9)
    for step in range(60):
        ids = torch.randperm(E, generator=g)[:10].to(torch.int32)
        if step == 20:
            # push every live stamp and the clock close to 2^31
            off = cache.offsets
            hdr = cache.state[off[0]:off[0] + 64].view(torch.int32)
            st = cache.state[off[7]:off[7] + 4 * S].view(torch.int32)
            live = st > 0
            st[live] += 0x7FFF0000 - 64
            hdr[_lib.HDR["clock"]] += 0x7FFF0000 - 64
        cache.gap(ids.cuda())
        m.gap(ids.tolist())
        snap = cache.snapshot()
        assert snap["protected"] == m.segment_order(PROTECTED), step
        assert snap["probation"] == m.segment_order(PROBATION), step
        assert snap["expert_map"] == m.expert_map, step
    assert cache.header()["clock"] < 0x7FFF0000


def test_gap_op_is_registered_and_returns_a_clone():
    from sluice_b200 import ops
    sc = {"num_slots": 8, "protect_frac": 0.5, "fast_hit": True, "prefill_resident": False,
          "local_n": 16, "global_n": 16, "local_of": list(range(16)), "pins": None}
    cache = _install(sc)
    idx = ops.register_gap_layer(cache)
    hs = torch.randn(2, 64, device="cuda").to(torch.bfloat16)
    ids = torch.tensor([[1, 2], [3, 1]], dtype=torch.int32, device="cuda")
    out = torch.ops.sluice.sluice_stream_gap(hs, ids, idx)
    assert torch.equal(out, hs) and out.data_ptr() != hs.data_ptr()
    m = cache.expert_map.cpu().tolist()
    assert m[1] >= 0 and m[2] >= 0 and m[3] >= 0 and sum(v >= 0 for v in m) == 3


def test_empty_step_changes_nothing_but_the_gap_count():
    """A gap over zero ids (an empty decode batch) touches no slot."""
    sc = {"num_slots": 8, "protect_frac": 0.5, "fast_hit": True, "prefill_resident": False,
          "local_n": 16, "global_n": 16, "local_of": list(range(16)), "pins": None}
    cache = _install(sc)
    m = SlotPolicyModel(8, list(range(16)), 16, 0.5, True)
    for ids in ([1, 2, 3], [], [4, 1], [], []):
        cache.gap(torch.tensor(ids, dtype=torch.int32, device="cuda"))
        m.gap(ids)
        snap = cache.snapshot()
        assert snap["expert_map"] == m.expert_map
        assert snap["protected"] == m.segment_order(PROTECTED)
        assert snap["probation"] == m.segment_order(PROBATION)
        c = snap["counters"]
        assert (c["gaps"], c["misses"], c["fast_hits"]) == (m.gaps, m.misses, m.fast_hits)
