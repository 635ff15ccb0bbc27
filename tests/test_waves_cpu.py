"""CPU properties of expert-wave planning, over many random caches and step
mixes (the oracle's restatement of the reference's run_moe / _run_waves,
itself pinned to the reference's traces in test_oracle_golden.py):

* the waves partition the step's owned selected experts: every one is
  computed by exactly one wave, so the waves' outputs sum to the step's;
* every wave after the first streams exactly the experts it maps;
* the host's per-step wave count (``SlotCache.waves_for``'s bound) is never
  short, so the fixed number of waves a captured step issues covers it;
* the stream ordering the host uses is safe: with ping-pong groups, wave k's
  fills touch no slot that wave k - 1 reads, and wave 1 and 2's fills only
  reuse slots after wave 0 (the host makes them wait for wave 0's GEMMs).
"""

import random

import pytest

from oracle.slot_policy import PINNED, PROTECTED, SlotOverflow, SlotPolicyModel
from sluice_b200.offloader import max_waves_for, waves_pingpong


def _random_cache(rng: random.Random):
    S = rng.randint(2, 48)
    L = rng.randint(S + 1, 96)
    owned_lo = rng.choice([0, 0, rng.randint(0, 64)])
    G = max(L + owned_lo, L + rng.choice([0, 0, 32]))
    local_of = [-1] * G
    for i in range(L):
        local_of[owned_lo + i] = i
    m = SlotPolicyModel(S, local_of, L, protect_frac=rng.choice([0.0, 0.3, 0.5, 0.9]),
                        fast_hit=rng.random() < 0.7, lfu=rng.random() < 0.3)
    if rng.random() < 0.3:
        m.apply_pins([rng.randrange(G) for _ in range(rng.randint(1, 6))])
    return m, G


def _ids(rng, T, k, G, lo, hi):
    """T tokens x k distinct ids (an occasional invalid id, as routers emit
    none but the op accepts them)."""
    out = []
    for _ in range(T):
        row = rng.sample(range(lo, hi), min(k, hi - lo))
        row += [rng.randrange(G)] * (k - len(row))
        if rng.random() < 0.05:
            row[0] = rng.choice([-1, G + 3])
        out += row
    return out


@pytest.mark.parametrize("seed", range(12))
def test_wave_plans_partition_and_fit_the_bound(seed):
    rng = random.Random(1000 + seed)
    for _case in range(25):
        m, G = _random_cache(rng)
        n_pinned = sum(1 for v in m.seg if v == PINNED)
        pingpong = waves_pingpong(m.num_slots, m.protected_cap, n_pinned)
        for _step in range(rng.randint(4, 12)):
            k = rng.randint(1, 8)
            # a popular subset some steps, the whole id space others
            lo, hi = (0, G) if rng.random() < 0.5 else (0, max(k, G // 3))
            if rng.random() < 0.4:
                T = rng.randint(1, max(1, m.num_slots // k))
                try:
                    m.gap(_ids(rng, T, k, G, lo, hi))
                except SlotOverflow:
                    pass  # pins can leave fewer usable slots than the envelope
                continue
            T = rng.randint(1, 64)
            ids = _ids(rng, T, k, G, lo, hi)
            d = rng.choice([-1, 0, 0, rng.randint(1, T), T, T])
            waves = m.run_moe(ids, k, d)
            owned = {g for g in ids if 0 <= g < G and m.local_of[g] >= 0}
            # partition: every owned selected expert in exactly one wave
            seen = [g for w in waves for g, _ in w["map"]]
            assert sorted(seen) == sorted(owned)
            for w in waves:
                slots = [s for _, s in w["map"]]
                assert len(slots) == len(set(slots))
            for w in waves[1:]:
                assert sorted(g for g, _ in w["map"]) == sorted(
                    m.global_of_local[loc] for loc, _ in w["fills"])
                assert all(s for s in w["fills"])
            # the host's per-step wave count covers the plan (tighter when
            # every row is a decode: every expert decode-class)
            bound = max_waves_for(m.num_slots, min(m.local_n, len(ids)), m.protected_cap,
                                  n_pinned, all_decode=(d == T))
            assert len(waves) <= bound <= max_waves_for(m.num_slots, m.local_n,
                                                        m.protected_cap, n_pinned)
            # stream ordering: wave k's fills avoid wave k - 1's slots
            if pingpong:
                for a, b in zip(waves[1:], waves[2:]):
                    assert not {s for _, s in a["map"]} & {s for _, s in b["fills"]}
            # the state stays consistent
            for s, loc in enumerate(m.expert_in_slot):
                if loc >= 0:
                    assert m.slot_of[loc] == s
            assert sum(1 for v in m.seg if v == PROTECTED) <= m.protected_cap
            assert not m.map_is_standing
            last = waves[-1]["map"]
            assert m.expert_map == [dict(last).get(g, -1) for g in range(G)]


@pytest.mark.parametrize("seed", range(6))
def test_all_decode_wave_bound_is_tight_enough(seed):
    """Decode steps beyond the envelope (every row a decode), the expert-
    parallel decode case: many random warm caches, the decode-aware bound
    never short, and reached by some step."""
    rng = random.Random(5000 + seed)
    reached = 0
    for _case in range(40):
        m, G = _random_cache(rng)
        n_pinned = sum(1 for v in m.seg if v == PINNED)
        for _step in range(rng.randint(3, 10)):
            k = rng.randint(1, 8)
            T = rng.randint(1, 48)
            lo, hi = (0, G) if rng.random() < 0.5 else (0, max(k, G // 2))
            ids = _ids(rng, T, k, G, lo, hi)
            waves = m.run_moe(ids, k, T)
            bound = max_waves_for(m.num_slots, min(m.local_n, len(ids)), m.protected_cap,
                                  n_pinned, all_decode=True)
            assert len(waves) <= bound
            reached += len(waves) == bound and bound > 1
    assert reached > 0


def test_single_rotation_group_is_not_pingpong():
    """With one probation slot the rotation has a single group: every later
    wave reuses it, so the host must order wave k's fills after wave k - 1."""
    m = SlotPolicyModel(8, list(range(32)), 32, protect_frac=0.9, fast_hit=False)
    assert not waves_pingpong(8, m.protected_cap, 0)
    m.gap(list(range(8)))      # fills every slot
    m.gap(list(range(7)))      # 7 decode hits promote (no FAST_HIT): protected is full
    assert sum(1 for v in m.seg if v == PROTECTED) == m.protected_cap == 7
    ids = list(range(8, 32))
    waves = m.run_moe(ids, 8, -1)  # a scan: misses never take protected slots
    assert len(waves) == 24 and all(len(w["fills"]) == 1 for w in waves)
    rot = {s for w in waves[1:] for _, s in w["fills"]}
    assert len(rot) == 1
    assert len(waves) <= max_waves_for(8, min(32, len(ids)), m.protected_cap, 0)
