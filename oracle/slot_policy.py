"""CPU restatement of the router-split gap's slot cache (TEST INFRASTRUCTURE).

Restates, in plain Python over small integer arrays, the per-layer expert slot
cache that kfirtoledo/sluice keeps in ``src/sluice/offloader.py``:

* state: ``_ExpertLayerCache`` (offloader.py:121-169) — slot owners, the
  free list, the protected/probation SLRU segments, the expert map;
* install: ``_install_cache`` (offloader.py:936-1007) — ``num_slots =
  min(SLUICE_SLOTS, local_n)``, ``protected_cap = min(int(slots*frac),
  slots-1)``, free list ``[slots-1, ..., 0]`` popped from the end;
* pins: ``_apply_pins`` (offloader.py:1046-1083);
* policy: ``_touch`` (2009-2021), ``_coldest_protected`` (2023-2034),
  ``_acquire_slot`` (2036-2074), ``_evict_to`` (2076-2081);
* the LFU hybrid (``SLUICE_LFU=1``): ``_bump_freq`` (1993-2007: +1 per
  selected owned expert per step, counts halved every ``LFU_AGE_STEPS`` =
  256 steps, offloader.py:118) and the frequency-ordered protected victims of
  ``_coldest_protected`` / ``_acquire_slot`` (ties in LRU order);
* maps: ``_write_map`` / ``_write_standing_map`` (2083-2123);
* the gap body: ``_router_split_gap`` (2362-2467), FAST_HIT on or off;
* steps beyond the envelope: the classic hook's planning, ``run_moe``
  (1452-1764: decode / scan classification, touches, wave 0) and
  ``_run_waves`` (1846-1933: the remaining misses rotate through the
  probation slots in ping-pong groups, one expert wave per group), with the
  reference's default switches (hook-lite, prefill blocks, lazy modes and the
  non-MLA classifier off).

Recency is kept as a per-slot stamp from one per-layer clock instead of
ordered dictionaries: a segment's LRU order is its slots sorted by stamp, and
"move to end" / "insert at end" is "take a new stamp". This is the same
representation the CUDA planner uses, so the oracle also documents it.

Under LFU the counts are bumped once per gap call, before the FAST_HIT check
(the reference bumps them in its hook for every real step, then runs the
gap's policy with them).
"""

from __future__ import annotations

FREE, PROBATION, PROTECTED, PINNED = 0, 1, 2, 3
LFU_AGE_STEPS = 256  # offloader.py:118


class SlotOverflow(RuntimeError):
    """The reference raises RuntimeError here (offloader.py:2456-2460).

    ``fills`` lists the acquisitions (and streams) done before the failure.
    """

    def __init__(self, msg: str, fills=()):
        super().__init__(msg)
        self.fills = list(fills)


def protected_cap_for(num_slots: int, protect_frac: float) -> int:
    """offloader.py:236-241 (frac clamp) and 937 (cap)."""
    frac = min(max(float(protect_frac), 0.0), 0.9)
    return max(min(int(num_slots * frac), num_slots - 1), 0)


class SlotPolicyModel:
    """One layer's slot cache, driven one gap call at a time."""

    def __init__(self, num_slots: int, local_of: list[int], local_n: int,
                 protect_frac: float = 0.5, fast_hit: bool = True,
                 bytes_per_expert: int = 0, prefill_resident: bool = False,
                 lfu: bool = False):
        self.num_slots = int(num_slots)
        self.local_of = [int(v) for v in local_of]
        self.global_n = len(self.local_of)
        self.local_n = int(local_n)
        self.protected_cap = protected_cap_for(self.num_slots, protect_frac)
        self.fast_hit = bool(fast_hit)
        self.lfu = bool(lfu)
        self.freq = [0] * int(local_n)
        self.lfu_steps = 0
        self.bytes_per_expert = int(bytes_per_expert)
        self.global_of_local = [-1] * self.local_n
        for g, loc in enumerate(self.local_of):
            if 0 <= loc < self.local_n:
                self.global_of_local[loc] = g
        S = self.num_slots
        self.expert_in_slot = [-1] * S
        self.slot_of = [-1] * self.local_n
        self.seg = [FREE] * S
        self.stamp = [0] * S
        self.clock = 0
        # popped from the end: lowest slot index first (offloader.py:944)
        self.free_stack = list(range(S - 1, -1, -1))
        self.expert_map = [-1] * self.global_n
        self.map_is_standing = False
        self.gaps = 0
        self.fast_hits = 0
        self.misses = 0
        self.bytes_streamed = 0
        self.scan_steps = 0     # classic-hook steps (run_moe) and their waves
        self.scan_hits = 0
        self.scan_misses = 0
        self.scan_waves = 0
        self.prefetches = 0     # opt-in cross-layer prefetch fills
        if prefill_resident:
            # offloader.py:992-1003: every local expert preloaded into slot ==
            # local index, outside both SLRU segments; extra slots stay free.
            for loc in range(self.local_n):
                self.slot_of[loc] = loc
                self.expert_in_slot[loc] = loc
                self.seg[loc] = PINNED
            self.free_stack = list(range(S - 1, self.local_n - 1, -1))

    # -- helpers ---------------------------------------------------------
    def _tick(self) -> int:
        self.clock += 1
        return self.clock

    def _lru(self, seg: int) -> list[int]:
        return sorted((s for s in range(self.num_slots) if self.seg[s] == seg),
                      key=lambda s: self.stamp[s])

    def segment_order(self, seg: int) -> list[int]:
        """Slots of a segment, least recently used first."""
        return self._lru(seg)

    def protected_count(self) -> int:
        return sum(1 for s in self.seg if s == PROTECTED)

    # -- pins (offloader.py:1046-1083) ------------------------------------
    def apply_pins(self, wanted: list[int]) -> list[tuple[int, int]]:
        fills = []
        budget = self.protected_cap
        n = 0
        for g in wanted:
            if n >= budget:
                break
            if not (0 <= g < self.global_n):
                continue
            loc = self.local_of[g]
            if loc < 0 or self.slot_of[loc] >= 0 or not self.free_stack:
                continue
            slot = self.free_stack.pop()
            self.expert_in_slot[slot] = loc
            self.slot_of[loc] = slot
            self.seg[slot] = PINNED
            fills.append((loc, slot))
            n += 1
        self.protected_cap -= n
        return fills

    # -- policy ------------------------------------------------------------
    def _touch(self, slot: int, friendly: bool) -> None:
        """offloader.py:2009-2021 (pinned slots are in neither segment)."""
        if self.seg[slot] == PROTECTED:
            self.stamp[slot] = self._tick()
        elif self.seg[slot] == PROBATION:
            if friendly and self.protected_cap > 0:
                self.seg[slot] = PROTECTED
                self.stamp[slot] = self._tick()
                while self.protected_count() > self.protected_cap:
                    demoted = self._coldest_protected()
                    self.seg[demoted] = PROBATION
                    self.stamp[demoted] = self._tick()
            else:
                self.stamp[slot] = self._tick()

    def _coldest_protected(self) -> int:
        """offloader.py:2023-2034: least frequently used under LFU (ties in
        LRU order), else least recently used."""
        order = self._lru(PROTECTED)
        if self.lfu:
            return min(order, key=lambda s: self.freq[self.expert_in_slot[s]])
        return order[0]

    def bump_freq(self, ids: list[int]) -> None:
        """offloader.py:1993-2007 over this step's selected owned experts."""
        for g in sorted(set(int(v) for v in ids)):
            if 0 <= g < self.global_n and self.local_of[g] >= 0:
                self.freq[self.local_of[g]] += 1
        self.lfu_steps += 1
        if self.lfu_steps >= LFU_AGE_STEPS:
            self.lfu_steps = 0
            self.freq = [f >> 1 for f in self.freq]

    def _acquire(self, loc: int, claimed: set, allow_protected: bool = True) -> int | None:
        """offloader.py:2036-2074 (the gap calls it with allow_protected=True;
        the classic hook passes the miss's decode class)."""
        slot = None
        if self.free_stack:
            slot = self.free_stack.pop()
        else:
            for cand in self._lru(PROBATION):
                if cand not in claimed:
                    slot = cand
                    break
            if slot is None and allow_protected:
                order = self._lru(PROTECTED)
                if self.lfu:  # coldest first, LRU order among equals
                    order = sorted(order, key=lambda s: self.freq[self.expert_in_slot[s]])
                for cand in order:
                    if cand not in claimed:
                        slot = cand
                        break
        if slot is None:
            return None
        self._evict_to(slot, loc)
        self.seg[slot] = PROBATION                       # new entries: probation
        self.stamp[slot] = self._tick()
        return slot

    def _evict_to(self, slot: int, loc: int) -> None:
        """offloader.py:2076-2081: the slot's owner changes; its segment and
        recency do not."""
        old = self.expert_in_slot[slot]
        if old >= 0:
            self.slot_of[old] = -1
        self.expert_in_slot[slot] = loc
        self.slot_of[loc] = slot

    def _write_standing_map(self) -> None:
        """offloader.py:2112-2123 via _write_map 2083-2110."""
        m = [-1] * self.global_n
        for slot, loc in enumerate(self.expert_in_slot):
            if loc >= 0:
                m[self.global_of_local[loc]] = slot
        self.expert_map = m
        self.map_is_standing = True

    # -- the gap (offloader.py:2362-2467) -----------------------------------
    def gap(self, ids: list[int]) -> list[tuple[int, int]]:
        """Run one gap call over the flattened topk ids.

        Returns the fills ``[(local, slot), ...]`` in streaming order. Raises
        SlotOverflow with the state mutated up to the failed acquisition, as
        the reference does.
        """
        self.gaps += 1
        ids = [int(g) for g in ids]
        G = self.global_n
        if self.lfu:
            self.bump_freq(ids)
        if self.fast_hit and self.map_is_standing:          # 2409-2424
            all_hit = True
            for g in ids:
                if 0 <= g < G:
                    loc = self.local_of[g]
                    if loc >= 0 and self.slot_of[loc] < 0:
                        all_hit = False
                        break
            if all_hit:
                self.fast_hits += 1
                return []
        missing, hit_slots = [], set()
        for g in sorted(set(ids)):                            # 2427-2441
            if 0 <= g < G:
                loc = self.local_of[g]
                if loc < 0:
                    continue
                slot = self.slot_of[loc]
                if slot < 0:
                    missing.append(loc)
                else:
                    hit_slots.add(slot)
                    self._touch(slot, True)
        fills = []
        changed = False
        if missing:                                           # 2442-2465
            claimed = set(hit_slots)
            for loc in missing:
                slot = self._acquire(loc, claimed)
                if slot is None:
                    raise SlotOverflow(
                        "working set exceeds slots on a decode-sized step",
                        fills)
                fills.append((loc, slot))
                self.bytes_streamed += self.bytes_per_expert
                claimed.add(slot)
            self.misses += len(missing)
            changed = True
        if changed or not self.map_is_standing:               # 2466-2467
            self._write_standing_map()
        return fills

    # -- opt-in cross-layer prefetch (no counterpart in the reference) -------
    def prefetch(self, ids: list[int], max_fills: int) -> list[tuple[int, int]]:
        """Fill predicted experts ahead of this layer's gap (this build's
        opt-in prefetch; the reference measured its gate-ahead prefetch
        neutral and removed it, docs/EVALUATION.md:94-97, so there is no
        reference code to follow).

        Predicted owned experts that are not resident, in ascending id order,
        at most ``max_fills``: each takes the free list's next slot, else the
        least recently used probation slot that neither holds a predicted
        expert nor was taken by this call (never a protected or pinned slot),
        and becomes a new probation entry. No
        touches, no LFU bump, no gap counters; the standing map is rewritten
        when it was standing and something was filled."""
        fills = []
        wanted = sorted(set(int(v) for v in ids if 0 <= int(v) < self.global_n))
        # predicted residents keep their slots
        claimed = {self.slot_of[self.local_of[g]] for g in wanted
                   if self.local_of[g] >= 0 and self.slot_of[self.local_of[g]] >= 0}
        for g in wanted:
            if len(fills) >= max_fills:
                break
            loc = self.local_of[g]
            if loc < 0 or self.slot_of[loc] >= 0:
                continue
            if self.free_stack:
                slot = self.free_stack.pop()
            else:
                slot = next((c for c in self._lru(PROBATION) if c not in claimed), None)
                if slot is None:
                    break
            self._evict_to(slot, loc)
            self.seg[slot] = PROBATION
            self.stamp[slot] = self._tick()
            claimed.add(slot)
            fills.append((loc, slot))
        self.prefetches = getattr(self, "prefetches", 0) + len(fills)
        self.bytes_streamed += len(fills) * self.bytes_per_expert
        if fills and self.map_is_standing:
            self._write_standing_map()
        return fills

    # -- steps beyond the envelope (offloader.py:1452-1764, 1846-1933) --------
    def run_moe(self, ids: list[int], topk: int, decode_rows=0) -> list[dict]:
        """Plan one step through the classic hook over the flattened topk ids
        of ``len(ids) // topk`` tokens, on a real step.

        ``decode_rows`` is the step's decode signal (``_split_signal``): ``d > 0``
        — rows [0, d) are single-token decodes (vLLM's ``num_decode_tokens``
        equal to ``num_decodes``, decode rows first); ``0`` — no per-token
        signal (a pure prefill, or a backend without a decode count), so the
        working-set heuristic classifies the step; ``-1`` — short prefills
        folded into the decode count, so every expert is scan-class. A list of
        row indices is the opt-in non-MLA classifier's signal
        (``_non_mla_decode_rows`` 1802-1844, 1595-1611): those rows are the
        decodes, wherever they sit; an empty list is a pure prefill, every
        expert scan-class.

        Returns the waves in execution order, each ``{"map": [(global, slot)],
        "fills": [(local, slot)]}``: a wave's fills are streamed before its
        GEMM, its map routes exactly its experts, and the step's output is the
        sum of the waves' outputs. The expert map is left holding the last
        wave's map, not a standing one (``_write_map`` 2083-2110).
        """
        ids = [int(g) for g in ids]
        T = len(ids) // max(int(topk), 1)
        G = self.global_n
        selected = sorted(set(ids))                           # 1561
        decode_ids = None
        if not isinstance(decode_rows, int):                  # 1595-1611
            rows = [int(r) for r in decode_rows]
            forced_scan = False
            decode_ids = (set(selected) if len(rows) == T else
                          {ids[r * topk + j] for r in rows for j in range(topk)})
        else:
            forced_scan = decode_rows < 0                     # 1628 (nd > ndec)
            if 0 < decode_rows <= T:                          # 1578-1583
                decode_ids = (set(selected) if decode_rows == T
                              else set(ids[: decode_rows * topk]))
        pairs = []                                            # 1613-1621
        for g in selected:
            if 0 <= g < G and self.local_of[g] >= 0:
                pairs.append((g, self.local_of[g], decode_ids is not None and g in decode_ids))
        ws = len(pairs)
        if decode_ids is None and not forced_scan:            # 1629-1639
            n_pinned = sum(1 for v in self.seg if v == PINNED)
            if ws <= max(self.protected_cap + n_pinned, 1):
                pairs = [(g, loc, True) for g, loc, _ in pairs]
        if ws == 0:                                           # 1643-1645
            self.expert_map = [-1] * G
            self.map_is_standing = False
            return [{"map": [], "fills": []}]
        self.scan_steps += 1
        if self.lfu:                                          # 1662-1663
            self.bump_freq([g for g, _, _ in pairs])
        hits, missing = [], []                                # 1672-1681
        for g, loc, dcls in pairs:
            slot = self.slot_of[loc]
            if slot < 0:
                missing.append((g, loc, dcls))
            else:
                self._touch(slot, dcls)
                hits.append((g, slot))
        self.scan_hits += len(hits)
        self.scan_misses += len(missing)
        missing.sort(key=lambda m: not m[2])                  # 1689: decode class first
        claimed = {slot for _, slot in hits}
        wave0 = {"map": list(hits), "fills": []}
        taken = len(missing)
        for i, (g, loc, dcls) in enumerate(missing):          # 1701-1708
            slot = self._acquire(loc, claimed, allow_protected=dcls)
            if slot is None:
                taken = i
                break
            wave0["fills"].append((loc, slot))
            wave0["map"].append((g, slot))
            claimed.add(slot)
        waves = [wave0]
        leftover = [(g, loc) for g, loc, _ in missing[taken:]]
        if leftover:                                          # _run_waves
            rot = self._lru(PROBATION)                        # 1856-1862
            if not rot:
                rot = [s for s in range(self.num_slots)
                       if self.seg[s] != PINNED][-max(1, self.num_slots // 4):]
            half = (len(rot) + 1) // 2
            groups = (rot[:half], rot[half:] or rot[:half])
            i = 0
            while i < len(leftover):                          # 1874-1886
                group = groups[(len(waves) - 1) % 2]
                wave = {"map": [], "fills": []}
                for (g, loc), slot in zip(leftover[i: i + len(group)], group):
                    self._evict_to(slot, loc)
                    wave["fills"].append((loc, slot))
                    wave["map"].append((g, slot))
                i += len(wave["fills"])
                waves.append(wave)
        self.scan_waves += len(waves)
        self.bytes_streamed += self.bytes_per_expert * sum(len(w["fills"]) for w in waves)
        last = [-1] * G
        for g, slot in waves[-1]["map"]:
            last[g] = slot
        self.expert_map = last
        self.map_is_standing = False
        return waves

    # -- views ---------------------------------------------------------------
    def snapshot(self) -> dict:
        return {
            "expert_map": list(self.expert_map),
            "expert_in_slot": list(self.expert_in_slot),
            "protected": self._lru(PROTECTED),
            "probation": self._lru(PROBATION),
            "free": list(self.free_stack),
            "map_is_standing": self.map_is_standing,
            "gaps": self.gaps, "fast_hits": self.fast_hits,
            "misses": self.misses, "freq": list(self.freq),
        }
