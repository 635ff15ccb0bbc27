"""Per-layer expert slot cache with a device-resident SLRU policy.

Mirrors the reference's offloader state and lifecycle for the router-split
path (kfirtoledo/sluice ``src/sluice/offloader.py``):

* ``ExpertStreamOffloader(expert_cache_slots)`` — ``SLUICE_SLOTS`` slots per
  layer (``plugin.py:29-38``), ``SLUICE_PROTECT_FRAC`` (default 0.5, clamped to
  [0, 0.9]: ``offloader.py:236-241``), FAST_HIT (``SLUICE_RS_FAST_HIT``, on by
  default here as in the shipped configuration, ``README.md:90``).
* ``install_layer`` — ``_install_cache`` (895-1044): ``num_slots =
  min(slots, local_n)``, the protected cap, slot buffers ``[num_slots, ...]``
  per expert parameter, the host store of every local expert, the int32 expert
  map (``-1`` = not resident); full residency (``static_full``) installs the
  identity map and never streams; pins follow ``_apply_pins`` (1046-1083).
* ``SlotCache.gap(topk_ids)`` — the body of ``_router_split_gap``
  (2362-2467) on the device: the planner kernel updates the SLRU state and the
  standing expert map in place, the streamer kernel copies the misses from
  the mapped host store into their slots. No device-to-host synchronisation.
* ``SlotCache.plan_waves`` / ``stream_wave`` / ``wave_map`` — steps beyond
  the envelope, which the reference sends through its classic hook
  (``run_moe`` 1452-1764, ``_run_waves`` 1846-1933): the same state planned
  in expert waves on the device, each wave with its own fills and map.

Buffers are allocated once and never reallocated (captured CUDA graphs bake
pointers); a gap rewrites their contents only.
"""

from __future__ import annotations

import ctypes
import json
import os
import weakref
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from ._lib import CNT, HDR, SEG_FREE, SEG_PINNED, check, lib, ptr

PROTECT_FRAC_ENV = "SLUICE_PROTECT_FRAC"
SLOTS_ENV = "SLUICE_SLOTS"
FAST_HIT_ENV = "SLUICE_RS_FAST_HIT"
LFU_ENV = "SLUICE_LFU"
PIN_FILE_ENV = "SLUICE_PIN_FILE"


def load_pin_file(path: str) -> dict:
    """The static hot-expert pin file (offloader.py:466-483):
    ``{"layers": {"<MoE layer install ordinal>": [global ids, ...]}}`` (or the
    bare ``layers`` mapping). Unreadable or malformed files raise."""
    with open(path) as f:
        raw = json.load(f)
    layers = raw.get("layers", raw)
    return {int(k): [int(g) for g in v] for k, v in layers.items()}


def protected_cap_for(num_slots: int, protect_frac: float) -> int:
    """``min(int(slots * frac), slots - 1)`` with frac clamped to [0, 0.9]."""
    frac = min(max(float(protect_frac), 0.0), 0.9)
    return max(min(int(num_slots * frac), num_slots - 1), 0)


def max_waves_for(num_slots: int, local_n: int, protected_cap: int, n_pinned: int,
                  all_decode: bool = False) -> int:
    """An upper bound on the expert waves of one step (sl_plan_waves) that
    selects at most ``local_n`` of this rank's experts.

    When a miss finds no slot the free list is empty and the protected
    segment holds at most ``protected_cap`` slots, so the probation segment
    (the rotation) holds ``r >= num_slots - n_pinned - protected_cap``; wave 0
    claimed all of it, and every later wave takes a rotation group of at
    least ``r // 2`` slots (``_run_waves``, offloader.py:1856-1886). When every
    expert of the step is decode-class (``all_decode``), a miss may also take
    an unclaimed protected slot, so wave 0 claimed every unpinned slot."""
    r = max(num_slots - n_pinned - protected_cap, 1)
    wave0 = max(num_slots - n_pinned, r) if all_decode else r
    left = max(local_n - wave0, 0)
    g = max(r // 2, 1)
    return 1 + (left + g - 1) // g


def waves_pingpong(num_slots: int, protected_cap: int, n_pinned: int) -> bool:
    """Whether every wave step rotates two non-empty groups (so wave k's fills
    only wait for wave k - 2's GEMMs): a rotation of two or more slots."""
    return num_slots - n_pinned - protected_cap >= 2


def plan_ids_for(topk_ids: torch.Tensor, decode_rows) -> tuple[torch.Tensor, int]:
    """The ids ``sl_plan_waves`` plans a step from, and its decode signal.

    ``decode_rows`` is an int (rows [0, d) are decodes, 0 the working-set
    heuristic, < 0 a scan) or the indices of the decode rows wherever they
    sit — the opt-in non-MLA classifier's signal (``_non_mla_decode_rows``,
    offloader.py:1802-1844, used at 1595-1611). A wave plan depends only on
    the set of selected ids and on which of them decode rows select, not on
    row order, so the planner is given the decode rows first and their count;
    all rows decode is the whole step, no rows a scan (a pure prefill)."""
    ids = topk_ids if topk_ids.dtype == torch.int32 and topk_ids.is_contiguous() \
        else topk_ids.contiguous().to(torch.int32)
    if isinstance(decode_rows, int):
        return ids, decode_rows
    T = ids.shape[0]
    rows = torch.unique(torch.as_tensor(decode_rows, dtype=torch.long).flatten().cpu())
    if rows.numel() == 0:
        return ids, -1
    if rows.numel() == T:
        return ids, T
    mask = torch.zeros(T, dtype=torch.bool)
    mask[rows] = True
    order = torch.cat([rows, torch.nonzero(~mask).flatten()])
    return ids.index_select(0, order.to(ids.device)).contiguous(), int(rows.numel())


@dataclass
class InitialSlotState:
    """Host-computed starting residency of one layer's slots."""

    num_slots: int
    protected_cap: int
    expert_in_slot: list      # local id per slot, -1 free
    seg: list                 # SEG_* per slot
    free_stack: list          # bottom first; the next slot taken is the last
    fills: list               # (local, slot) copies to make at install


def initial_slot_state(num_slots: int, local_of: list, local_n: int, protect_frac: float,
                       pins: list | None = None,
                       prefill_resident: bool = False) -> InitialSlotState:
    """Starting state per ``_install_cache`` (936-1003) and ``_apply_pins``
    (1046-1083): free list ``[S-1, ..., 0]`` popped from the end; pins take
    free slots, sit outside both SLRU segments and reduce the protected cap."""
    S = num_slots
    cap = protected_cap_for(S, protect_frac)
    eis = [-1] * S
    seg = [SEG_FREE] * S
    free = list(range(S - 1, -1, -1))
    fills = []
    if prefill_resident:
        for loc in range(local_n):
            eis[loc] = loc
            seg[loc] = SEG_PINNED
            fills.append((loc, loc))
        free = list(range(S - 1, local_n - 1, -1))
    if pins:
        resident = set(v for v in eis if v >= 0)
        n = 0
        for g in pins:
            if n >= cap:
                break
            if not (0 <= g < len(local_of)):
                continue
            loc = local_of[g]
            if loc < 0 or loc in resident or not free:
                continue
            slot = free.pop()
            eis[slot] = loc
            seg[slot] = SEG_PINNED
            resident.add(loc)
            fills.append((loc, slot))
            n += 1
        cap -= n
    return InitialSlotState(S, cap, eis, seg, free, fills)


class HostStore:
    """Page-locked, device-mapped host buffer (``cudaHostAlloc`` Mapped|Portable)."""

    def __init__(self, nbytes: int):
        p = ctypes.c_void_p()
        check(lib().sl_host_alloc_mapped(nbytes, ctypes.byref(p)), "sl_host_alloc_mapped")
        self.ptr = p.value
        self.nbytes = nbytes
        buf = (ctypes.c_uint8 * nbytes).from_address(self.ptr)
        self.bytes = torch.frombuffer(buf, dtype=torch.uint8)
        self._fin = weakref.finalize(self, lib().sl_host_free, ctypes.c_void_p(self.ptr))

    def view(self, dtype, shape) -> torch.Tensor:
        return self.bytes.view(dtype).view(shape)


class SlotCache:
    """One MoE layer's slots, host store, expert map and device SLRU state.

    Per-expert parameters: ``w13``, ``w2`` and, for fp8 block-scaled experts,
    ``w13_scale``, ``w2_scale`` — every one streamed on a miss."""

    def __init__(self, num_slots: int, local_n: int, global_n: int, local_of: list,
                 protected_cap: int, static_full: bool, device: torch.device,
                 gpu_cache: dict, cpu_store: dict, expert_map: torch.Tensor,
                 state: torch.Tensor | None, bytes_per_expert: int, n_pinned: int = 0):
        self.num_slots = num_slots
        self.local_n = local_n
        self.global_n = global_n
        self.local_of = local_of
        self.protected_cap = protected_cap
        self.static_full = static_full
        self.device = device
        self.gpu_cache = gpu_cache
        self.cpu_store = cpu_store
        self.expert_map = expert_map
        self.state = state
        self.bytes_per_expert = bytes_per_expert
        self._stream_args = None
        if state is not None:
            offs = (ctypes.c_size_t * (_lib.STATE_NFIELDS + 1))()
            check(lib().sl_slot_state_offsets(num_slots, global_n, local_n, offs),
                  "sl_slot_state_offsets")
            self.offsets = list(offs)
            names = list(gpu_cache)
            n = len(names)
            src = (ctypes.c_void_p * n)(*[cpu_store[k].data_ptr() for k in names])
            dst = (ctypes.c_void_p * n)(*[gpu_cache[k].data_ptr() for k in names])
            nb = (ctypes.c_size_t * n)(*[cpu_store[k][0].numel() * cpu_store[k].element_size()
                                         for k in names])
            # bytes between consecutive experts of each parameter in the host
            # store: the parameter's size, or the record size of a packed store
            hs = (ctypes.c_size_t * n)(*[cpu_store[k].stride(0) * cpu_store[k].element_size()
                                         for k in names])
            self._stream_args = (n, src, dst, nb, hs)
            # the wave plan of steps beyond the envelope (sl_plan_waves)
            self.n_pinned = n_pinned
            self.max_waves = max_waves_for(num_slots, local_n, protected_cap, n_pinned)
            self.waves_pingpong = waves_pingpong(num_slots, protected_cap, n_pinned)
            nbytes = lib().sl_wave_plan_bytes(num_slots, global_n, self.max_waves)
            self.waves = torch.empty(nbytes, dtype=torch.uint8, device=device)
            check(lib().sl_wave_plan_init(ptr(self.waves), num_slots, global_n, self.max_waves,
                                          torch.cuda.current_stream(device).cuda_stream),
                  "sl_wave_plan_init")
            woff = (ctypes.c_size_t * (_lib.WAVE_NFIELDS + 1))()
            check(lib().sl_wave_plan_offsets(num_slots, global_n, self.max_waves, woff),
                  "sl_wave_plan_offsets")
            self.wave_offsets = list(woff)
            words = self.waves.view(torch.int32)
            self.wave_maps = words[woff[4] // 4: woff[4] // 4 + self.max_waves * global_n] \
                .view(self.max_waves, global_n)

    @property
    def w13(self) -> torch.Tensor:
        return self.gpu_cache["w13"]

    @property
    def w2(self) -> torch.Tensor:
        return self.gpu_cache["w2"]

    @property
    def w13_scale(self) -> torch.Tensor | None:
        return self.gpu_cache.get("w13_scale")

    @property
    def w2_scale(self) -> torch.Tensor | None:
        return self.gpu_cache.get("w2_scale")

    # -- the gap ---------------------------------------------------------
    def gap(self, topk_ids: torch.Tensor, stream_ctas: int = 0) -> None:
        """Plan slots for this step's ids and stream the misses (async)."""
        if self.static_full:
            return
        self.plan(topk_ids)
        self.stream(stream_ctas)

    def plan(self, topk_ids: torch.Tensor) -> None:
        """The gap's slot planning on the current stream (updates the map)."""
        ids = topk_ids if topk_ids.dtype == torch.int32 and topk_ids.is_contiguous() \
            else topk_ids.contiguous().to(torch.int32)
        check(lib().sl_plan_slots(ptr(self.state), ptr(ids), ids.numel(), ptr(self.expert_map),
                                  torch.cuda.current_stream().cuda_stream), "sl_plan_slots")

    def prefetch(self, topk_ids: torch.Tensor, max_fills: int) -> None:
        """Opt-in cross-layer prefetch on the current stream
        (``sl_prefetch_slots``): up to ``max_fills`` predicted experts that are
        not resident take free or least recently used probation slots; call
        ``stream()`` after it, and order this layer's next ``plan()`` after
        that stream."""
        ids = topk_ids if topk_ids.dtype == torch.int32 and topk_ids.is_contiguous() \
            else topk_ids.contiguous().to(torch.int32)
        check(lib().sl_prefetch_slots(ptr(self.state), ptr(ids), ids.numel(), int(max_fills),
                                      ptr(self.expert_map),
                                      torch.cuda.current_stream().cuda_stream),
              "sl_prefetch_slots")

    def stream(self, stream_ctas: int = 0) -> None:
        """Stream the last plan's fills on the current stream."""
        n, src, dst, nb, hs = self._stream_args
        check(lib().sl_stream_experts_strided(ptr(self.state), n, src, dst, nb, hs,
                                              int(stream_ctas),
                                              torch.cuda.current_stream().cuda_stream),
              "sl_stream_experts_strided")

    # -- steps beyond the envelope: expert waves -----------------------------
    def plan_waves(self, topk_ids: torch.Tensor, decode_rows=0) -> None:
        """Plan this step's expert waves on the current stream (run_moe and
        _run_waves, offloader.py:1452-1764, 1846-1933): ``topk_ids`` [T, k];
        ``decode_rows`` > 0 marks rows [0, decode_rows) as decodes, 0 leaves
        the class to the working-set heuristic, < 0 makes every expert
        scan-class; a sequence / tensor of row indices marks those rows
        (``plan_ids_for``)."""
        ids, d = plan_ids_for(topk_ids, decode_rows)
        T, k = ids.shape
        check(lib().sl_plan_waves(ptr(self.state), ptr(ids), T, k, int(d),
                                  ptr(self.expert_map), ptr(self.waves),
                                  torch.cuda.current_stream().cuda_stream), "sl_plan_waves")

    def waves_for(self, pairs: int, all_decode: bool = False) -> int:
        """The waves a step of ``pairs`` (token, expert) pairs can need: it
        selects at most ``min(local_n, pairs)`` experts; ``all_decode``: every
        one of them decode-class."""
        return min(self.max_waves, max_waves_for(self.num_slots, min(self.local_n, pairs),
                                                 self.protected_cap, self.n_pinned,
                                                 all_decode))

    def stream_wave(self, wave: int, stream_ctas: int = 0) -> None:
        """Stream wave ``wave``'s fills of the last wave plan (current stream)."""
        n, src, dst, nb, hs = self._stream_args
        check(lib().sl_stream_wave(ptr(self.waves), int(wave), n, src, dst, nb, hs,
                                   int(stream_ctas), torch.cuda.current_stream().cuda_stream),
              "sl_stream_wave")

    def wave_map(self, wave: int) -> torch.Tensor:
        """Wave ``wave``'s expert map (int32 [global_n], a view of the plan)."""
        return self.wave_maps[wave]

    def wave_plan(self) -> list[dict]:
        """The last wave plan as ``[{"map": [(global, slot)], "fills":
        [(local, slot)]}]`` (synchronises; for tests)."""
        words = self.waves.view(torch.int32).cpu().numpy()
        o = [v // 4 for v in self.wave_offsets]
        S, G = self.num_slots, self.global_n
        nw = int(words[_lib.WAVE_HDR["num_waves"]])
        out = []
        for k in range(nw):
            c = int(words[o[1] + k])
            loc = words[o[2] + k * S: o[2] + k * S + c].tolist()
            slot = words[o[3] + k * S: o[3] + k * S + c].tolist()
            m = words[o[4] + k * G: o[4] + (k + 1) * G]
            out.append({"map": [(g, int(m[g])) for g in range(G) if m[g] >= 0],
                        "fills": list(zip(loc, slot))})
        return out

    def wave_header(self) -> dict:
        h = self.waves[:64].view(torch.int32).cpu().tolist()
        return {k: int(h[v]) for k, v in _lib.WAVE_HDR.items()}

    # -- saving and restoring the cache (benchmarks, tests) -------------------
    def save(self) -> dict:
        """A device copy of everything a gap reads or writes: the planner
        state, the expert map and the slot buffers (allocates their size)."""
        return {"state": None if self.state is None else self.state.clone(),
                "expert_map": self.expert_map.clone(),
                "slots": {k: t.clone() for k, t in self.gpu_cache.items()}}

    def restore(self, saved: dict) -> None:
        """Put back a ``save()``: the next gap plans exactly as it would have
        then (copies on the current stream; buffers keep their addresses)."""
        if self.state is not None:
            self.state.copy_(saved["state"])
        self.expert_map.copy_(saved["expert_map"])
        for k, t in self.gpu_cache.items():
            t.copy_(saved["slots"][k])

    def last_fill_counts(self, wave_steps: bool = False) -> list[int]:
        """Experts streamed by the last gap (one entry) or, with
        ``wave_steps``, by each wave of the last wave plan (synchronises)."""
        if self.state is None:
            return []
        if not wave_steps:
            return [self.header()["fill_count"]]
        words = self.waves.view(torch.int32)
        o = self.wave_offsets[1] // 4
        nw = int(words[_lib.WAVE_HDR["num_waves"]].item())
        counts = words[o: o + self.max_waves].cpu().tolist()
        # waves past the plan's count stream nothing (their entries are stale)
        return [c if k < nw else 0 for k, c in enumerate(counts)]

    # -- host-side views (synchronise) ----------------------------------------
    def _field(self, i: int, dtype, count: int) -> np.ndarray:
        b = self.state[self.offsets[i]: self.offsets[i] + count * np.dtype(dtype).itemsize]
        return b.cpu().numpy().view(dtype)

    def header(self) -> dict:
        h = self._field(0, np.int32, 16)
        return {k: int(h[v]) for k, v in HDR.items()}

    def counters(self) -> dict:
        c = self._field(1, np.uint64, _lib.NUM_COUNTERS)
        return {k: int(c[v]) for k, v in CNT.items()}

    def check(self) -> None:
        """Raise the reference's overflow error if the last gap overflowed."""
        if self.state is None:
            return
        st = self.header()["status"]
        if st != _lib.SL_OK:
            raise _lib.SluiceError("sluice_stream_gap", st)

    def snapshot(self) -> dict:
        """Expert map, slot owners, SLRU order and counters (for tests)."""
        S = self.num_slots
        eis = self._field(5, np.int32, S).tolist()
        seg = self._field(6, np.uint8, S).tolist()
        stamp = self._field(7, np.uint32, S).tolist()
        order = lambda v: sorted((s for s in range(S) if seg[s] == v), key=lambda s: stamp[s])
        return {
            "expert_map": self.expert_map.cpu().tolist(),
            "expert_in_slot": eis,
            "protected": order(_lib.SEG_PROTECTED),
            "probation": order(_lib.SEG_PROBATION),
            "header": self.header(),
            "counters": self.counters(),
            "freq": self._field(11, np.uint32, self.local_n).tolist(),
            "fills": list(zip(self._field(9, np.int32, S).tolist(),
                              self._field(10, np.int32, S).tolist()))[: self.header()["fill_count"]],
        }

    def stats(self) -> dict:
        if self.state is None:
            return {"static_full": True}
        c = self.counters()
        c["bytes_streamed"] = c["fills"] * self.bytes_per_expert
        return c


class ExpertStreamOffloader:
    """Installs slot caches for MoE layers (``SLUICE_SLOTS`` per layer)."""

    def __init__(self, expert_cache_slots: int, protect_frac: float | None = None,
                 fast_hit: bool | None = None, no_static_full: bool = False,
                 lfu: bool | None = None, pin_file: str | None = None,
                 packed_host_store: bool = False):
        if expert_cache_slots <= 0:
            raise ValueError("expert_cache_slots must be positive")
        self.expert_cache_slots = int(expert_cache_slots)
        if protect_frac is None:
            try:
                protect_frac = float(os.environ.get(PROTECT_FRAC_ENV, "0.5"))
            except ValueError:
                protect_frac = 0.5
        self.protect_frac = min(max(protect_frac, 0.0), 0.9)
        if fast_hit is None:
            fast_hit = os.environ.get(FAST_HIT_ENV, "1") != "0"
        self.fast_hit = bool(fast_hit)
        # SLUICE_LFU=1 (offloader.py:242-247): popularity-ordered protected victims
        if lfu is None:
            lfu = os.environ.get(LFU_ENV, "0") == "1"
        self.lfu = bool(lfu)
        # SLUICE_PIN_FILE: per-layer static pins, applied in install order
        if pin_file is None:
            pin_file = os.environ.get(PIN_FILE_ENV) or None
        self.pin_layers = load_pin_file(pin_file) if pin_file else None
        self.no_static_full = bool(no_static_full)
        # one host record per expert ([w13 | w2 | scales]) instead of one
        # host array per parameter: each fill reads one contiguous range
        self.packed_host_store = bool(packed_host_store)
        self.caches: list[SlotCache] = []

    @classmethod
    def from_env(cls) -> "ExpertStreamOffloader | None":
        raw = os.environ.get(SLOTS_ENV)
        if not raw:
            return None
        return cls(int(raw))

    def install_layer(self, w13: torch.Tensor, w2: torch.Tensor, global_n: int | None = None,
                      local_of: list | None = None, pins: list | None = None,
                      device: torch.device | str = "cuda",
                      w13_scale: torch.Tensor | None = None,
                      w2_scale: torch.Tensor | None = None,
                      prefill_resident: bool | None = None) -> SlotCache:
        """Install one layer from its local experts ``w13`` [L, 2I, H], ``w2``
        [L, H, I] (bf16, or fp8 e4m3 with fp32 128x128 block scales
        ``w13_scale`` [L, 2I/128, H/128], ``w2_scale`` [L, H/128, I/128]; CPU or
        CUDA tensors, copied into the host store). ``prefill_resident=False``
        starts a cache with room for every expert (``no_static_full``) holding
        only the pins, so the rest stream in on first use."""
        device = torch.device(device)
        local_n = w13.shape[0]
        if global_n is None:
            global_n = local_n
        if local_of is None:
            if global_n != local_n:
                raise ValueError("local_of is required when global_n != local_n")
            local_of = list(range(global_n))
        local_of = [int(v) for v in local_of]
        S = min(self.expert_cache_slots, local_n)
        resident_all = S >= local_n
        static_full = resident_all and not self.no_static_full
        params = {"w13": w13, "w2": w2}
        if w13_scale is not None:
            params["w13_scale"] = w13_scale.float().contiguous()
            params["w2_scale"] = w2_scale.float().contiguous()
        gpu_cache, cpu_store = {}, {}
        bpe = 0
        sizes = {name: p[0].numel() * p.element_size() for name, p in params.items()}
        packed = (self.packed_host_store and not static_full and
                  all(b % 16 == 0 for b in sizes.values()))
        record = sum(sizes.values())
        pstore = HostStore(local_n * record) if packed else None
        offset = 0
        for name, p in params.items():
            gpu_cache[name] = torch.empty((S, *p.shape[1:]), dtype=p.dtype, device=device)
            bpe += sizes[name]
            if static_full:
                gpu_cache[name].copy_(p)
            elif packed:
                # parameter `name` of expert l at byte l * record + offset
                es = p.element_size()
                inner = torch.empty(p.shape[1:], dtype=p.dtype, device="meta").stride()
                t = torch.as_strided(pstore.bytes.view(p.dtype), (local_n, *p.shape[1:]),
                                     (record // es, *inner), offset // es)
                t.copy_(p)
                t._sluice_store = pstore  # keep the allocation alive with the view
                cpu_store[name] = t
                offset += sizes[name]
            else:
                store = HostStore(p.numel() * p.element_size())
                t = store.view(p.dtype, p.shape)
                t.copy_(p)
                t._sluice_store = store  # keep the allocation alive with the view
                cpu_store[name] = t
        emap = torch.full((global_n,), -1, dtype=torch.int32, device=device)
        if static_full:
            lo = torch.tensor(local_of, dtype=torch.int32)
            emap.copy_(torch.where(lo >= 0, lo, torch.full_like(lo, -1)))
            cache = SlotCache(S, local_n, global_n, local_of, 0, True, device, gpu_cache,
                              cpu_store, emap, None, bpe)
            self.caches.append(cache)
            return cache
        if pins is None and self.pin_layers is not None:
            # the reference applies the file's list for this install ordinal
            # to every layer that is not static_full (offloader.py:1025-1026)
            pins = self.pin_layers.get(len(self.caches), [])
        init = initial_slot_state(S, local_of, local_n, self.protect_frac, pins,
                                  prefill_resident=resident_all if prefill_resident is None
                                  else prefill_resident)
        nbytes = lib().sl_slot_state_bytes(S, global_n, local_n)
        state = torch.zeros(nbytes, dtype=torch.uint8, device=device)
        arr = lambda v, t: (t * len(v))(*v)
        rc = lib().sl_slot_state_init(
            ptr(state), S, global_n, local_n, init.protected_cap,
            (_lib.PLAN_FAST_HIT if self.fast_hit else 0) | (_lib.PLAN_LFU if self.lfu else 0),
            arr(local_of, ctypes.c_int32), arr(init.expert_in_slot, ctypes.c_int32),
            arr(init.seg, ctypes.c_uint8), arr(init.free_stack or [0], ctypes.c_int32),
            len(init.free_stack), torch.cuda.current_stream(device).cuda_stream)
        check(rc, "sl_slot_state_init")
        for loc, slot in init.fills:
            for name in params:
                gpu_cache[name][slot].copy_(cpu_store[name][loc])
        cache = SlotCache(S, local_n, global_n, local_of, init.protected_cap, False, device,
                          gpu_cache, cpu_store, emap, state, bpe,
                          n_pinned=sum(1 for v in init.seg if v == SEG_PINNED))
        self.caches.append(cache)
        return cache

    def get_stats(self) -> list[dict]:
        return [c.stats() for c in self.caches]
