// Device-resident slot cache: state layout, planner (the router-split gap's
// SLRU policy, no host round trip) and the GPU-initiated expert streamer.
//
// Reference: kfirtoledo/sluice src/sluice/offloader.py
//   state      _ExpertLayerCache 121-169, _install_cache 936-1003
//   gap        _router_split_gap 2362-2467 (FAST_HIT 2409-2424)
//   policy     _touch 2009-2021, _coldest_protected 2023-2034,
//              _acquire_slot 2036-2074, _evict_to 2076-2081
//   LFU        _bump_freq 1993-2007 (SLUICE_LFU; LFU_AGE_STEPS = 256, line 118)
//   map        _write_map / _write_standing_map 2083-2123
//   streaming  _stream_in 2709-2723
//
// Recency: every slot of the probation / protected segments carries a
// 32-bit stamp from one per-layer clock; a segment's LRU order is ascending
// stamp, and "move to end" is "take the next stamp". Stamps are renumbered
// (order kept) before the clock could overflow.
#include <stdlib.h>
#include <string.h>

#include "common.cuh"
#include "slot_state.cuh"

namespace {

constexpr int kMaxSlots = 1024;
constexpr int kMaxGlobal = 4096;
constexpr uint32_t kClockRenorm = 0x7fff0000u;
constexpr int kLfuAgeSteps = 256;  // offloader.py:118

// Planner shared memory, carved at run time from the state's dimensions:
// the id bitmaps, the sorted unique ids, and copies of every state array the
// sequential pass touches (so it never waits on global memory).
constexpr int kPlanSmemBytes = 72 * 1024;
constexpr int kMaxWaves = kMaxGlobal + 1;

enum PlanField {
  PS_SCAL, PS_BITMAP, PS_DBITMAP, PS_WORD_BASE, PS_UNIQ, PS_LOCAL_OF, PS_SLOT_OF,
  PS_MISS_LOC, PS_STAMP, PS_EIS, PS_FREE, PS_SFREQ, PS_ROT, PS_SEG, PS_CLAIMED, PS_MCLS,
  PS_N
};

struct PlanSmem {
  int* scal;          // gap: [0] any miss, [1] unique ids, [2] map decision;
                      // waves: [0] working set, [1] unique ids, [2] pinned slots, [3] waves
  uint32_t* bitmap;   // [W] selected ids
  uint32_t* dbitmap;  // [W] ids selected by decode rows (waves)
  uint32_t* word_base;
  int32_t* uniq;      // [G] sorted unique ids (waves: afterwards the ordered misses)
  int32_t* local_of;  // [G]
  int32_t* slot_of;   // [L]
  int32_t* miss_loc;  // [max(S + 1, L)]
  uint32_t* stamp;    // [S]
  int32_t* eis;       // [S]
  int32_t* free_s;    // [S]
  uint32_t* sfreq;    // [S] LFU count of each slot's expert
  int32_t* rot;       // [S] rotation slots (waves)
  uint8_t* seg;       // [S]
  uint8_t* claimed;   // [S]
  uint8_t* mcls;      // [L] decode class of each miss (waves)
};

__host__ __device__ inline void plan_smem_layout(int S, int G, int L, size_t* off) {
  const size_t W = (G + 31) / 32, M = S + 1 > L ? S + 1 : L;
  const size_t s4 = 4 * size_t(S);
  const size_t bytes[PS_N] = {16,    4 * W, 4 * W, 4 * W,     4 * size_t(G), 4 * size_t(G),
                              4 * size_t(L), 4 * M, s4, s4, s4, s4, s4, size_t(S),
                              size_t(S), size_t(L)};
  size_t o = 0;
  for (int i = 0; i < PS_N; ++i) {
    off[i] = o;
    o += round16(bytes[i]);
  }
  off[PS_N] = o;
}

__host__ __device__ inline size_t plan_smem_bytes(int S, int G, int L) {
  size_t off[PS_N + 1];
  plan_smem_layout(S, G, L, off);
  return off[PS_N];
}

__host__ __device__ inline bool plan_dims_ok(int S, int G, int L) {
  return S > 0 && S <= kMaxSlots && G > 0 && G <= kMaxGlobal && L > 0 && L <= kMaxGlobal &&
         plan_smem_bytes(S, G, L) <= kPlanSmemBytes;
}

__device__ inline PlanSmem plan_smem(uint8_t* base, int S, int G, int L) {
  size_t off[PS_N + 1];
  plan_smem_layout(S, G, L, off);
  PlanSmem m;
  m.scal = reinterpret_cast<int*>(base + off[PS_SCAL]);
  m.bitmap = reinterpret_cast<uint32_t*>(base + off[PS_BITMAP]);
  m.dbitmap = reinterpret_cast<uint32_t*>(base + off[PS_DBITMAP]);
  m.word_base = reinterpret_cast<uint32_t*>(base + off[PS_WORD_BASE]);
  m.uniq = reinterpret_cast<int32_t*>(base + off[PS_UNIQ]);
  m.local_of = reinterpret_cast<int32_t*>(base + off[PS_LOCAL_OF]);
  m.slot_of = reinterpret_cast<int32_t*>(base + off[PS_SLOT_OF]);
  m.miss_loc = reinterpret_cast<int32_t*>(base + off[PS_MISS_LOC]);
  m.stamp = reinterpret_cast<uint32_t*>(base + off[PS_STAMP]);
  m.eis = reinterpret_cast<int32_t*>(base + off[PS_EIS]);
  m.free_s = reinterpret_cast<int32_t*>(base + off[PS_FREE]);
  m.sfreq = reinterpret_cast<uint32_t*>(base + off[PS_SFREQ]);
  m.rot = reinterpret_cast<int32_t*>(base + off[PS_ROT]);
  m.seg = base + off[PS_SEG];
  m.claimed = base + off[PS_CLAIMED];
  m.mcls = base + off[PS_MCLS];
  return m;
}

// Least-recently-used slot of segment `want` (optionally skipping claimed
// slots), or -1. Whole warp; stamps of live slots are unique.
__device__ int warp_lru(const PlanSmem& sm, int S, uint8_t want, bool skip_claimed) {
  const int lane = threadIdx.x & 31;
  uint32_t best = 0xffffffffu;
  int bslot = -1;
  for (int s = lane; s < S; s += 32) {
    if (sm.seg[s] == want && !(skip_claimed && sm.claimed[s]) && sm.stamp[s] < best) {
      best = sm.stamp[s];
      bslot = s;
    }
  }
  const uint32_t m = __reduce_min_sync(0xffffffffu, best);
  const uint32_t bal = __ballot_sync(0xffffffffu, bslot >= 0 && best == m);
  if (!bal) return -1;
  return __shfl_sync(0xffffffffu, bslot, __ffs(bal) - 1);
}

// Least-frequently-used slot of segment `want`, least recently used among
// equal counts (the LFU order of offloader.py:2023-2034 / 2056-2066), or -1.
// Whole warp; the key (count, stamp) is unique among live slots.
__device__ int warp_lfu(const PlanSmem& sm, int S, uint8_t want, bool skip_claimed) {
  const int lane = threadIdx.x & 31;
  unsigned long long best = ~0ull;
  int bslot = -1;
  for (int s = lane; s < S; s += 32) {
    const unsigned long long key =
        (static_cast<unsigned long long>(sm.sfreq[s]) << 32) | sm.stamp[s];
    if (sm.seg[s] == want && !(skip_claimed && sm.claimed[s]) && key < best) {
      best = key;
      bslot = s;
    }
  }
  unsigned long long m = best;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long v = __shfl_xor_sync(0xffffffffu, m, o);
    m = v < m ? v : m;
  }
  const uint32_t bal = __ballot_sync(0xffffffffu, bslot >= 0 && best == m);
  if (!bal) return -1;
  return __shfl_sync(0xffffffffu, bslot, __ffs(bal) - 1);
}

// Copy the state arrays the sequential pass uses into shared memory and clear
// the bitmaps, the claims and the scalars. Block-wide.
__device__ void load_plan_state(const StateView& st, const PlanSmem& sm, int S, int G, int L) {
  const int tid = threadIdx.x, nthr = blockDim.x, nwords = (G + 31) >> 5;
  for (int i = tid; i < nwords; i += nthr) sm.bitmap[i] = 0, sm.dbitmap[i] = 0;
  for (int g = tid; g < G; g += nthr) sm.local_of[g] = st.local_of[g];
  for (int l = tid; l < L; l += nthr) sm.slot_of[l] = st.slot_of[l];
  for (int s = tid; s < S; s += nthr) {
    sm.seg[s] = st.seg[s];
    sm.stamp[s] = st.stamp[s];
    sm.eis[s] = st.eis[s];
    sm.free_s[s] = st.free_stack[s];
    sm.claimed[s] = 0;
  }
  if (tid < 4) sm.scal[tid] = 0;
}

// _bump_freq (offloader.py:1993-2007): +1 per selected owned expert (each set
// bit once), the periodic halving, then the count of each slot's expert.
// Block-wide; the caller synchronises before reading sfreq.
__device__ void lfu_bump(const StateView& st, const PlanSmem& sm, int S, int G, int L) {
  const int tid = threadIdx.x, nthr = blockDim.x, nwords = (G + 31) >> 5;
  for (int w = tid; w < nwords; w += nthr) {
    uint32_t bits = sm.bitmap[w];
    while (bits) {
      const int g = (w << 5) + __ffs(bits) - 1;
      bits &= bits - 1;
      const int loc = sm.local_of[g];
      if (loc >= 0) st.freq[loc] += 1;
    }
  }
  __syncthreads();
  const int steps = st.hdr[SL_HDR_LFU_STEPS] + 1;
  const bool age = steps >= kLfuAgeSteps;
  if (age)
    for (int l = tid; l < L; l += nthr) st.freq[l] >>= 1;
  __syncthreads();
  if (tid == 0) st.hdr[SL_HDR_LFU_STEPS] = age ? 0 : steps;
  for (int s = tid; s < S; s += nthr) sm.sfreq[s] = sm.eis[s] >= 0 ? st.freq[sm.eis[s]] : 0;
}

// sorted(set(ids)): expand the bitmap in ascending order into uniq; the count
// goes to scal[1]. Block-wide; ends synchronised.
__device__ void expand_uniques(const PlanSmem& sm, int G) {
  const int tid = threadIdx.x, nthr = blockDim.x, nwords = (G + 31) >> 5;
  if (tid < 32) {
    uint32_t run = 0;
    for (int w0 = 0; w0 < nwords; w0 += 32) {
      const int w = w0 + tid;
      const uint32_t c = w < nwords ? __popc(sm.bitmap[w]) : 0;
      uint32_t incl = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t n = __shfl_up_sync(0xffffffffu, incl, o);
        if (tid >= o) incl += n;
      }
      if (w < nwords) sm.word_base[w] = run + incl - c;
      run += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (tid == 0) sm.scal[1] = static_cast<int>(run);
  }
  __syncthreads();
  for (int w = tid; w < nwords; w += nthr) {
    uint32_t bits = sm.bitmap[w];
    uint32_t pos = sm.word_base[w];
    while (bits) {
      const int b = __ffs(bits) - 1;
      bits &= bits - 1;
      sm.uniq[pos++] = (w << 5) + b;
    }
  }
  __syncthreads();
}

// Renumber the live stamps (order kept) before the per-layer clock can wrap;
// returns the clock to continue from. Block-wide; ends synchronised.
__device__ uint32_t renorm_stamps(const StateView& st, const PlanSmem& sm, int S) {
  const int tid = threadIdx.x, nthr = blockDim.x;
  uint32_t clock0 = static_cast<uint32_t>(st.hdr[SL_HDR_CLOCK]);
  if (clock0 > kClockRenorm) {
    uint32_t newstamp[kMaxSlots / 256];
    int nlive = 0;
    for (int s = 0; s < S; ++s) nlive += (sm.seg[s] == SL_SEG_PROBATION || sm.seg[s] == SL_SEG_PROTECTED);
    for (int k = 0, s = tid; s < S; s += nthr, ++k) {
      uint32_t r = 0;
      if (sm.seg[s] == SL_SEG_PROBATION || sm.seg[s] == SL_SEG_PROTECTED)
        for (int q = 0; q < S; ++q)
          r += (sm.seg[q] == SL_SEG_PROBATION || sm.seg[q] == SL_SEG_PROTECTED) &&
               sm.stamp[q] < sm.stamp[s];
      newstamp[k] = r + 1;
    }
    __syncthreads();
    for (int k = 0, s = tid; s < S; s += nthr, ++k)
      if (sm.seg[s] == SL_SEG_PROBATION || sm.seg[s] == SL_SEG_PROTECTED) sm.stamp[s] = newstamp[k];
    clock0 = static_cast<uint32_t>(nlive);
  }
  __syncthreads();
  return clock0;
}

// _touch (offloader.py:2009-2021) of a hit slot: protected hits and
// unfriendly probation hits move to their segment's end; friendly probation
// hits are promoted, demoting the coldest protected slots while the segment
// is over its cap. Whole warp (uniform arguments); lane 0 writes.
__device__ void warp_touch(const PlanSmem& sm, int S, int slot, bool friendly, int cap, bool lfu,
                           int& pcount, uint32_t& clock) {
  const int lane = threadIdx.x & 31;
  const uint8_t sg = sm.seg[slot];
  if (sg == SL_SEG_PROTECTED) {
    ++clock;
    if (lane == 0) sm.stamp[slot] = clock;
  } else if (sg == SL_SEG_PROBATION) {
    ++clock;
    if (friendly && cap > 0) {
      if (lane == 0) {
        sm.seg[slot] = SL_SEG_PROTECTED;
        sm.stamp[slot] = clock;
      }
      ++pcount;
      while (pcount > cap) {
        __syncwarp();
        const int v = lfu ? warp_lfu(sm, S, SL_SEG_PROTECTED, false)
                          : warp_lru(sm, S, SL_SEG_PROTECTED, false);
        ++clock;
        if (lane == 0) {
          sm.seg[v] = SL_SEG_PROBATION;
          sm.stamp[v] = clock;
        }
        --pcount;
      }
    } else if (lane == 0) {
      sm.stamp[slot] = clock;
    }
  }
}

// _acquire_slot (offloader.py:2036-2074) up to the eviction: the free list,
// then the least recently used unclaimed probation slot, then (if allowed)
// the coldest unclaimed protected slot; -1 when none. Whole warp.
__device__ int warp_acquire(const PlanSmem& sm, int S, bool allow_protected, bool lfu,
                            int& free_top, int& pcount) {
  if (free_top > 0) return sm.free_s[--free_top];
  int slot = warp_lru(sm, S, SL_SEG_PROBATION, true);
  if (slot < 0 && allow_protected) {
    slot = lfu ? warp_lfu(sm, S, SL_SEG_PROTECTED, true)
               : warp_lru(sm, S, SL_SEG_PROTECTED, true);
    if (slot >= 0) --pcount;
  }
  return slot;
}

// _evict_to (offloader.py:2076-2081): the slot's owner becomes `loc`.
__device__ inline void evict_to(const PlanSmem& sm, int slot, int loc) {
  const int old = sm.eis[slot];
  if (old >= 0) sm.slot_of[old] = -1;
  sm.eis[slot] = loc;
  sm.slot_of[loc] = slot;
}

// A miss placed by _acquire_slot: evicted into, a new probation entry, claimed.
__device__ inline void place_fill(const StateView& st, const PlanSmem& sm, int slot, int loc,
                                  uint32_t clock, bool lfu) {
  evict_to(sm, slot, loc);
  sm.seg[slot] = SL_SEG_PROBATION;
  sm.stamp[slot] = clock;
  sm.claimed[slot] = 1;
  if (lfu) sm.sfreq[slot] = st.freq[loc];
}

__device__ void store_plan_state(const StateView& st, const PlanSmem& sm, int S, int L) {
  const int tid = threadIdx.x, nthr = blockDim.x;
  for (int s = tid; s < S; s += nthr) {
    st.seg[s] = sm.seg[s];
    st.stamp[s] = sm.stamp[s];
    st.eis[s] = sm.eis[s];
  }
  for (int l = tid; l < L; l += nthr) st.slot_of[l] = sm.slot_of[l];
}

__global__ void __launch_bounds__(256) plan_kernel(uint8_t* state,
                                                   const int32_t* __restrict__ ids,
                                                   int num_ids, int32_t* __restrict__ emap) {
  extern __shared__ __align__(16) uint8_t plan_smem_raw[];
  sl::pdl_wait();
  sl::pdl_trigger();
  int S, G, L;
  StateView st = view_from_header(state, S, G, L);
  if (!plan_dims_ok(S, G, L)) {
    if (threadIdx.x == 0) st.hdr[SL_HDR_STATUS] = SL_ERR_INVALID;
    return;
  }
  PlanSmem sm = plan_smem(plan_smem_raw, S, G, L);
  const int tid = threadIdx.x, nthr = blockDim.x;
  load_plan_state(st, sm, S, G, L);
  __syncthreads();
  for (int p = tid; p < num_ids; p += nthr) {
    const int g = ids[p];
    if (g >= 0 && g < G) {
      atomicOr(&sm.bitmap[g >> 5], 1u << (g & 31));
      const int loc = sm.local_of[g];
      if (loc >= 0 && sm.slot_of[loc] < 0) sm.scal[0] = 1;
    }
  }
  __syncthreads();
  const int flags = st.hdr[SL_HDR_FLAGS];
  const int standing = st.hdr[SL_HDR_MAP_IS_STANDING];
  const bool lfu = (flags & SL_PLAN_LFU) != 0;
  // the counts are bumped before the FAST_HIT check, like the reference's hook
  if (lfu) lfu_bump(st, sm, S, G, L);
  if (tid == 0) {
    st.cnt[SL_CNT_GAPS] += 1;
    st.hdr[SL_HDR_STATUS] = SL_OK;
    st.hdr[SL_HDR_FILL_COUNT] = 0;
    st.hdr[SL_HDR_LAST_MISSES] = 0;
  }
  if ((flags & SL_PLAN_FAST_HIT) && standing && !sm.scal[0]) {
    if (tid == 0) st.cnt[SL_CNT_FAST_HITS] += 1;
    return;  // all-hit: no touches, no map write (offloader.py:2409-2424)
  }
  expand_uniques(sm, G);
  const uint32_t clock0 = renorm_stamps(st, sm, S);

  if (tid < 32) {
    const int lane = tid;
    uint32_t clock = clock0;
    int pcount = st.hdr[SL_HDR_PROTECTED_COUNT];
    int free_top = st.hdr[SL_HDR_FREE_TOP];
    const int cap = st.hdr[SL_HDR_PROTECTED_CAP];
    const int U = sm.scal[1];
    int nmiss = 0;
    unsigned long long hits = 0;
    // touch hits, collect misses (offloader.py:2427-2441)
    for (int i = 0; i < U; ++i) {
      const int g = sm.uniq[i];
      const int loc = sm.local_of[g];
      if (loc < 0) continue;  // owned by another rank
      const int slot = sm.slot_of[loc];
      if (slot < 0) {
        if (lane == 0 && nmiss <= kMaxSlots) sm.miss_loc[min(nmiss, S)] = loc;
        ++nmiss;
        continue;
      }
      ++hits;
      if (lane == 0) sm.claimed[slot] = 1;
      warp_touch(sm, S, slot, true, cap, lfu, pcount, clock);
      __syncwarp();
    }
    // acquire a slot per miss, ascending id order (offloader.py:2442-2465);
    // at most S misses can succeed, so S + 1 entries decide overflow
    int fc = 0;
    bool overflow = false;
    const int nm = min(nmiss, S + 1);
    for (int i = 0; i < nm; ++i) {
      const int loc = sm.miss_loc[i];
      const int slot = warp_acquire(sm, S, true, lfu, free_top, pcount);
      if (slot < 0) {
        overflow = true;
        break;
      }
      ++clock;
      if (lane == 0) {
        place_fill(st, sm, slot, loc, clock, lfu);
        st.fill_local[fc] = loc;
        st.fill_slot[fc] = slot;
      }
      ++fc;
      __syncwarp();
    }
    if (lane == 0) {
      st.hdr[SL_HDR_FREE_TOP] = free_top;
      st.hdr[SL_HDR_PROTECTED_COUNT] = pcount;
      st.hdr[SL_HDR_CLOCK] = static_cast<int32_t>(clock);
      st.hdr[SL_HDR_FILL_COUNT] = fc;
      st.hdr[SL_HDR_STATUS] = overflow ? SL_ERR_OVERFLOW : SL_OK;
      st.hdr[SL_HDR_LAST_MISSES] = overflow ? 0 : nmiss;
      st.cnt[SL_CNT_HITS] += hits;
      st.cnt[SL_CNT_FILLS] += fc;
      if (overflow) st.cnt[SL_CNT_OVERFLOWS] += 1;
      else st.cnt[SL_CNT_MISSES] += nmiss;
      sm.scal[2] = overflow ? -1 : nmiss;  // map-write decision
    }
  }
  __syncthreads();
  const int decision = sm.scal[2];
  store_plan_state(st, sm, S, L);
  if (decision >= 0 && (decision > 0 || !standing)) {
    // standing map: every resident expert -> its slot (offloader.py:2112-2123)
    for (int g = tid; g < G; g += nthr) emap[g] = -1;
    __syncthreads();
    for (int s = tid; s < S; s += nthr) {
      const int loc = sm.eis[s];
      if (loc >= 0) emap[st.global_of_local[loc]] = s;
    }
    if (tid == 0) st.hdr[SL_HDR_MAP_IS_STANDING] = 1;
  }
}

// Opt-in cross-layer prefetch (no counterpart in the reference): predicted
// owned experts that are not resident, ascending id, at most max_fills, each
// into the free list's next slot or the least recently used probation slot
// neither holding a predicted expert nor taken by this call (never protected
// or pinned), as a new probation entry. No touches, no LFU bump, no gap counters. The fills become the
// state's fill list (stream them with sl_stream_experts); the standing map,
// if standing, is rewritten.
__global__ void __launch_bounds__(256) prefetch_kernel(uint8_t* state,
                                                       const int32_t* __restrict__ ids,
                                                       int num_ids, int max_fills,
                                                       int32_t* __restrict__ emap) {
  extern __shared__ __align__(16) uint8_t plan_smem_raw[];
  sl::pdl_wait();
  sl::pdl_trigger();
  int S, G, L;
  StateView st = view_from_header(state, S, G, L);
  if (!plan_dims_ok(S, G, L)) {
    if (threadIdx.x == 0) st.hdr[SL_HDR_STATUS] = SL_ERR_INVALID;
    return;
  }
  PlanSmem sm = plan_smem(plan_smem_raw, S, G, L);
  const int tid = threadIdx.x, nthr = blockDim.x;
  load_plan_state(st, sm, S, G, L);
  __syncthreads();
  // predicted owned experts: residents keep their slots (claimed), the
  // others are the candidates
  for (int p = tid; p < num_ids; p += nthr) {
    const int g = ids[p];
    if (g >= 0 && g < G) {
      const int loc = sm.local_of[g];
      if (loc < 0) continue;
      const int slot = sm.slot_of[loc];
      if (slot < 0) atomicOr(&sm.bitmap[g >> 5], 1u << (g & 31));
      else sm.claimed[slot] = 1;
    }
  }
  if (tid == 0) {
    st.hdr[SL_HDR_STATUS] = SL_OK;
    st.hdr[SL_HDR_FILL_COUNT] = 0;
  }
  __syncthreads();
  expand_uniques(sm, G);
  const uint32_t clock0 = renorm_stamps(st, sm, S);
  if (tid < 32) {
    const int lane = tid;
    uint32_t clock = clock0;
    int free_top = st.hdr[SL_HDR_FREE_TOP];
    const int U = sm.scal[1];
    int fc = 0;
    for (int i = 0; i < U && fc < max_fills; ++i) {
      const int loc = sm.local_of[sm.uniq[i]];
      int slot = free_top > 0 ? sm.free_s[--free_top] : -1;
      if (slot < 0) slot = warp_lru(sm, S, SL_SEG_PROBATION, true);
      if (slot < 0) break;
      ++clock;
      if (lane == 0) {
        place_fill(st, sm, slot, loc, clock, false);
        st.fill_local[fc] = loc;
        st.fill_slot[fc] = slot;
      }
      ++fc;
      __syncwarp();
    }
    if (lane == 0) {
      st.hdr[SL_HDR_FREE_TOP] = free_top;
      st.hdr[SL_HDR_CLOCK] = static_cast<int32_t>(clock);
      st.hdr[SL_HDR_FILL_COUNT] = fc;
      st.hdr[SL_HDR_PREFETCH_FILLS] = fc;
      st.cnt[SL_CNT_PREFETCHES] += fc;
      st.cnt[SL_CNT_FILLS] += fc;
      sm.scal[2] = fc;
    }
  }
  __syncthreads();
  const int filled = sm.scal[2];
  store_plan_state(st, sm, S, L);
  if (filled > 0 && st.hdr[SL_HDR_MAP_IS_STANDING]) {
    __syncthreads();
    for (int g = tid; g < G; g += nthr) emap[g] = -1;
    __syncthreads();
    for (int s = tid; s < S; s += nthr) {
      const int loc = sm.eis[s];
      if (loc >= 0) emap[st.global_of_local[loc]] = s;
    }
  }
}

// One step beyond the envelope, planned in expert waves: the classic hook's
// run_moe (offloader.py:1452-1764) and _run_waves (1846-1933) with the
// reference's default switches, on a real step, no host round trip.
__global__ void __launch_bounds__(256) wave_plan_kernel(uint8_t* state,
                                                        const int32_t* __restrict__ ids,
                                                        int T, int topk, int decode_rows,
                                                        int32_t* __restrict__ emap,
                                                        int32_t* __restrict__ waves) {
  extern __shared__ __align__(16) uint8_t plan_smem_raw[];
  sl::pdl_wait();
  sl::pdl_trigger();
  int S, G, L;
  StateView st = view_from_header(state, S, G, L);
  const int MW = waves[SL_WAVE_HDR_MAX_WAVES];
  if (!plan_dims_ok(S, G, L) || waves[SL_WAVE_HDR_NUM_SLOTS] != S ||
      waves[SL_WAVE_HDR_GLOBAL_N] != G || MW < 1 || MW > kMaxWaves) {
    if (threadIdx.x == 0) {
      st.hdr[SL_HDR_STATUS] = SL_ERR_INVALID;
      waves[SL_WAVE_HDR_STATUS] = SL_ERR_INVALID;
    }
    return;
  }
  const WaveView wv = wave_view(waves, S, G, MW);
  PlanSmem sm = plan_smem(plan_smem_raw, S, G, L);
  const int tid = threadIdx.x, nthr = blockDim.x;
  const int num_ids = T * topk;
  // rows [0, decode_rows) are decodes (1578-1583); else the step is one class
  const bool per_token = decode_rows > 0 && decode_rows <= T;
  const int decode_ids = per_token ? decode_rows * topk : 0;
  load_plan_state(st, sm, S, G, L);
  for (int i = tid; i < MW * G; i += nthr) wv.map[i] = -1;
  for (int k = tid; k < MW; k += nthr) wv.count[k] = 0;
  __syncthreads();
  for (int p = tid; p < num_ids; p += nthr) {
    const int g = ids[p];
    if (g >= 0 && g < G) {
      atomicOr(&sm.bitmap[g >> 5], 1u << (g & 31));
      if (p < decode_ids) atomicOr(&sm.dbitmap[g >> 5], 1u << (g & 31));
    }
  }
  __syncthreads();
  expand_uniques(sm, G);
  // the owned working set (1613-1622) and the pinned slots (1636)
  for (int i = tid; i < sm.scal[1]; i += nthr)
    if (sm.local_of[sm.uniq[i]] >= 0) atomicAdd(&sm.scal[0], 1);
  for (int s = tid; s < S; s += nthr)
    if (sm.seg[s] == SL_SEG_PINNED) atomicAdd(&sm.scal[2], 1);
  __syncthreads();
  if (sm.scal[0] == 0) {
    // nothing owned: one wave with an empty map (1643-1645)
    for (int g = tid; g < G; g += nthr) emap[g] = -1;
    if (tid == 0) {
      st.hdr[SL_HDR_STATUS] = SL_OK;
      st.hdr[SL_HDR_FILL_COUNT] = 0;
      st.hdr[SL_HDR_LAST_MISSES] = 0;
      st.hdr[SL_HDR_MAP_IS_STANDING] = 0;
      wv.hdr[SL_WAVE_HDR_NUM_WAVES] = 1;
      wv.hdr[SL_WAVE_HDR_STATUS] = SL_OK;
      wv.hdr[SL_WAVE_HDR_LEFTOVER] = 0;
      wv.hdr[SL_WAVE_HDR_ROTATION] = 0;
    }
    return;
  }
  const bool lfu = (st.hdr[SL_HDR_FLAGS] & SL_PLAN_LFU) != 0;
  if (lfu) lfu_bump(st, sm, S, G, L);  // 1662-1663
  const uint32_t clock0 = renorm_stamps(st, sm, S);

  if (tid < 32) {
    const int lane = tid;
    uint32_t clock = clock0;
    int pcount = st.hdr[SL_HDR_PROTECTED_COUNT];
    int free_top = st.hdr[SL_HDR_FREE_TOP];
    const int cap = st.hdr[SL_HDR_PROTECTED_CAP];
    const int U = sm.scal[1], ws = sm.scal[0], npinned = sm.scal[2];
    // without a per-token signal the working-set heuristic classifies the
    // whole step (1629-1639); decode_rows < 0 forces scan (1628)
    const bool step_friendly = !per_token && decode_rows >= 0 && ws <= max(cap + npinned, 1);
    int nmiss = 0;
    unsigned long long hits = 0;
    // touch hits, collect misses (1672-1681); a hit is wave 0's
    for (int i = 0; i < U; ++i) {
      const int g = sm.uniq[i];
      const int loc = sm.local_of[g];
      if (loc < 0) continue;
      const bool dcls = per_token ? ((sm.dbitmap[g >> 5] >> (g & 31)) & 1u) != 0 : step_friendly;
      const int slot = sm.slot_of[loc];
      if (slot < 0) {
        // owned ids map to distinct local experts (checked at init): < L misses
        if (nmiss < L) {
          if (lane == 0) {
            sm.miss_loc[nmiss] = loc;
            sm.mcls[nmiss] = dcls;
          }
          ++nmiss;
        }
        continue;
      }
      ++hits;
      if (lane == 0) {
        sm.claimed[slot] = 1;
        wv.map[g] = slot;
      }
      warp_touch(sm, S, slot, dcls, cap, lfu, pcount, clock);
      __syncwarp();
    }
    // decode-class misses first, each class in ascending id order (1689);
    // the order goes where the unique ids were
    __syncwarp();
    if (lane == 0) {
      int o = 0;
      for (int i = 0; i < nmiss; ++i)
        if (sm.mcls[i]) sm.uniq[o++] = i;
      for (int i = 0; i < nmiss; ++i)
        if (!sm.mcls[i]) sm.uniq[o++] = i;
    }
    __syncwarp();
    // wave 0: a slot per miss until one finds none (1700-1708)
    int fc = 0;
    for (; fc < nmiss; ++fc) {
      const int mi = sm.uniq[fc];
      const int loc = sm.miss_loc[mi];
      const int slot = warp_acquire(sm, S, sm.mcls[mi] != 0, lfu, free_top, pcount);
      if (slot < 0) break;
      ++clock;
      if (lane == 0) {
        place_fill(st, sm, slot, loc, clock, lfu);
        st.fill_local[fc] = loc;
        st.fill_slot[fc] = slot;
        wv.loc[fc] = loc;
        wv.slot[fc] = slot;
        wv.map[st.global_of_local[loc]] = slot;
      }
      __syncwarp();
    }
    const int nleft = nmiss - fc;
    int nrot = 0;
    if (nleft > 0) {
      // rotation slots: the probation segment, least recently used first
      // (1856); stamps of live slots are unique, so ranks are positions
      int cnt = 0;
      for (int s = lane; s < S; s += 32) {
        if (sm.seg[s] != SL_SEG_PROBATION) continue;
        int r = 0;
        for (int q = 0; q < S; ++q) r += sm.seg[q] == SL_SEG_PROBATION && sm.stamp[q] < sm.stamp[s];
        sm.rot[r] = s;
        ++cnt;
      }
      nrot = static_cast<int>(__reduce_add_sync(0xffffffffu, static_cast<unsigned>(cnt)));
      __syncwarp();
    }
    if (lane == 0) {
      int nw = 1, assigned = 0;
      bool overflow = false;
      if (nleft > 0) {
        if (nrot == 0) {
          // no probation slot: the last max(1, S/4) unpinned slots (1857-1861)
          int np = 0;
          for (int s = 0; s < S; ++s) np += sm.seg[s] != SL_SEG_PINNED;
          const int take = min(np, max(1, S / 4));
          for (int s = 0, seen = 0; s < S; ++s) {
            if (sm.seg[s] == SL_SEG_PINNED) continue;
            if (seen++ >= np - take) sm.rot[nrot++] = s;
          }
        }
        // ping-pong groups rot[:half] and rot[half:] (a single group when
        // the second is empty, 1862-1867); each wave fills one group
        const int half = (nrot + 1) / 2;
        const bool pingpong = nrot - half > 0;
        overflow = nrot == 0;
        while (assigned < nleft && !overflow) {
          if (nw >= MW) {
            overflow = true;
            break;
          }
          const bool second = pingpong && ((nw - 1) & 1);
          const int* grp = second ? sm.rot + half : sm.rot;
          const int gn = second ? nrot - half : half;
          int c = 0;
          for (; c < gn && assigned < nleft; ++c, ++assigned) {
            const int loc = sm.miss_loc[sm.uniq[fc + assigned]];
            const int slot = grp[c];
            evict_to(sm, slot, loc);
            wv.loc[size_t(nw) * S + c] = loc;
            wv.slot[size_t(nw) * S + c] = slot;
            wv.map[size_t(nw) * G + st.global_of_local[loc]] = slot;
          }
          wv.count[nw] = c;
          ++nw;
        }
      }
      wv.count[0] = fc;
      st.hdr[SL_HDR_FREE_TOP] = free_top;
      st.hdr[SL_HDR_PROTECTED_COUNT] = pcount;
      st.hdr[SL_HDR_CLOCK] = static_cast<int32_t>(clock);
      st.hdr[SL_HDR_FILL_COUNT] = fc;
      st.hdr[SL_HDR_LAST_MISSES] = nmiss;
      st.hdr[SL_HDR_MAP_IS_STANDING] = 0;
      st.hdr[SL_HDR_STATUS] = overflow ? SL_ERR_OVERFLOW : SL_OK;
      st.cnt[SL_CNT_SCAN_STEPS] += 1;
      st.cnt[SL_CNT_SCAN_HITS] += hits;
      st.cnt[SL_CNT_SCAN_MISSES] += nmiss;
      st.cnt[SL_CNT_FILLS] += fc + assigned;
      st.cnt[SL_CNT_WAVES] += nw;
      if (overflow) st.cnt[SL_CNT_OVERFLOWS] += 1;
      wv.hdr[SL_WAVE_HDR_NUM_WAVES] = nw;
      wv.hdr[SL_WAVE_HDR_STATUS] = overflow ? SL_ERR_OVERFLOW : SL_OK;
      wv.hdr[SL_WAVE_HDR_LEFTOVER] = nleft;
      wv.hdr[SL_WAVE_HDR_ROTATION] = nrot;
      sm.scal[3] = nw;
    }
  }
  __syncthreads();
  store_plan_state(st, sm, S, L);
  // the expert map keeps the last wave's map (_write_map, 2083-2110)
  const int32_t* last = wv.map + size_t(sm.scal[3] - 1) * G;
  for (int g = tid; g < G; g += nthr) emap[g] = last[g];
}

// ---------------------------------------------------------------- streamer
constexpr int kMaxParams = 8;
constexpr int kChunkVec = 4096;  // 64 KiB per work unit
constexpr int kStreamThreads = 256;
constexpr int kStreamUnroll = 8;

struct StreamArgs {
  int n;
  const uint4* src[kMaxParams];
  uint4* dst[kMaxParams];
  unsigned long long vec[kMaxParams];     // 16-byte vectors per expert
  unsigned long long chunks[kMaxParams];  // work units per expert
  unsigned long long src_stride[kMaxParams];  // vectors between experts in the host store
  const int32_t* waves;  // a wave plan (sl_stream_wave), else the state's fill list
  int wave;
};

__device__ __forceinline__ uint4 ld_host_nc(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__global__ void __launch_bounds__(kStreamThreads) stream_kernel(const uint8_t* state,
                                                                StreamArgs a) {
  sl::pdl_wait();
  sl::pdl_trigger();
  int fc;
  const int32_t* fill_local;
  const int32_t* fill_slot;
  if (a.waves) {
    const int S = a.waves[SL_WAVE_HDR_NUM_SLOTS], G = a.waves[SL_WAVE_HDR_GLOBAL_N];
    const int MW = a.waves[SL_WAVE_HDR_MAX_WAVES];
    if (a.wave >= MW || a.wave >= a.waves[SL_WAVE_HDR_NUM_WAVES]) return;
    const WaveView wv = wave_view(const_cast<int32_t*>(a.waves), S, G, MW);
    fc = min(wv.count[a.wave], S);
    fill_local = wv.loc + size_t(a.wave) * S;
    fill_slot = wv.slot + size_t(a.wave) * S;
  } else {
    int S, G, L;
    const StateView st = view_from_header(const_cast<uint8_t*>(state), S, G, L);
    fc = st.hdr[SL_HDR_FILL_COUNT];
    fill_local = st.fill_local;
    fill_slot = st.fill_slot;
  }
  if (fc <= 0) return;
  unsigned long long per_fill = 0;
  for (int p = 0; p < a.n; ++p) per_fill += a.chunks[p];
  const unsigned long long total = per_fill * static_cast<unsigned long long>(fc);
  for (unsigned long long u = blockIdx.x; u < total; u += gridDim.x) {
    const int f = static_cast<int>(u / per_fill);
    unsigned long long r = u - static_cast<unsigned long long>(f) * per_fill;
    int p = 0;
    while (r >= a.chunks[p]) {
      r -= a.chunks[p];
      ++p;
    }
    const unsigned long long v0 = r * kChunkVec;
    const unsigned long long nvec = min(static_cast<unsigned long long>(kChunkVec), a.vec[p] - v0);
    const uint4* src =
        a.src[p] + static_cast<unsigned long long>(fill_local[f]) * a.src_stride[p] + v0;
    uint4* dst = a.dst[p] + static_cast<unsigned long long>(fill_slot[f]) * a.vec[p] + v0;
    for (unsigned long long base = 0; base < nvec; base += kStreamThreads * kStreamUnroll) {
      uint4 v[kStreamUnroll];
#pragma unroll
      for (int k = 0; k < kStreamUnroll; ++k) {
        const unsigned long long i = base + k * kStreamThreads + threadIdx.x;
        if (i < nvec) v[k] = ld_host_nc(src + i);
      }
#pragma unroll
      for (int k = 0; k < kStreamUnroll; ++k) {
        const unsigned long long i = base + k * kStreamThreads + threadIdx.x;
        if (i < nvec) dst[i] = v[k];
      }
    }
  }
}

int g_default_stream_ctas = 0;

}  // namespace

extern "C" size_t sl_slot_state_bytes(int num_slots, int global_n, int local_n) {
  if (num_slots <= 0 || global_n <= 0 || local_n <= 0) return 0;
  size_t off[13];
  state_layout(num_slots, global_n, local_n, off);
  return off[12];
}

extern "C" int sl_slot_state_offsets(int num_slots, int global_n, int local_n,
                                     size_t* offsets) {
  if (num_slots <= 0 || global_n <= 0 || local_n <= 0 || !offsets) return SL_ERR_INVALID;
  size_t off[13];
  state_layout(num_slots, global_n, local_n, off);
  for (int i = 0; i <= SL_STATE_NFIELDS; ++i) offsets[i] = off[i];
  return SL_OK;
}

extern "C" int sl_slot_state_init(void* state, int num_slots, int global_n, int local_n,
                                  int protected_cap, int flags, const int32_t* local_of,
                                  const int32_t* expert_in_slot, const uint8_t* seg,
                                  const int32_t* free_stack, int n_free,
                                  sl_stream_t stream) {
  const int S = num_slots, G = global_n, L = local_n;
  if (!state || S <= 0 || G <= 0 || L <= 0) return SL_ERR_INVALID;
  if (S > kMaxSlots || G > kMaxGlobal || L > kMaxGlobal ||
      plan_smem_bytes(S, G, L) > kPlanSmemBytes)
    return SL_ERR_UNSUPPORTED;
  if (!local_of || !expert_in_slot || !seg || n_free < 0 || n_free > S ||
      (n_free > 0 && !free_stack) || protected_cap < 0 || protected_cap > S)
    return SL_ERR_INVALID;
  size_t off[13];
  state_layout(S, G, L, off);
  uint8_t* img = static_cast<uint8_t*>(calloc(1, off[12]));
  if (!img) return SL_ERR_INVALID;
  int32_t* hdr = reinterpret_cast<int32_t*>(img + off[0]);
  int32_t* lof = reinterpret_cast<int32_t*>(img + off[2]);
  int32_t* gol = reinterpret_cast<int32_t*>(img + off[3]);
  int32_t* sof = reinterpret_cast<int32_t*>(img + off[4]);
  int32_t* eis = reinterpret_cast<int32_t*>(img + off[5]);
  uint8_t* sg = img + off[6];
  uint32_t* stamp = reinterpret_cast<uint32_t*>(img + off[7]);
  int32_t* fs = reinterpret_cast<int32_t*>(img + off[8]);
  int rc = SL_OK;
  for (int l = 0; l < L; ++l) gol[l] = -1, sof[l] = -1;
  for (int g = 0; g < G; ++g) {
    lof[g] = local_of[g];
    if (lof[g] >= L) rc = SL_ERR_INVALID;
    else if (lof[g] >= 0) {
      if (gol[lof[g]] >= 0) rc = SL_ERR_INVALID;  // two global ids, one local expert
      gol[lof[g]] = g;
    }
  }
  int pcount = 0;
  uint32_t clock = 0;
  for (int s = 0; s < S && rc == SL_OK; ++s) {
    eis[s] = expert_in_slot[s];
    sg[s] = seg[s];
    if (sg[s] > SL_SEG_PINNED || eis[s] >= L) rc = SL_ERR_INVALID;
    else if (eis[s] >= 0) {
      if (sg[s] == SL_SEG_FREE || sof[eis[s]] >= 0) rc = SL_ERR_INVALID;
      else sof[eis[s]] = s;
    } else if (sg[s] != SL_SEG_FREE) {
      rc = SL_ERR_INVALID;
    }
    if (sg[s] == SL_SEG_PROBATION || sg[s] == SL_SEG_PROTECTED) stamp[s] = ++clock;
    if (sg[s] == SL_SEG_PROTECTED) ++pcount;
  }
  for (int i = 0; i < n_free && rc == SL_OK; ++i) {
    fs[i] = free_stack[i];
    if (fs[i] < 0 || fs[i] >= S || seg[fs[i]] != SL_SEG_FREE) rc = SL_ERR_INVALID;
  }
  if (rc != SL_OK) {
    free(img);
    return rc;
  }
  hdr[SL_HDR_NUM_SLOTS] = S;
  hdr[SL_HDR_GLOBAL_N] = G;
  hdr[SL_HDR_LOCAL_N] = L;
  hdr[SL_HDR_PROTECTED_CAP] = protected_cap;
  hdr[SL_HDR_FLAGS] = flags;
  hdr[SL_HDR_MAP_IS_STANDING] = 0;
  hdr[SL_HDR_FREE_TOP] = n_free;
  hdr[SL_HDR_PROTECTED_COUNT] = pcount;
  hdr[SL_HDR_CLOCK] = static_cast<int32_t>(clock);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // pageable source: the copy is staged before this call returns
  cudaError_t e = cudaMemcpyAsync(state, img, off[12], cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  free(img);
  return e == cudaSuccess ? SL_OK : SL_ERR_CUDA;
}

extern "C" int sl_plan_slots(void* state, const int32_t* topk_ids, int num_ids,
                             int32_t* expert_map, sl_stream_t stream) {
  if (!state || !expert_map || num_ids < 0 || (num_ids > 0 && !topk_ids)) return SL_ERR_INVALID;
  static std::atomic<uint64_t> smem_set{0};
  SL_CUDA_TRY(sl::ensure_smem_limit(plan_kernel, kPlanSmemBytes, smem_set));
  SL_CUDA_TRY(sl::launch(plan_kernel, dim3(1), dim3(256), kPlanSmemBytes,
                         reinterpret_cast<cudaStream_t>(stream), static_cast<uint8_t*>(state),
                         topk_ids, num_ids, expert_map));
  return SL_OK;
}

namespace {

int make_stream_args(StreamArgs& a, int num_params, const void* const* host_src,
                     void* const* slot_dst, const size_t* bytes_per_expert,
                     const size_t* host_stride_bytes) {
  if (num_params <= 0 || num_params > kMaxParams || !host_src || !slot_dst || !bytes_per_expert)
    return SL_ERR_INVALID;
  memset(&a, 0, sizeof(a));
  a.n = num_params;
  for (int p = 0; p < num_params; ++p) {
    const size_t b = bytes_per_expert[p];
    if (b == 0 || (b & 15) || !host_src[p] || !slot_dst[p] ||
        ((reinterpret_cast<uintptr_t>(host_src[p]) | reinterpret_cast<uintptr_t>(slot_dst[p])) & 15))
      return SL_ERR_INVALID;
    a.src[p] = static_cast<const uint4*>(host_src[p]);
    a.dst[p] = static_cast<uint4*>(slot_dst[p]);
    a.vec[p] = b / 16;
    a.chunks[p] = (a.vec[p] + kChunkVec - 1) / kChunkVec;
    const size_t stride = host_stride_bytes ? host_stride_bytes[p] : b;
    if (stride < b || (stride & 15)) return SL_ERR_INVALID;
    a.src_stride[p] = stride / 16;
  }
  return SL_OK;
}

int launch_stream(const uint8_t* state, const StreamArgs& a, int num_ctas, sl_stream_t stream) {
  if (num_ctas <= 0) {
    if (g_default_stream_ctas <= 0) g_default_stream_ctas = 64;
    num_ctas = g_default_stream_ctas;
  }
  SL_CUDA_TRY(sl::launch(stream_kernel, dim3(num_ctas), dim3(kStreamThreads), 0,
                         reinterpret_cast<cudaStream_t>(stream), state, a));
  return SL_OK;
}

}  // namespace

extern "C" int sl_stream_experts_strided(const void* state, int num_params,
                                         const void* const* host_src, void* const* slot_dst,
                                         const size_t* bytes_per_expert,
                                         const size_t* host_stride_bytes, int num_ctas,
                                         sl_stream_t stream) {
  if (!state) return SL_ERR_INVALID;
  StreamArgs a;
  const int rc =
      make_stream_args(a, num_params, host_src, slot_dst, bytes_per_expert, host_stride_bytes);
  if (rc != SL_OK) return rc;
  return launch_stream(static_cast<const uint8_t*>(state), a, num_ctas, stream);
}

extern "C" int sl_stream_wave(const void* waves, int wave, int num_params,
                              const void* const* host_src, void* const* slot_dst,
                              const size_t* bytes_per_expert, const size_t* host_stride_bytes,
                              int num_ctas, sl_stream_t stream) {
  if (!waves || wave < 0 || (reinterpret_cast<uintptr_t>(waves) & 15)) return SL_ERR_INVALID;
  StreamArgs a;
  const int rc =
      make_stream_args(a, num_params, host_src, slot_dst, bytes_per_expert, host_stride_bytes);
  if (rc != SL_OK) return rc;
  a.waves = static_cast<const int32_t*>(waves);
  a.wave = wave;
  return launch_stream(nullptr, a, num_ctas, stream);
}

extern "C" size_t sl_wave_plan_bytes(int num_slots, int global_n, int max_waves) {
  if (num_slots <= 0 || global_n <= 0 || max_waves <= 0 || max_waves > kMaxWaves) return 0;
  size_t off[6];
  wave_layout(num_slots, global_n, max_waves, off);
  return off[5] * 4;
}

extern "C" int sl_wave_plan_offsets(int num_slots, int global_n, int max_waves,
                                    size_t* offsets) {
  if (num_slots <= 0 || global_n <= 0 || max_waves <= 0 || max_waves > kMaxWaves || !offsets)
    return SL_ERR_INVALID;
  size_t off[6];
  wave_layout(num_slots, global_n, max_waves, off);
  for (int i = 0; i <= SL_WAVE_NFIELDS; ++i) offsets[i] = off[i] * 4;
  return SL_OK;
}

extern "C" int sl_wave_plan_init(void* waves, int num_slots, int global_n, int max_waves,
                                 sl_stream_t stream) {
  const size_t bytes = sl_wave_plan_bytes(num_slots, global_n, max_waves);
  if (!waves || bytes == 0 || (reinterpret_cast<uintptr_t>(waves) & 15)) return SL_ERR_INVALID;
  int32_t* img = static_cast<int32_t*>(calloc(1, bytes));
  if (!img) return SL_ERR_INVALID;
  const WaveView wv = wave_view(img, num_slots, global_n, max_waves);
  wv.hdr[SL_WAVE_HDR_STATUS] = SL_OK;
  wv.hdr[SL_WAVE_HDR_MAX_WAVES] = max_waves;
  wv.hdr[SL_WAVE_HDR_GLOBAL_N] = global_n;
  wv.hdr[SL_WAVE_HDR_NUM_SLOTS] = num_slots;
  for (size_t i = 0; i < size_t(max_waves) * global_n; ++i) wv.map[i] = -1;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(waves, img, bytes, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  free(img);
  return e == cudaSuccess ? SL_OK : SL_ERR_CUDA;
}

extern "C" int sl_plan_waves(void* state, const int32_t* topk_ids, int num_tokens, int topk,
                             int decode_rows, int32_t* expert_map, void* waves,
                             sl_stream_t stream) {
  if (!state || !expert_map || !waves || num_tokens < 0 || topk <= 0 ||
      (num_tokens > 0 && !topk_ids) || static_cast<long long>(num_tokens) * topk > 0x7fffffffLL ||
      (reinterpret_cast<uintptr_t>(waves) & 15))
    return SL_ERR_INVALID;
  static std::atomic<uint64_t> smem_set{0};
  SL_CUDA_TRY(sl::ensure_smem_limit(wave_plan_kernel, kPlanSmemBytes, smem_set));
  SL_CUDA_TRY(sl::launch(wave_plan_kernel, dim3(1), dim3(256), kPlanSmemBytes,
                         reinterpret_cast<cudaStream_t>(stream), static_cast<uint8_t*>(state),
                         topk_ids, num_tokens, topk, decode_rows, expert_map,
                         static_cast<int32_t*>(waves)));
  return SL_OK;
}

extern "C" int sl_prefetch_slots(void* state, const int32_t* topk_ids, int num_ids,
                                 int max_fills, int32_t* expert_map, sl_stream_t stream) {
  if (!state || !expert_map || num_ids < 0 || (num_ids > 0 && !topk_ids) || max_fills < 0)
    return SL_ERR_INVALID;
  static std::atomic<uint64_t> smem_set{0};
  SL_CUDA_TRY(sl::ensure_smem_limit(prefetch_kernel, kPlanSmemBytes, smem_set));
  SL_CUDA_TRY(sl::launch(prefetch_kernel, dim3(1), dim3(256), kPlanSmemBytes,
                         reinterpret_cast<cudaStream_t>(stream), static_cast<uint8_t*>(state),
                         topk_ids, num_ids, max_fills, expert_map));
  return SL_OK;
}

extern "C" int sl_stream_experts(const void* state, int num_params,
                                 const void* const* host_src, void* const* slot_dst,
                                 const size_t* bytes_per_expert, int num_ctas,
                                 sl_stream_t stream) {
  return sl_stream_experts_strided(state, num_params, host_src, slot_dst, bytes_per_expert,
                                   nullptr, num_ctas, stream);
}

extern "C" int sl_host_alloc_mapped(size_t bytes, void** host_ptr) {
  if (!host_ptr || bytes == 0) return SL_ERR_INVALID;
  *host_ptr = nullptr;
  SL_CUDA_TRY(cudaHostAlloc(host_ptr, bytes, cudaHostAllocMapped | cudaHostAllocPortable));
  return SL_OK;
}

extern "C" int sl_host_free(void* host_ptr) {
  if (!host_ptr) return SL_OK;
  SL_CUDA_TRY(cudaFreeHost(host_ptr));
  return SL_OK;
}
