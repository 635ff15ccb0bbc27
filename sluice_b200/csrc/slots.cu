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
// the id bitmap, the sorted unique ids, and copies of every state array the
// sequential pass touches (so it never waits on global memory).
constexpr int kPlanSmemBytes = 72 * 1024;

struct PlanSmem {
  int* scal;          // [0] any_missing, [1] n_uniq, [2] decision
  uint32_t* bitmap;   // [W]
  uint32_t* word_base;
  int32_t* uniq;      // [G]
  int32_t* local_of;  // [G]
  int32_t* slot_of;   // [L]
  int32_t* miss_loc;  // [S + 1]
  uint32_t* stamp;    // [S]
  int32_t* eis;       // [S]
  int32_t* free_s;    // [S]
  uint8_t* seg;       // [S]
  uint8_t* claimed;   // [S]
  uint32_t* sfreq;    // [S] LFU count of each slot's expert
};

__host__ __device__ inline size_t plan_smem_bytes(int S, int G, int L) {
  const size_t W = (G + 31) / 32;
  return 16 + 8 * W + 8 * size_t(G) + 4 * size_t(L) + 4 * size_t(S + 1) + 16 * size_t(S) +
         2 * size_t(S) + 80;
}

__device__ inline PlanSmem plan_smem(uint8_t* base, int S, int G, int L) {
  PlanSmem m;
  const int W = (G + 31) / 32;
  uint8_t* p = base;
  auto take = [&](size_t bytes) {
    uint8_t* r = p;
    p += (bytes + 15) & ~size_t(15);
    return r;
  };
  m.scal = reinterpret_cast<int*>(take(16));
  m.bitmap = reinterpret_cast<uint32_t*>(take(4 * W));
  m.word_base = reinterpret_cast<uint32_t*>(take(4 * W));
  m.uniq = reinterpret_cast<int32_t*>(take(4 * size_t(G)));
  m.local_of = reinterpret_cast<int32_t*>(take(4 * size_t(G)));
  m.slot_of = reinterpret_cast<int32_t*>(take(4 * size_t(L)));
  m.miss_loc = reinterpret_cast<int32_t*>(take(4 * size_t(S + 1)));
  m.stamp = reinterpret_cast<uint32_t*>(take(4 * size_t(S)));
  m.eis = reinterpret_cast<int32_t*>(take(4 * size_t(S)));
  m.free_s = reinterpret_cast<int32_t*>(take(4 * size_t(S)));
  m.seg = take(S);
  m.claimed = take(S);
  m.sfreq = reinterpret_cast<uint32_t*>(take(4 * size_t(S)));
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

__global__ void __launch_bounds__(256) plan_kernel(uint8_t* state,
                                                   const int32_t* __restrict__ ids,
                                                   int num_ids, int32_t* __restrict__ emap) {
  extern __shared__ __align__(16) uint8_t plan_smem_raw[];
  sl::pdl_wait();
  sl::pdl_trigger();
  int S, G, L;
  StateView st = view_from_header(state, S, G, L);
  if (S <= 0 || S > kMaxSlots || G <= 0 || G > kMaxGlobal || L <= 0 || L > kMaxGlobal ||
      plan_smem_bytes(S, G, L) > kPlanSmemBytes) {
    if (threadIdx.x == 0) st.hdr[SL_HDR_STATUS] = SL_ERR_INVALID;
    return;
  }
  PlanSmem sm = plan_smem(plan_smem_raw, S, G, L);
  const int tid = threadIdx.x, nthr = blockDim.x;
  const int nwords = (G + 31) >> 5;
  for (int i = tid; i < nwords; i += nthr) sm.bitmap[i] = 0;
  for (int g = tid; g < G; g += nthr) sm.local_of[g] = st.local_of[g];
  for (int l = tid; l < L; l += nthr) sm.slot_of[l] = st.slot_of[l];
  for (int s = tid; s < S; s += nthr) {
    sm.seg[s] = st.seg[s];
    sm.stamp[s] = st.stamp[s];
    sm.eis[s] = st.eis[s];
    sm.free_s[s] = st.free_stack[s];
    sm.claimed[s] = 0;
  }
  if (tid == 0) sm.scal[0] = 0;
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
  if (lfu) {
    // _bump_freq: +1 per selected owned expert (each set bit once), then the
    // periodic halving; before the FAST_HIT check, like the reference's hook
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
  // sorted(set(ids)): expand the bitmap in ascending order
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
  // renumber stamps (order kept) before the clock can wrap
  uint32_t clock0 = static_cast<uint32_t>(st.hdr[SL_HDR_CLOCK]);
  if (clock0 > kClockRenorm) {
    __syncthreads();
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
      const uint8_t sg = sm.seg[slot];
      if (lane == 0) sm.claimed[slot] = 1;
      if (sg == SL_SEG_PROTECTED) {
        ++clock;
        if (lane == 0) sm.stamp[slot] = clock;
      } else if (sg == SL_SEG_PROBATION) {
        ++clock;
        if (cap > 0) {
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
      __syncwarp();
    }
    // acquire a slot per miss, ascending id order (offloader.py:2442-2465);
    // at most S misses can succeed, so S + 1 entries decide overflow
    int fc = 0;
    bool overflow = false;
    const int nm = min(nmiss, S + 1);
    for (int i = 0; i < nm; ++i) {
      const int loc = sm.miss_loc[i];
      int slot = -1;
      if (free_top > 0) {
        slot = sm.free_s[--free_top];
      } else {
        slot = warp_lru(sm, S, SL_SEG_PROBATION, true);
        if (slot < 0) {
          slot = lfu ? warp_lfu(sm, S, SL_SEG_PROTECTED, true)
                     : warp_lru(sm, S, SL_SEG_PROTECTED, true);
          if (slot >= 0) --pcount;
        }
      }
      if (slot < 0) {
        overflow = true;
        break;
      }
      ++clock;
      if (lane == 0) {
        const int old = sm.eis[slot];
        if (old >= 0) sm.slot_of[old] = -1;
        sm.eis[slot] = loc;
        sm.slot_of[loc] = slot;
        sm.seg[slot] = SL_SEG_PROBATION;
        sm.stamp[slot] = clock;
        sm.claimed[slot] = 1;
        if (lfu) sm.sfreq[slot] = st.freq[loc];
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
  for (int s = tid; s < S; s += nthr) {
    st.seg[s] = sm.seg[s];
    st.stamp[s] = sm.stamp[s];
    st.eis[s] = sm.eis[s];
  }
  for (int l = tid; l < L; l += nthr) st.slot_of[l] = sm.slot_of[l];
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
  int S, G, L;
  const StateView st = view_from_header(const_cast<uint8_t*>(state), S, G, L);
  const int fc = st.hdr[SL_HDR_FILL_COUNT];
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
        a.src[p] + static_cast<unsigned long long>(st.fill_local[f]) * a.src_stride[p] + v0;
    uint4* dst = a.dst[p] + static_cast<unsigned long long>(st.fill_slot[f]) * a.vec[p] + v0;
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
    else if (lof[g] >= 0) gol[lof[g]] = g;
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

extern "C" int sl_stream_experts_strided(const void* state, int num_params,
                                         const void* const* host_src, void* const* slot_dst,
                                         const size_t* bytes_per_expert,
                                         const size_t* host_stride_bytes, int num_ctas,
                                         sl_stream_t stream) {
  if (!state || num_params <= 0 || num_params > kMaxParams || !host_src || !slot_dst ||
      !bytes_per_expert)
    return SL_ERR_INVALID;
  StreamArgs a;
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
  if (num_ctas <= 0) {
    if (g_default_stream_ctas <= 0) g_default_stream_ctas = 64;
    num_ctas = g_default_stream_ctas;
  }
  SL_CUDA_TRY(sl::launch(stream_kernel, dim3(num_ctas), dim3(kStreamThreads), 0,
                         reinterpret_cast<cudaStream_t>(stream),
                         static_cast<const uint8_t*>(state), a));
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
