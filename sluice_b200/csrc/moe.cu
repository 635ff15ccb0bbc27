// fused_experts on sm_100a: token grouping through the expert map, two
// tcgen05 grouped GEMMs (gate/up with SwiGLU fused in the epilogue, then
// down), and the weighted top-k combine with the shared experts.
//
// Reference semantics (kfirtoledo/sluice calls vLLM for this step):
//   offloader.py:2590-2602  fused_experts(h, w13, w2, tw, ti, "silu",
//                           global_num_experts, expert_map) + shared MLP
//   vLLM fused_moe.py:1587-1869 (map lookup, -1 = skip, SiLU-and-mul,
//   routed weight, moe_sum), runner/moe_runner.py:350-366, 663-680 (routed
//   scaling, shared + routed).
//
// Data flow per call (all on the caller's stream, no host sync):
//   align    1 CTA: slot of every (token, choice) via the map, per-slot counts,
//            work items of BN tokens, row of every pair; gathers token rows
//            into X (rows grouped by item) and copies the shared rows.
//   gemm1    persistent, one CTA per SM: tile = (item, 128 intermediate
//            columns). TMA loads a 128x64 gate tile, a 128x64 up tile and the
//            BNx64 token tile per stage; two tcgen05.mma (M=128, N=BN, K=16
//            x4) into two TMEM accumulators; the epilogue computes
//            a = silu(g) * u per (column, token) and writes bf16 rows of A.
//   gemm2    same pipeline: tile = (item, 128 hidden rows), K = I; epilogue
//            writes bf16 z rows of Z.
//   combine  out[t] = shared(t) + scale * sum_j w[t,j] z(t,j).
// Warp roles in the GEMMs: warp 0 TMA producer, warp 1 MMA issuer (one
// thread) and TMEM owner, warps 2-5 epilogue (TMEM lanes 32*(warp%4)..).
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cudaTypedefs.h>
#include <mutex>
#include <stdlib.h>

#include "common.cuh"
#include "slot_state.cuh"

namespace {

constexpr int BM = 128;      // weight rows per tile
constexpr int BK = 64;       // K per stage: one 128-byte swizzle atom of bf16
constexpr int kThreads = 192;
constexpr int kMaxCode = 1056;  // slots + shared experts per call
constexpr int kMaxShared = 32;

// workspace header (int32 words)
enum {
  WS_STATUS = 0, WS_NUM_ITEMS = 1, WS_NUM_ROWS = 2, WS_NUM_HIT_ITEMS = 3, WS_SH_BASE = 8,
  WS_HDR_WORDS = 64
};

struct WsLayout {
  size_t items, pair_pos, x, act, z, gu, total;
  int max_items, max_rows;
};

__host__ __device__ inline size_t r256(size_t v) { return (v + 255) & ~size_t(255); }

// Token-tile width from the average tokens per used slot: decode steps (a few
// tokens per expert) use 16, prefill-sized steps 64 or 128 so each weight
// tile is reused across more tokens.
// fp8 keeps 16-token tiles below kF8WideMinAvg tokens per expert on average
// (decode steps: one item per expert). From there on it runs the wide-tile
// GEMMs: items of up to 192 tokens whose MMA width follows the item's token
// count, so an expert with a few dozen tokens is one item (its weights read
// once) that promotes only the columns it uses; gate/up is one GEMM over the
// 2I rows. (V3 experts: T=512 2.22 against 2.35 ms, T=1024 2.57 against
// 3.34 ms with 16-token tiles.)
constexpr int kF8WideBN = 192;
constexpr long kF8WideMinAvg = 16;
inline int choose_bn(int T, int topk, int S, bool fp8 = false) {
  const long P = static_cast<long>(T) * topk;
  const long used = P < S ? P : S;
  const long avg = used > 0 ? (P + used - 1) / used : 1;
  if (fp8) return avg < kF8WideMinAvg ? 16 : kF8WideBN;
  return avg <= 16 ? 16 : avg <= 64 ? 64 : 128;
}

// The wide fp8 path (`gu`) adds a bf16 buffer for the gate/up output rows
// [max_rows, 2I] ahead of the SwiGLU quantisation.
inline WsLayout ws_layout(int T, int topk, int H, int I, int S, int n_sh, int BN,
                          bool gu = false) {
  WsLayout w;
  const long P = static_cast<long>(T) * topk;
  const long routed = P / BN + (P < S ? P : S);
  const long shared = static_cast<long>(n_sh) * ((T + BN - 1) / BN);
  w.max_items = static_cast<int>(routed + shared + 1);
  w.max_rows = w.max_items * BN;
  size_t o = r256(WS_HDR_WORDS * 4);
  w.items = o; o += r256(sizeof(int4) * w.max_items);
  w.pair_pos = o; o += r256(sizeof(int32_t) * (P > 0 ? P : 1));
  w.x = o; o += r256(sizeof(__nv_bfloat16) * size_t(w.max_rows) * H);
  w.act = o; o += r256(sizeof(__nv_bfloat16) * size_t(w.max_rows) * I);
  w.z = o; o += r256(sizeof(__nv_bfloat16) * size_t(w.max_rows) * H);
  w.gu = o;
  if (gu) o += r256(sizeof(__nv_bfloat16) * size_t(w.max_rows) * 2 * I);
  w.total = o;
  return w;
}

// ------------------------------------------------------------------ align
__global__ void __launch_bounds__(1024) align_kernel(
    const int32_t* __restrict__ ids, int T, int topk, const int32_t* __restrict__ emap,
    int G, int S, int n_sh, int sh_t0, int sh_nt, int BN,
    const __nv_bfloat16* __restrict__ hs, int H,
    int32_t* __restrict__ ws_hdr, int4* __restrict__ items, int32_t* __restrict__ pair_pos,
    __nv_bfloat16* __restrict__ X, int max_items, const uint8_t* __restrict__ fill_state,
    int do_gather) {
  __shared__ int cnt[kMaxCode];
  __shared__ int ibase[kMaxCode + 1];
  __shared__ int cursor[kMaxCode];
  __shared__ int warp_sums[32];
  __shared__ uint32_t fill_bits[kMaxCode / 32 + 1];
  __shared__ int n_hit_items;
  __shared__ int grp_total;
  sl::pdl_wait();
  sl::pdl_trigger();
  const int tid = threadIdx.x, nthr = blockDim.x;
  const int P = T * topk;
  const int C = S + n_sh;
  for (int c = tid; c < C; c += nthr) {
    cnt[c] = c < S ? 0 : sh_nt;
    cursor[c] = 0;
  }
  __syncthreads();
  for (int p = tid; p < P; p += nthr) {
    const int g = ids[p];
    int s = -1;
    if (emap) {
      if (g >= 0 && g < G) s = emap[g];
    } else {
      s = g;
    }
    if (s < 0 || s >= S) s = -1;
    pair_pos[p] = s;
    if (s >= 0) atomicAdd(&cnt[s], 1);
  }
  __syncthreads();
  // codes whose slot is being filled by this gap's streamer go last, so the
  // items of already-resident experts form a prefix that can run first
  for (int w = tid; w <= kMaxCode / 32; w += nthr) fill_bits[w] = 0;
  __syncthreads();
  if (fill_state != nullptr) {
    int fS, fG, fL;
    const StateView fv = view_from_header(const_cast<uint8_t*>(fill_state), fS, fG, fL);
    const int nf = fv.hdr[SL_HDR_FILL_COUNT];
    for (int f = tid; f < nf; f += nthr) {
      const int slot = fv.fill_slot[f];
      if (slot >= 0 && slot < S) atomicOr(&fill_bits[slot >> 5], 1u << (slot & 31));
    }
  }
  __syncthreads();
  const int lane = tid & 31, warp = tid >> 5;
  const int c0 = 2 * tid, c1 = 2 * tid + 1;  // C <= kMaxCode <= 2 * blockDim
  auto is_fill = [&](int c) { return ((fill_bits[c >> 5] >> (c & 31)) & 1u) != 0; };
  auto tiles = [&](int c) { return (cnt[c] + BN - 1) / BN; };
  // block-wide exclusive scan; `total` receives the sum over the block
  auto block_scan = [&](int v, int& total) -> int {
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += n;
    }
    if (lane == 31) warp_sums[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      const int ws = warp_sums[lane];
      int wi = ws;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, wi, o);
        if (lane >= o) wi += n;
      }
      warp_sums[lane] = wi - ws;
      if (lane == 31) grp_total = wi;
    }
    __syncthreads();
    const int r = warp_sums[warp] + incl - v;
    total = grp_total;
    __syncthreads();
    return r;
  };
  // group 0: resident (hit) codes; group 1: codes being filled
  int n_hit = 0, n_fill = 0;
  {
    const int a0 = (c0 < C && !is_fill(c0)) ? tiles(c0) : 0;
    const int a1 = (c1 < C && !is_fill(c1)) ? tiles(c1) : 0;
    const int ex = block_scan(a0 + a1, n_hit);
    if (c0 < C && !is_fill(c0)) ibase[c0] = ex;
    if (c1 < C && !is_fill(c1)) ibase[c1] = ex + a0;
  }
  {
    const int a0 = (c0 < C && is_fill(c0)) ? tiles(c0) : 0;
    const int a1 = (c1 < C && is_fill(c1)) ? tiles(c1) : 0;
    const int ex = block_scan(a0 + a1, n_fill);
    if (c0 < C && is_fill(c0)) ibase[c0] = n_hit + ex;
    if (c1 < C && is_fill(c1)) ibase[c1] = n_hit + ex + a0;
  }
  if (tid == 0) {
    ibase[C] = n_hit + n_fill;
    n_hit_items = n_hit;
  }
  __syncthreads();
  const int n_items = ibase[C];
  if (tid == 0) {
    ws_hdr[WS_STATUS] = (n_items > max_items) ? SL_ERR_INVALID : SL_OK;
    ws_hdr[WS_NUM_ITEMS] = n_items <= max_items ? n_items : 0;
    ws_hdr[WS_NUM_ROWS] = n_items * BN;
    ws_hdr[WS_NUM_HIT_ITEMS] = n_items <= max_items ? n_hit_items : 0;
    for (int i = 0; i < n_sh; ++i) ws_hdr[WS_SH_BASE + i] = ibase[S + i] * BN;
  }
  if (n_items > max_items) return;
  for (int c = tid; c < C; c += nthr) {
    const int nt = (cnt[c] + BN - 1) / BN;
    for (int i = 0; i < nt; ++i)
      items[ibase[c] + i] = make_int4(c, (ibase[c] + i) * BN, min(BN, cnt[c] - i * BN), 0);
  }
  for (int p = tid; p < P; p += nthr) {
    const int s = pair_pos[p];
    if (s >= 0) pair_pos[p] = ibase[s] * BN + atomicAdd(&cursor[s], 1);
  }
  __syncthreads();
  if (!do_gather) return;  // large steps: gather_kernel copies the rows
  // gather token rows: routed pairs, then every token once per shared expert;
  // four independent 16-byte copies per thread per round
  const int vrow = H >> 3;
  const uint4* src = reinterpret_cast<const uint4*>(hs);
  uint4* dst = reinterpret_cast<uint4*>(X);
  const long n_routed = static_cast<long>(P) * vrow;
  const long n_total = n_routed + static_cast<long>(n_sh) * sh_nt * vrow;
  for (long q0 = tid; q0 < n_total; q0 += 4L * nthr) {
    uint4 v[4];
    long d[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const long q = q0 + static_cast<long>(u) * nthr;
      d[u] = -1;
      if (q < n_routed) {
        const int p = static_cast<int>(q / vrow), c = static_cast<int>(q % vrow);
        const int pos = pair_pos[p];
        if (pos >= 0) {
          d[u] = static_cast<long>(pos) * vrow + c;
          v[u] = src[static_cast<long>(p / topk) * vrow + c];
        }
      } else if (q < n_total) {
        const long r = (q - n_routed) / vrow;
        const int c = static_cast<int>((q - n_routed) % vrow);
        const int i = static_cast<int>(r / sh_nt), t = static_cast<int>(r % sh_nt);
        d[u] = static_cast<long>(ibase[S + i] * BN + t) * vrow + c;
        v[u] = src[static_cast<long>(sh_t0 + t) * vrow + c];
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (d[u] >= 0) dst[d[u]] = v[u];
  }
}

// Decode-sized steps (at most kSmallP pairs): the same grouping computed
// redundantly and deterministically by every CTA of a small grid (a pair's
// row is its rank among the earlier pairs of its slot), so each CTA can
// gather its share of the token rows at once; CTA 0 publishes the metadata.
constexpr int kSmallP = 1024;
constexpr int kAlignSmallThreads = 256;
constexpr int kAlignSmallCtas = 32;

__global__ void __launch_bounds__(kAlignSmallThreads) align_small_kernel(
    const int32_t* __restrict__ ids, int T, int topk, const int32_t* __restrict__ emap,
    int G, int S, int n_sh, int sh_t0, int sh_nt, int BN,
    const __nv_bfloat16* __restrict__ hs, int H,
    int32_t* __restrict__ ws_hdr, int4* __restrict__ items, int32_t* __restrict__ pair_pos,
    __nv_bfloat16* __restrict__ X, int max_items, const uint8_t* __restrict__ fill_state) {
  __shared__ int cnt[kMaxCode];
  __shared__ int ibase[kMaxCode];
  __shared__ int sp[kSmallP];    // slot of each pair, then its row
  __shared__ uint32_t fill_bits[kMaxCode / 32 + 1];
  __shared__ int warp_sums[kAlignSmallThreads / 32];
  __shared__ int grp_total;
  sl::pdl_wait();
  sl::pdl_trigger();
  const int tid = threadIdx.x, nthr = blockDim.x;
  const int lane = tid & 31, warp = tid >> 5, nwarps = nthr >> 5;
  const int P = T * topk;
  const int C = S + n_sh;
  for (int c = tid; c < C; c += nthr) cnt[c] = c < S ? 0 : sh_nt;
  for (int w = tid; w <= kMaxCode / 32; w += nthr) fill_bits[w] = 0;
  __syncthreads();
  for (int p = tid; p < P; p += nthr) {
    const int g = ids[p];
    int sl_ = -1;
    if (emap) {
      if (g >= 0 && g < G) sl_ = emap[g];
    } else {
      sl_ = g;
    }
    if (sl_ < 0 || sl_ >= S) sl_ = -1;
    sp[p] = sl_;
    if (sl_ >= 0) atomicAdd(&cnt[sl_], 1);
  }
  if (fill_state != nullptr) {
    int fS, fG, fL;
    const StateView fv = view_from_header(const_cast<uint8_t*>(fill_state), fS, fG, fL);
    const int nf = fv.hdr[SL_HDR_FILL_COUNT];
    for (int f = tid; f < nf; f += nthr) {
      const int slot = fv.fill_slot[f];
      if (slot >= 0 && slot < S) atomicOr(&fill_bits[slot >> 5], 1u << (slot & 31));
    }
  }
  __syncthreads();
  auto is_fill = [&](int c) { return ((fill_bits[c >> 5] >> (c & 31)) & 1u) != 0; };
  auto tiles = [&](int c) { return (cnt[c] + BN - 1) / BN; };
  auto block_scan = [&](int v, int& total) -> int {
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += n;
    }
    if (lane == 31) warp_sums[warp] = incl;
    __syncthreads();
    if (tid == 0) {
      int run = 0;
      for (int w = 0; w < nwarps; ++w) {
        const int t = warp_sums[w];
        warp_sums[w] = run;
        run += t;
      }
      grp_total = run;
    }
    __syncthreads();
    const int r = warp_sums[warp] + incl - v;
    total = grp_total;
    __syncthreads();
    return r;
  };
  // each thread owns a run of consecutive codes; resident codes first
  const int per = (C + nthr - 1) / nthr;
  const int c_lo = min(C, tid * per), c_hi = min(C, c_lo + per);
  int n_hit = 0, n_fill = 0;
  for (int group = 0; group < 2; ++group) {
    int local = 0;
    for (int c = c_lo; c < c_hi; ++c)
      if (is_fill(c) == (group == 1)) local += tiles(c);
    int total = 0;
    int run = block_scan(local, total) + (group == 1 ? n_hit : 0);
    for (int c = c_lo; c < c_hi; ++c)
      if (is_fill(c) == (group == 1)) {
        ibase[c] = run;
        run += tiles(c);
      }
    if (group == 0) n_hit = total;
    else n_fill = total;
  }
  __syncthreads();
  const int n_items = n_hit + n_fill;
  const bool lead = blockIdx.x == 0;
  if (lead && tid == 0) {
    ws_hdr[WS_STATUS] = (n_items > max_items) ? SL_ERR_INVALID : SL_OK;
    ws_hdr[WS_NUM_ITEMS] = n_items <= max_items ? n_items : 0;
    ws_hdr[WS_NUM_ROWS] = n_items * BN;
    ws_hdr[WS_NUM_HIT_ITEMS] = n_items <= max_items ? n_hit : 0;
    for (int i = 0; i < n_sh; ++i) ws_hdr[WS_SH_BASE + i] = ibase[S + i] * BN;
  }
  if (n_items > max_items) return;
  if (lead)
    for (int c = tid; c < C; c += nthr) {
      const int nt = tiles(c);
      for (int i = 0; i < nt; ++i)
        items[ibase[c] + i] = make_int4(c, (ibase[c] + i) * BN, min(BN, cnt[c] - i * BN), 0);
    }
  // row of each pair: rank among the earlier pairs of the same slot
  int myrow[kSmallP / kAlignSmallThreads];
#pragma unroll
  for (int k = 0; k < kSmallP / kAlignSmallThreads; ++k) {
    const int p = tid + k * nthr;
    myrow[k] = -1;
    if (p < P) {
      const int s0 = sp[p];
      if (s0 >= 0) {
        int r = 0;
        for (int q = 0; q < p; ++q) r += sp[q] == s0;
        myrow[k] = ibase[s0] * BN + r;
      }
    }
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < kSmallP / kAlignSmallThreads; ++k) {
    const int p = tid + k * nthr;
    if (p < P) {
      sp[p] = myrow[k];
      if (lead) pair_pos[p] = myrow[k];
    }
  }
  __syncthreads();
  if (X == nullptr) return;  // fp8 weights: a quantising gather follows
  // this CTA's share of the rows: routed pairs, then each shared expert's tokens
  const int vrow = H >> 3;
  const uint4* src = reinterpret_cast<const uint4*>(hs);
  uint4* dst = reinterpret_cast<uint4*>(X);
  const long n_routed = static_cast<long>(P) * vrow;
  const long n_total = n_routed + static_cast<long>(n_sh) * sh_nt * vrow;
  const long stride = static_cast<long>(gridDim.x) * nthr;
  for (long q0 = static_cast<long>(blockIdx.x) * nthr + tid; q0 < n_total; q0 += 4 * stride) {
    uint4 v[4];
    long d[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const long q = q0 + u * stride;
      d[u] = -1;
      if (q < n_routed) {
        const int p = static_cast<int>(q / vrow), c = static_cast<int>(q % vrow);
        const int pos = sp[p];
        if (pos >= 0) {
          d[u] = static_cast<long>(pos) * vrow + c;
          v[u] = src[static_cast<long>(p / topk) * vrow + c];
        }
      } else if (q < n_total) {
        const long r = (q - n_routed) / vrow;
        const int c = static_cast<int>((q - n_routed) % vrow);
        const int i = static_cast<int>(r / sh_nt), t = static_cast<int>(r % sh_nt);
        d[u] = static_cast<long>(ibase[S + i] * BN + t) * vrow + c;
        v[u] = src[static_cast<long>(sh_t0 + t) * vrow + c];
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (d[u] >= 0) dst[d[u]] = v[u];
  }
}

// Token-row gather for large steps, spread over the whole GPU: row of pair p
// (pair_pos) <- hidden row p / topk; shared experts' rows <- their tokens.
__global__ void __launch_bounds__(256) gather_kernel(
    const int32_t* __restrict__ ws_hdr, const int32_t* __restrict__ pair_pos, int P, int topk,
    int n_sh, int sh_t0, int sh_nt, const __nv_bfloat16* __restrict__ hs, int H,
    __nv_bfloat16* __restrict__ X) {
  sl::pdl_wait();
  sl::pdl_trigger();
  const int vrow = H >> 3;
  const uint4* src = reinterpret_cast<const uint4*>(hs);
  uint4* dst = reinterpret_cast<uint4*>(X);
  const long n_routed = static_cast<long>(P) * vrow;
  const long n_total = n_routed + static_cast<long>(n_sh) * sh_nt * vrow;
  const long stride = static_cast<long>(gridDim.x) * blockDim.x;
  for (long q0 = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; q0 < n_total;
       q0 += 4 * stride) {
    uint4 v[4];
    long d[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const long q = q0 + u * stride;
      d[u] = -1;
      if (q < n_routed) {
        const int p = static_cast<int>(q / vrow), c = static_cast<int>(q % vrow);
        const int pos = pair_pos[p];
        if (pos >= 0) {
          d[u] = static_cast<long>(pos) * vrow + c;
          v[u] = src[static_cast<long>(p / topk) * vrow + c];
        }
      } else if (q < n_total) {
        const long r = (q - n_routed) / vrow;
        const int c = static_cast<int>((q - n_routed) % vrow);
        const int i = static_cast<int>(r / sh_nt), t = static_cast<int>(r % sh_nt);
        d[u] = static_cast<long>(ws_hdr[WS_SH_BASE + i] + t) * vrow + c;
        v[u] = src[static_cast<long>(sh_t0 + t) * vrow + c];
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (d[u] >= 0) dst[d[u]] = v[u];
  }
}

// ------------------------------------------------------------- tcgen05 GEMM
// Weight-stationary orientation ("swap AB"): the weight rows are the MMA's M
// dimension (128), the tokens of one work item its N dimension (BN), K runs
// over the hidden (gate/up) or intermediate (down) dimension in 64-element
// stages of 128-byte swizzled tiles.
// GATED = true (gate/up GEMM): a 128-row A tile is 64 gate rows stacked on the
//   64 up rows of the same intermediate columns, so one M=128 MMA per K step
//   covers both; the epilogue pairs row r (gate) with row r + 64 (up) through
//   a small shared-memory exchange and writes silu(g) * u for 64 columns.
// GATED = false (down GEMM): 128 output rows per tile.
// The epilogue drains TMEM 16 token columns at a time, so BN can reach 128.
constexpr int kXchgStride = 17;  // padded fp32 row of the gate/up exchange

template <int BN, bool GATED>
struct TileShape {
  static constexpr int kRowsOut = GATED ? 64 : 128;   // output columns per tile
  static constexpr int kAccCols = BN;                 // TMEM columns per accumulator
  static constexpr int kTmemCols = (2 * BN) <= 32 ? 32 : (2 * BN) <= 64 ? 64
                                   : (2 * BN) <= 128 ? 128 : 256;
};

__device__ __forceinline__ void named_bar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// OR of a predicate over the four epilogue warps (named barrier 2), so they
// leave the tile loop together and never strand one another at barrier 1.
__device__ __forceinline__ bool epi_any(bool p) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred a, b;\n\t"
      "setp.ne.u32 a, %1, 0;\n\t"
      "bar.red.or.pred b, 2, 128, a;\n\t"
      "selp.u32 %0, 1, 0, b;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(p))
      : "memory");
  return r != 0;
}

// Drain one accumulator (TMEM lanes = the tile's 128 weight rows, columns =
// tokens) into bf16 output rows. Called by the four epilogue warps.
template <int BN, bool GATED>
__device__ __forceinline__ void epilogue_tile(uint32_t tmem_acc, int q, int lane, int4 it, int mt,
                                              __nv_bfloat16* __restrict__ out, int out_ld,
                                              float* xchg) {
  using TS = TileShape<BN, GATED>;
  const int row = q * 32 + lane;
  const uint32_t taddr = tmem_acc + (static_cast<uint32_t>(q * 32) << 16);
  for (int c0 = 0; c0 < BN; c0 += 16) {
    if (c0 >= it.z) break;  // it.z is the same for the four warps
    float v[16];
    sl::tmem_ld16(taddr + c0, v);
    if constexpr (GATED) {
      if (q >= 2) {
#pragma unroll
        for (int i = 0; i < 16; ++i) xchg[(row - 64) * kXchgStride + i] = v[i];
      }
      named_bar_sync(1, 128);
      if (q < 2) {
        __nv_bfloat16* dst = out + static_cast<size_t>(it.y + c0) * out_ld + mt * TS::kRowsOut + row;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          if (c0 + i < it.z) {
            // vLLM's torch-native chain: bf16 GEMM outputs, bf16 SiLU, bf16 mul
            const float g = sl::bf16_round(v[i]);
            const float u = sl::bf16_round(xchg[row * kXchgStride + i]);
            const float sg = sl::bf16_round(g / (1.0f + expf(-g)));
            dst[static_cast<size_t>(i) * out_ld] = __float2bfloat16(sg * u);
          }
        }
      }
      named_bar_sync(1, 128);  // the exchange rows are rewritten next chunk
    } else {
      __nv_bfloat16* dst = out + static_cast<size_t>(it.y + c0) * out_ld + mt * TS::kRowsOut + row;
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (c0 + i < it.z) dst[static_cast<size_t>(i) * out_ld] = __float2bfloat16(v[i]);
    }
  }
}

template <int BN, int STAGES, bool GATED>
struct GemmCfg {
  using TS = TileShape<BN, GATED>;
  static constexpr int kATile = BM * BK;  // bf16 elements
  static constexpr int kBTile = BN * BK;
  static constexpr int kStageBytes = (kATile + kBTile) * 2;
  static constexpr int kSmemBytes = STAGES * kStageBytes + 1024 /*align*/ + 512 /*bars*/ +
                                    64 * kXchgStride * 4;
};

template <int BN, int STAGES, bool GATED>
__global__ void __launch_bounds__(kThreads, 1) moe_gemm_kernel(
    const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_wsh,
    const __grid_constant__ CUtensorMap tm_b, const int32_t* __restrict__ ws_hdr,
    const int4* __restrict__ items, __nv_bfloat16* __restrict__ out, int S, int K,
    int M_total /* rows of one expert's weight block in this GEMM's view */,
    int out_ld, int32_t* __restrict__ status, int phase,
    const uint8_t* __restrict__ w_raw, const uint8_t* __restrict__ wsh_raw) {
  using Cfg = GemmCfg<BN, STAGES, GATED>;
  using TS = TileShape<BN, GATED>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  __nv_bfloat16* sA = reinterpret_cast<__nv_bfloat16*>(smem);  // [STAGES][BM*BK]
  __nv_bfloat16* sB = sA + STAGES * Cfg::kATile;               // [STAGES][BN*BK]
  float* xchg = reinterpret_cast<float*>(sB + STAGES * Cfg::kBTile);
  uint64_t* full = reinterpret_cast<uint64_t*>(xchg + 64 * kXchgStride);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* mma_done = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if constexpr (GATED) {
    // the work items, token rows and slot weights come from the launches
    // just before this one
    sl::pdl_wait();
    sl::pdl_trigger();
  }
  // down GEMM: items were written two launches back (align), so they may be
  // read before the wait; its B operand (the activations) may not.
  // phase -1: every item; 0: items of resident experts; 1: items of experts
  // streamed in by this gap (they follow the resident ones)
  const int m_tiles = M_total / TS::kRowsOut;
  const int num_items = ws_hdr[WS_NUM_ITEMS];
  const int n_hit = ws_hdr[WS_NUM_HIT_ITEMS];
  const int item_lo = phase == 1 ? n_hit : 0;
  const int item_hi = phase == 0 ? n_hit : num_items;
  const int num_tiles = (item_hi > item_lo ? item_hi - item_lo : 0) * m_tiles;
  const int k_blocks = K / BK;
  if (static_cast<int>(blockIdx.x) >= num_tiles) {
    // nothing for this CTA (e.g. phase 1 of a step without misses): leave
    // before any set-up; a dependent may start only once this grid has waited
    if constexpr (!GATED) {
      sl::pdl_wait();
      sl::pdl_trigger();
    }
    return;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      sl::mbar_init(&full[s], 1);
      sl::mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      sl::mbar_init(&tfull[a], 1);
      sl::mbar_init(&tempty[a], 4);
    }
    sl::mbar_init(mma_done, 1);
    *abort_flag = 0;
    sl::fence_barrier_init();
    sl::tma_prefetch_desc(&tm_w);
    sl::tma_prefetch_desc(&tm_wsh);
    sl::tma_prefetch_desc(&tm_b);
  }
  if (warp == 1) sl::tmem_alloc(tmem_slot, TS::kTmemCols);
  sl::tc_fence_before();
  __syncthreads();
  sl::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    if (sl::elect_one()) {
      const uint64_t pol_w = sl::policy_evict_first();
      const uint64_t pol_b = sl::policy_evict_last();
      int stage = 0;
      uint32_t phase_bit = 0;
      uint32_t issued_phase_mask = 0;  // stages with a TMA in flight at exit
      bool ok = true;
      // Down GEMM under PDL: the first STAGES weight tiles are fetched before
      // waiting on the gate/up GEMM; their activation tiles follow the wait.
      bool waited = GATED;
      int pend_n = 0;
      int pend_stage[STAGES], pend_kb[STAGES], pend_row[STAGES];
      if constexpr (!GATED) {
        // While the gate/up GEMM finishes, ask L2 for this CTA's first tile:
        // its 128 weight rows over all of K are one contiguous range.
        const int4 it = items[item_lo + blockIdx.x / m_tiles];
        const int e = it.x >= S ? it.x - S : it.x;
        const uint8_t* src = (it.x >= S ? wsh_raw : w_raw) +
                             (static_cast<size_t>(e) * M_total + (blockIdx.x % m_tiles) * BM) *
                                 static_cast<size_t>(K) * 2;
        const size_t bytes = static_cast<size_t>(BM) * K * 2;
        for (size_t o = 0; o < bytes; o += 65536)
          sl::prefetch_l2(src + o, static_cast<uint32_t>(bytes - o < 65536 ? bytes - o : 65536));
      }
      auto flush = [&]() {
        sl::pdl_wait();
        sl::pdl_trigger();
        waited = true;
        for (int i = 0; i < pend_n; ++i)
          sl::tma_load_2d(sB + pend_stage[i] * Cfg::kBTile, &tm_b, &full[pend_stage[i]],
                          pend_kb[i] * BK, pend_row[i], pol_b);
        pend_n = 0;
      };
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int4 it = items[item_lo + tile / m_tiles];
        const int mt = tile % m_tiles;
        const bool sh = it.x >= S;
        const CUtensorMap* tw = sh ? &tm_wsh : &tm_w;
        const int e = sh ? it.x - S : it.x;
        // weight rows in the 2-D view [experts * rows, K]
        const int row0 = GATED ? e * 2 * M_total + mt * 64 : e * M_total + mt * BM;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (*abort_flag || !sl::mbar_wait(&empty[stage], phase_bit ^ 1)) {
            ok = false;
            break;
          }
          sl::mbar_arrive_expect_tx(&full[stage], Cfg::kStageBytes);
          __nv_bfloat16* a0 = sA + stage * Cfg::kATile;
          sl::tma_load_2d(a0, tw, &full[stage], kb * BK, row0, pol_w);
          if constexpr (GATED)  // up rows under the gate rows
            sl::tma_load_2d(a0 + 64 * BK, tw, &full[stage], kb * BK, row0 + M_total, pol_w);
          if (waited) {
            sl::tma_load_2d(sB + stage * Cfg::kBTile, &tm_b, &full[stage], kb * BK, it.y, pol_b);
          } else {
            pend_stage[pend_n] = stage;
            pend_kb[pend_n] = kb;
            pend_row[pend_n] = it.y;
            if (++pend_n == STAGES) flush();
          }
          issued_phase_mask = (issued_phase_mask & ~(1u << stage)) | (phase_bit << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase_bit ^= 1;
          }
        }
      }
      if (!waited) flush();
      if (!ok) {
        atomicExch(status, SL_ERR_TIMEOUT);
        *abort_flag = 1;
        // let every TMA issued into shared memory land before the CTA exits
        for (int s = 0; s < STAGES; ++s)
          (void)sl::mbar_wait(&full[s], (issued_phase_mask >> s) & 1u);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------- MMA issuer
    if (sl::elect_one()) {
      constexpr uint32_t idesc = sl::umma_idesc_bf16(BM, BN);
      int stage = 0;
      uint32_t phase_bit = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        if (*abort_flag || !sl::mbar_wait(&tempty[acc], acc_phase ^ 1)) {
          ok = false;
          break;
        }
        sl::tc_fence_after();
        const uint32_t d0 = tmem_base + acc * TS::kAccCols;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (*abort_flag || !sl::mbar_wait(&full[stage], phase_bit)) {
            ok = false;
            break;
          }
          sl::tc_fence_after();
          const uint32_t a_addr = sl::smem_u32(sA + stage * Cfg::kATile);
          const uint32_t b_addr = sl::smem_u32(sB + stage * Cfg::kBTile);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            sl::umma_bf16(d0, sl::umma_desc_sw128(a_addr + k * 32),
                          sl::umma_desc_sw128(b_addr + k * 32), idesc, (kb | k) != 0);
          sl::umma_commit(&empty[stage]);  // stage free once these MMAs finish
          if (++stage == STAGES) {
            stage = 0;
            phase_bit ^= 1;
          }
        }
        if (!ok) break;
        sl::umma_commit(&tfull[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      if (!ok) {
        atomicExch(status, SL_ERR_TIMEOUT);
        *abort_flag = 1;
      }
      // every MMA this thread issued has completed before TMEM is freed
      sl::umma_commit(mma_done);
      (void)sl::mbar_wait(mma_done, 0);
    }
  } else {
    // --------------------------------------------------------- epilogue
    const int q = warp & 3;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      const bool ok = !*abort_flag && sl::mbar_wait(&tfull[acc], acc_phase);
      // the four epilogue warps must agree before the exchange barriers
      if (epi_any(!ok)) {
        atomicExch(status, SL_ERR_TIMEOUT);
        *abort_flag = 1;
        break;
      }
      sl::tc_fence_after();
      const int4 it = items[item_lo + tile / m_tiles];
      epilogue_tile<BN, GATED>(tmem_base + acc * TS::kAccCols, q, lane, it, tile % m_tiles,
                               out, out_ld, xchg);
      sl::tc_fence_before();
      __syncwarp();
      if (lane == 0) sl::mbar_arrive(&tempty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }
  sl::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    sl::tc_fence_after();
    sl::tmem_dealloc(tmem_base, TS::kTmemCols);
  }
}

// ------------------------------------------------------ fp8 (w8a8) GEMM
// vLLM's block-fp8 MoE arithmetic (fused_experts with use_fp8_w8a8 and
// block_shape [128, 128]): the activations are quantised per row and
// 128-column group to e4m3 with an fp32 scale (amax / 448), the weights are
// e4m3 with fp32 128x128 block scales. Each 128-wide K block is one tcgen05
// kind::f8f6f4 accumulation (4 MMAs of K = 32) into a TMEM buffer, which the
// promotion warps scale by (weight block scale x the token's group scale)
// and add into fp32 registers.
// GATED (gate/up GEMM): a tile is 128 gate rows and the 128 up rows of the
//   same intermediate columns (two M=128 MMAs per K step into two TMEM
//   column ranges), so SwiGLU is thread-local and one tile covers one
//   128-column group of the intermediate: the epilogue quantises it per
//   token for the down GEMM (group amax across the four lane quadrants).
// !GATED (down GEMM): 128 output rows per tile, bf16 out per (pair, row).
// Roles: warp 0 TMA producer, warp 1 MMA issuer + TMEM owner, warps 2.. the
// promotion / epilogue warps: four per group of 16 token columns (the
// 16-token tiles of decode-sized steps: four). Each promotion warp reads its K
// block's accumulator columns from TMEM and scales them with its own
// products of weight block scale and token group scale, so no barrier is
// taken inside the K loop.
constexpr int F8_BK = 128;  // K per stage: one scale block, one 128-byte swizzle row
constexpr int kF8MaxKBlocks = 64;  // K <= 8192: a tile's weight scales fit in shared memory

template <int BN, bool GATED>
struct F8Cfg {
  // promotion warps: four per column group of 16 tokens (one per TMEM lane
  // quadrant), so a warp's accumulators stay at 16 (down) or 32 (gate/up)
  // registers and the warps of a K block work without waiting on each other
  static constexpr int kNP = 4 * (BN / 16);
  static constexpr int kGroups = kNP / 4;                // token-column groups
  static constexpr int kThreads = 64 + 32 * kNP;
  static constexpr int kCW = BN / kGroups;               // token columns per promotion warp
  static constexpr int kATiles = GATED ? 2 : 1;          // 128-row weight tiles per stage
  static constexpr int kABytes = kATiles * 128 * F8_BK;
  static constexpr int kBBytes = BN * F8_BK;
  static constexpr int kStageBytes = kABytes + kBBytes;   // multiple of 1024
  static constexpr int kTxBytes = kStageBytes + BN * 4;   // + the tokens' group scales
  static constexpr int kAccCols = kATiles * BN;          // TMEM columns per buffer
  static constexpr int kNB = kAccCols * 4 <= 512 ? 4 : 2;
  static constexpr int kTmemUsed = kNB * kAccCols;
  static constexpr int kTmemCols = kTmemUsed <= 32 ? 32 : kTmemUsed <= 64 ? 64
                                   : kTmemUsed <= 128 ? 128 : kTmemUsed <= 256 ? 256 : 512;
  // + amax exchange [4][BN], the tile's weight block scales
  // [column groups][gate, up][64 K blocks]
  static constexpr int kFixed = 1024 /*align*/ + 4 * BN * 4 + kGroups * 128 * 4 +
                                1024 /*barriers*/;
  static constexpr int kStagesRaw = (220 * 1024 - kFixed) / (kStageBytes + BN * 4);
  static constexpr int kStages = kStagesRaw > 12 ? 12 : kStagesRaw;
  static constexpr int kSmemBytes = kStages * (kStageBytes + BN * 4) + kFixed;
};

__device__ __forceinline__ uint32_t e4m3x4(float a, float b, float c, float d) {
  const __nv_fp8x2_storage_t lo =
      __nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
  const __nv_fp8x2_storage_t hi =
      __nv_cvt_float2_to_fp8x2(make_float2(c, d), __NV_SATFINITE, __NV_E4M3);
  return static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
}

// vLLM's per_token_group_quant_fp8 (fp8_utils.py, _per_token_group_quant_fp8):
// scale = max(amax, 1e-10) * (1 / 448), q = clamp(x / scale, -448, 448) ->
// e4m3 (round to nearest even).
constexpr float kF8Max = 448.0f;
__device__ __forceinline__ float group_scale(float amax) {
  return fmaxf(amax, 1e-10f) * (1.0f / kF8Max);
}
__device__ __forceinline__ float q_clamp(float x, float scale) {
  return fminf(fmaxf(__fdiv_rn(x, scale), -kF8Max), kF8Max);
}

// Token rows for the fp8 GEMMs, quantised per 128-column group once per token
// and written to every row that token feeds: its routed pairs' rows
// (pair_pos[t * topk + j]) and, for tokens in [sh_t0, sh_t0 + sh_nt), its
// row of each shared expert. A warp takes four groups of one token at a time
// (four independent 8-byte loads per lane in flight): Xq [max_rows, H] e4m3
// codes, Xs [H/128, max_rows] fp32 scales.
constexpr int kQuantGroups = 4;

__global__ void __launch_bounds__(256) gather_quant_kernel(
    const int32_t* __restrict__ ws_hdr, const int32_t* __restrict__ pair_pos, int T, int topk,
    int n_sh, int sh_t0, int sh_nt, const __nv_bfloat16* __restrict__ hs, int H,
    uint8_t* __restrict__ Xq, float* __restrict__ Xs, int max_rows) {
  sl::pdl_wait();
  sl::pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int G = H / 128;
  const int GU = (G + kQuantGroups - 1) / kQuantGroups;  // units per token
  const long n_units = static_cast<long>(T) * GU;
  const long nwarps = static_cast<long>(gridDim.x) * (blockDim.x >> 5);
  for (long u = static_cast<long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
       u < n_units; u += nwarps) {
    const int tok = static_cast<int>(u / GU), kb0 = static_cast<int>(u % GU) * kQuantGroups;
    uint2 raw[kQuantGroups];
#pragma unroll
    for (int g = 0; g < kQuantGroups; ++g)
      if (kb0 + g < G)
        raw[g] = *reinterpret_cast<const uint2*>(hs + static_cast<size_t>(tok) * H +
                                                 (kb0 + g) * 128 + lane * 4);
    uint32_t code[kQuantGroups];
    float scl[kQuantGroups];
#pragma unroll
    for (int g = 0; g < kQuantGroups; ++g) {
      if (kb0 + g >= G) break;
      const float2 f01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw[g].x));
      const float2 f23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw[g].y));
      float m = fmaxf(fmaxf(fabsf(f01.x), fabsf(f01.y)), fmaxf(fabsf(f23.x), fabsf(f23.y)));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      scl[g] = group_scale(m);
      code[g] = e4m3x4(q_clamp(f01.x, scl[g]), q_clamp(f01.y, scl[g]), q_clamp(f23.x, scl[g]),
                       q_clamp(f23.y, scl[g]));
    }
    const bool shared_tok = n_sh > 0 && tok >= sh_t0 && tok < sh_t0 + sh_nt;
    const int n_dst = topk + (shared_tok ? n_sh : 0);
    for (int j = 0; j < n_dst; ++j) {
      const int pos = j < topk ? pair_pos[static_cast<size_t>(tok) * topk + j]
                               : ws_hdr[WS_SH_BASE + (j - topk)] + (tok - sh_t0);
      if (pos < 0) continue;  // the same for the whole warp
#pragma unroll
      for (int g = 0; g < kQuantGroups; ++g) {
        const int kb = kb0 + g;
        if (kb >= G) break;
        *reinterpret_cast<uint32_t*>(Xq + static_cast<size_t>(pos) * H + kb * 128 + lane * 4) =
            code[g];
        if (lane == 0) Xs[static_cast<size_t>(kb) * max_rows + pos] = scl[g];
      }
    }
  }
}

template <int BN, bool GATED>
__global__ void __launch_bounds__(F8Cfg<BN, GATED>::kThreads, 1) moe_gemm_f8_kernel(
    const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_wsh,
    const __grid_constant__ CUtensorMap tm_b, const float* __restrict__ b_scale,
    const float* __restrict__ w_scale, const float* __restrict__ wsh_scale,
    const int32_t* __restrict__ ws_hdr, const int4* __restrict__ items,
    uint8_t* __restrict__ out_q, float* __restrict__ out_s, __nv_bfloat16* __restrict__ out_z,
    int S, int K, int M_total, int max_rows, int32_t* __restrict__ status, int phase,
    const uint8_t* __restrict__ w_raw, const uint8_t* __restrict__ wsh_raw) {
  using Cfg = F8Cfg<BN, GATED>;
  constexpr int ST = Cfg::kStages;
  constexpr int NB = Cfg::kNB;
  constexpr int CW = Cfg::kCW;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sAB = smem;                                                  // [ST][A | B]
  float* sS = reinterpret_cast<float*>(sAB + ST * Cfg::kStageBytes);    // [ST][BN]
  float* red = sS + ST * BN;                                            // [4][BN]
  float* wsc = red + 4 * BN;                                            // [groups][2][64]
  uint64_t* full = reinterpret_cast<uint64_t*>(wsc + Cfg::kGroups * 128);
  uint64_t* empty = full + ST;
  uint64_t* tfull = empty + ST;
  uint64_t* tempty = tfull + NB;
  uint64_t* mma_done = tempty + NB;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if constexpr (GATED) {
    sl::pdl_wait();
    sl::pdl_trigger();
  }
  // down GEMM: the items were written two launches back, so they may be read
  // before the wait; its B operand (the quantised activations) may not
  const int m_tiles = M_total / 128;
  const int num_items = ws_hdr[WS_NUM_ITEMS];
  const int n_hit = ws_hdr[WS_NUM_HIT_ITEMS];
  const int item_lo = phase == 1 ? n_hit : 0;
  const int item_hi = phase == 0 ? n_hit : num_items;
  const int num_tiles = (item_hi > item_lo ? item_hi - item_lo : 0) * m_tiles;
  const int k_blocks = K / F8_BK;
  const int kscale = K / 128;
  if (static_cast<int>(blockIdx.x) >= num_tiles) {
    if constexpr (!GATED) {
      sl::pdl_wait();
      sl::pdl_trigger();
    }
    return;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) {
      sl::mbar_init(&full[s], 1);
      sl::mbar_init(&empty[s], 1 + Cfg::kNP);  // the MMAs' commit + every promotion warp
    }
    for (int b = 0; b < NB; ++b) {
      sl::mbar_init(&tfull[b], 1);
      sl::mbar_init(&tempty[b], Cfg::kNP);
    }
    sl::mbar_init(mma_done, 1);
    *abort_flag = 0;
    sl::fence_barrier_init();
    sl::tma_prefetch_desc(&tm_w);
    sl::tma_prefetch_desc(&tm_wsh);
    sl::tma_prefetch_desc(&tm_b);
  }
  if (warp == 1) sl::tmem_alloc(tmem_slot, Cfg::kTmemCols);
  sl::tc_fence_before();
  __syncthreads();
  sl::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    if (sl::elect_one()) {
      const uint64_t pol_w = sl::policy_evict_first();
      const uint64_t pol_b = sl::policy_evict_last();
      int s = 0;
      uint32_t ph = 0;
      uint32_t issued_mask = 0;
      bool ok = true;
      bool waited = GATED;
      int pend_n = 0;
      int pend_s[ST], pend_kb[ST], pend_row[ST];
      if constexpr (!GATED) {
        // While the gate/up GEMM finishes, ask L2 for this CTA's first tile:
        // its 128 e4m3 weight rows over all of K are one contiguous range.
        const int4 it = items[item_lo + blockIdx.x / m_tiles];
        const int e = it.x >= S ? it.x - S : it.x;
        const uint8_t* src = (it.x >= S ? wsh_raw : w_raw) +
                             (static_cast<size_t>(e) * M_total + (blockIdx.x % m_tiles) * 128) *
                                 static_cast<size_t>(K);
        const size_t bytes = static_cast<size_t>(128) * K;
        for (size_t o = 0; o < bytes; o += 65536)
          sl::prefetch_l2(src + o, static_cast<uint32_t>(bytes - o < 65536 ? bytes - o : 65536));
      }
      auto load_b = [&](int st, int kb, int row) {
        sl::tma_load_2d(sAB + st * Cfg::kStageBytes + Cfg::kABytes, &tm_b, &full[st],
                        kb * F8_BK, row, pol_b);
        sl::bulk_load(sS + st * BN, b_scale + static_cast<size_t>(kb) * max_rows + row, BN * 4,
                      &full[st]);
      };
      auto flush = [&]() {
        sl::pdl_wait();
        sl::pdl_trigger();
        waited = true;
        for (int i = 0; i < pend_n; ++i) load_b(pend_s[i], pend_kb[i], pend_row[i]);
        pend_n = 0;
      };
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int4 it = items[item_lo + tile / m_tiles];
        const int mt = tile % m_tiles;
        const bool sh = it.x >= S;
        const CUtensorMap* tw = sh ? &tm_wsh : &tm_w;
        const int e = sh ? it.x - S : it.x;
        // weight rows in the 2-D view [experts * rows, K]
        const int row0 = GATED ? e * 2 * M_total + mt * 128 : e * M_total + mt * 128;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (*abort_flag || !sl::mbar_wait(&empty[s], ph ^ 1)) {
            ok = false;
            break;
          }
          sl::mbar_arrive_expect_tx(&full[s], Cfg::kTxBytes);
          uint8_t* a0 = sAB + s * Cfg::kStageBytes;
          sl::tma_load_2d(a0, tw, &full[s], kb * F8_BK, row0, pol_w);
          if constexpr (GATED)  // the up rows of the same intermediate columns
            sl::tma_load_2d(a0 + 128 * F8_BK, tw, &full[s], kb * F8_BK, row0 + M_total, pol_w);
          if (waited) {
            load_b(s, kb, it.y);
          } else {
            pend_s[pend_n] = s;
            pend_kb[pend_n] = kb;
            pend_row[pend_n] = it.y;
            if (++pend_n == ST) flush();
          }
          issued_mask = (issued_mask & ~(1u << s)) | (ph << s);
          if (++s == ST) {
            s = 0;
            ph ^= 1;
          }
        }
      }
      if (!waited) flush();
      if (!ok) {
        atomicExch(status, SL_ERR_TIMEOUT);
        *abort_flag = 1;
        for (int i = 0; i < ST; ++i) (void)sl::mbar_wait(&full[i], (issued_mask >> i) & 1u);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------- MMA issuer
    if (sl::elect_one()) {
      constexpr uint32_t idesc = sl::umma_idesc_e4m3(128, BN);
      int s = 0, b = 0;
      uint32_t ph = 0, bph = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (*abort_flag || !sl::mbar_wait(&tempty[b], bph ^ 1) ||
              !sl::mbar_wait(&full[s], ph)) {
            ok = false;
            break;
          }
          sl::tc_fence_after();
          const uint32_t d0 = tmem_base + b * Cfg::kAccCols;
          const uint32_t a_addr = sl::smem_u32(sAB + s * Cfg::kStageBytes);
          const uint32_t b_addr = a_addr + Cfg::kABytes;
#pragma unroll
          for (int k = 0; k < F8_BK / 32; ++k)
            sl::umma_e4m3(d0, sl::umma_desc_sw128(a_addr + k * 32),
                          sl::umma_desc_sw128(b_addr + k * 32), idesc, k != 0);
          if constexpr (GATED) {
#pragma unroll
            for (int k = 0; k < F8_BK / 32; ++k)
              sl::umma_e4m3(d0 + BN, sl::umma_desc_sw128(a_addr + 128 * F8_BK + k * 32),
                            sl::umma_desc_sw128(b_addr + k * 32), idesc, k != 0);
          }
          sl::umma_commit(&empty[s]);
          sl::umma_commit(&tfull[b]);
          if (++s == ST) {
            s = 0;
            ph ^= 1;
          }
          if (++b == NB) {
            b = 0;
            bph ^= 1;
          }
        }
      }
      if (!ok) {
        atomicExch(status, SL_ERR_TIMEOUT);
        *abort_flag = 1;
      }
      sl::umma_commit(mma_done);
      (void)sl::mbar_wait(mma_done, 0);
    }
  } else {
    // ------------------------------------------- promotion and epilogue
    const int pw = warp - 2;
    const int q = warp & 3;           // TMEM lane quadrant of this warp
    const int cg = pw >> 2;           // token-column group
    const int c0 = cg * CW;
    const int row = q * 32 + lane;    // weight row within the 128-row tile
    int s = 0, b = 0;
    uint32_t ph = 0, bph = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      const int4 it = items[item_lo + tile / m_tiles];
      const int mt = tile % m_tiles;
      const bool sh = it.x >= S;
      const int e = sh ? it.x - S : it.x;
      const float* scale = sh ? wsh_scale : w_scale;
      // this tile's weight block-scale rows (block row mt; up rows at I/128 + mt)
      const int srows = GATED ? 2 * (M_total / 128) : M_total / 128;
      const float* sc_g = scale + (static_cast<size_t>(e) * srows + mt) * kscale;
      const float* sc_u = GATED ? sc_g + static_cast<size_t>(M_total / 128) * kscale : sc_g;
      const int gt = (pw & 3) * 32 + lane;  // thread index within the column group
      // the tile's weight block scales into shared memory, once per tile
      float* my_wsc = wsc + cg * 128;        // [gate, up][64]
      if (gt < kscale) {
        my_wsc[gt] = __ldg(sc_g + gt);
        if constexpr (GATED) my_wsc[64 + gt] = __ldg(sc_u + gt);
      }
      named_bar_sync(1 + cg, 128);
      // accumulators as column pairs: the K-block update is packed fp32x2
      // arithmetic (two columns per instruction, each lane an IEEE fma)
      float2 acc_g2[CW / 2], acc_u2[GATED ? CW / 2 : 1];
#pragma unroll
      for (int i = 0; i < CW / 2; ++i) acc_g2[i] = make_float2(0.f, 0.f);
      if constexpr (GATED) {
#pragma unroll
        for (int i = 0; i < CW / 2; ++i) acc_u2[i] = make_float2(0.f, 0.f);
      }
      for (int kb = 0; kb < k_blocks; ++kb) {
        // the accumulator of this K block, then the stage's token scales
        // (landed with the stage; its full phase stays complete until this
        // warp releases the stage)
        ok = ok && !*abort_flag && sl::mbar_wait(&tfull[b], bph) && sl::mbar_wait(&full[s], ph);
        if (ok) {
          sl::tc_fence_after();
          const uint32_t taddr = tmem_base + b * Cfg::kAccCols +
                                 (static_cast<uint32_t>(q * 32) << 16) + c0;
          uint32_t vg[CW], vu[GATED ? CW : 1];
#pragma unroll
          for (int cc = 0; cc < CW; cc += 16)
            sl::tmem_ld16_nowait(taddr + cc, *reinterpret_cast<uint32_t(*)[16]>(vg + cc));
          if constexpr (GATED) {
#pragma unroll
            for (int cc = 0; cc < CW; cc += 16)
              sl::tmem_ld16_nowait(taddr + BN + cc, *reinterpret_cast<uint32_t(*)[16]>(vu + cc));
          }
          // while the loads are in flight: this K block's weight block scale
          // and the stage's token group scales of this warp's columns
          const float wg = my_wsc[kb];
          const float wu = GATED ? my_wsc[64 + kb] : 0.f;
          // combined scales of this warp's column pairs: weight block scale x
          // token group scale
          float2 cg2[CW / 2], cu2[GATED ? CW / 2 : 1];
#pragma unroll
          for (int i = 0; i < CW / 2; i += 2) {
            const float4 t4 = *reinterpret_cast<const float4*>(sS + s * BN + c0 + 2 * i);
            cg2[i] = __fmul2_rn(make_float2(wg, wg), make_float2(t4.x, t4.y));
            cg2[i + 1] = __fmul2_rn(make_float2(wg, wg), make_float2(t4.z, t4.w));
            if constexpr (GATED) {
              cu2[i] = __fmul2_rn(make_float2(wu, wu), make_float2(t4.x, t4.y));
              cu2[i + 1] = __fmul2_rn(make_float2(wu, wu), make_float2(t4.z, t4.w));
            }
          }
#pragma unroll
          for (int cc = 0; cc < CW; cc += 16)
            sl::tmem_wait_ld(*reinterpret_cast<uint32_t(*)[16]>(vg + cc));
          if constexpr (GATED) {
#pragma unroll
            for (int cc = 0; cc < CW; cc += 16)
              sl::tmem_wait_ld(*reinterpret_cast<uint32_t(*)[16]>(vu + cc));
          }
#pragma unroll
          for (int i = 0; i < CW / 2; ++i) {
            acc_g2[i] = __ffma2_rn(
                make_float2(__uint_as_float(vg[2 * i]), __uint_as_float(vg[2 * i + 1])), cg2[i],
                acc_g2[i]);
            if constexpr (GATED)
              acc_u2[i] = __ffma2_rn(
                  make_float2(__uint_as_float(vu[2 * i]), __uint_as_float(vu[2 * i + 1])),
                  cu2[i], acc_u2[i]);
          }
          sl::tc_fence_before();
        }
        __syncwarp();
        if (ok && lane == 0) {
          sl::mbar_arrive(&tempty[b]);
          sl::mbar_arrive(&empty[s]);
        }
        if (++s == ST) {
          s = 0;
          ph ^= 1;
        }
        if (++b == NB) {
          b = 0;
          bph ^= 1;
        }
      }
      if (!ok) {
        atomicExch(status, SL_ERR_TIMEOUT);
        *abort_flag = 1;
      }
      float acc_g[CW], acc_u[GATED ? CW : 1];
#pragma unroll
      for (int i = 0; i < CW / 2; ++i) {
        acc_g[2 * i] = acc_g2[i].x;
        acc_g[2 * i + 1] = acc_g2[i].y;
        if constexpr (GATED) {
          acc_u[2 * i] = acc_u2[i].x;
          acc_u[2 * i + 1] = acc_u2[i].y;
        }
      }
      if constexpr (GATED) {
        // every warp of this column group runs the same tiles and barriers
        // (a failed wait above only skips work), so the barriers cannot strand
        // one of them
        const int f = mt * 128 + row;  // intermediate column of this thread
#pragma unroll
        for (int i = 0; i < CW; ++i) {
          // vLLM's chain: bf16 GEMM outputs, bf16 SiLU, bf16 product
          const float g = sl::bf16_round(acc_g[i]);
          const float u = sl::bf16_round(acc_u[i]);
          const float sg = sl::bf16_round(g / (1.0f + expf(-g)));
          acc_g[i] = sl::bf16_round(sg * u);
          float m = fabsf(acc_g[i]);
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
          if (lane == 0) red[q * BN + c0 + i] = m;
        }
        named_bar_sync(1 + cg, 128);
#pragma unroll
        for (int i = 0; i < CW; ++i) {
          const int c = c0 + i;
          const float m = fmaxf(fmaxf(red[c], red[BN + c]), fmaxf(red[2 * BN + c], red[3 * BN + c]));
          const float sc = group_scale(m);
          if (ok && c < it.z) {
            const __nv_fp8_storage_t v = __nv_cvt_float_to_fp8(q_clamp(acc_g[i], sc),
                                                               __NV_SATFINITE, __NV_E4M3);
            out_q[static_cast<size_t>(it.y + c) * M_total + f] = v;
            if (row == 0) out_s[static_cast<size_t>(mt) * max_rows + it.y + c] = sc;
          }
        }
        named_bar_sync(1 + cg, 128);  // red is rewritten by the next tile
      } else {
        const int h = mt * 128 + row;
#pragma unroll
        for (int i = 0; i < CW; ++i)
          if (ok && c0 + i < it.z)
            out_z[static_cast<size_t>(it.y + c0 + i) * M_total + h] = __float2bfloat16(acc_g[i]);
      }
    }
  }
  sl::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    sl::tc_fence_after();
    sl::tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}


// ------------------------------------------- fp8 GEMM, wide token tiles
// Steps with many tokens per expert (prefill-sized) use items of up to 192
// tokens: the MMA is M=128 weight rows x N=round16(item tokens) x K=32, so
// each weight tile staged in shared memory feeds up to three times the
// multiply-adds of a 64-token tile and the per-K-block promotion work per
// multiply-add is amortised over 64 columns per warp. Gate/up is one plain
// GEMM over the 2I rows of w13 (bf16 g and u rows written to a buffer, then
// swiglu_quant_kernel applies vLLM's SiLU-and-mul chain and quantises per
// 128-column group), so a tile keeps one accumulator per (row, token).
// Roles: warp 0 TMA producer, warp 1 MMA issuer + TMEM owner, warps 2..13
// promotion: four lane quadrants x three column groups; group g owns the
// 16-column chunks g, g+3, g+6, g+9, so an item of n tokens costs each warp
// at most ceil(n/48) TMEM round trips per K block (a warp whose chunks hold
// no token of the item only releases the buffers). 14
// warps keep four per SM sub-partition, so a thread may hold 128 registers
// (64 fp32 accumulators plus one 16-column TMEM load).
// The token tile is loaded as 32-row boxes, only those that hold tokens.
constexpr int F8W_BN = 192;
static_assert(F8W_BN == kF8WideBN, "wide fp8 token tile");
constexpr int F8W_CW = 64;                             // token columns per promotion warp
constexpr int F8W_NG = F8W_BN / F8W_CW;                // column groups (chunk stride)
constexpr int F8W_NP = 4 * F8W_NG;
constexpr int F8W_THREADS = 64 + 32 * F8W_NP;
constexpr int F8W_ABYTES = 128 * F8_BK;                // one 128x128 e4m3 weight tile
constexpr int F8W_BBYTES = F8W_BN * F8_BK;             // up to 192 token rows
constexpr int F8W_STAGE = F8W_ABYTES + F8W_BBYTES;     // multiple of 1024
constexpr int F8W_STAGES = 5;
constexpr int F8W_NB = 2;                              // TMEM accumulator buffers
constexpr int F8W_TSTRIDE = 256;                       // TMEM columns per buffer
constexpr int F8W_SMEM = 1024 /*align*/ + F8W_STAGES * (F8W_STAGE + F8W_BN * 4) +
                         512 /*barriers*/;

__global__ void __launch_bounds__(F8W_THREADS, 1) moe_gemm_f8w_kernel(
    const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_wsh,
    const __grid_constant__ CUtensorMap tm_b, const float* __restrict__ b_scale,
    const float* __restrict__ w_scale, const float* __restrict__ wsh_scale,
    const int32_t* __restrict__ ws_hdr, const int4* __restrict__ items,
    __nv_bfloat16* __restrict__ out, int S, int K, int M_total, int max_rows,
    int32_t* __restrict__ status, int phase) {
  constexpr int ST = F8W_STAGES;
  constexpr int NB = F8W_NB;
  constexpr int CW = F8W_CW;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sAB = smem;                                                 // [ST][A | B]
  float* sS = reinterpret_cast<float*>(sAB + ST * F8W_STAGE);          // [ST][BN]
  uint64_t* full = reinterpret_cast<uint64_t*>(sS + ST * F8W_BN);
  uint64_t* empty = full + ST;
  uint64_t* tfull = empty + ST;
  uint64_t* tempty = tfull + NB;
  uint64_t* mma_done = tempty + NB;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // both wide GEMMs read what the kernel just before them wrote (the
  // quantised token rows, the quantised SwiGLU rows)
  sl::pdl_wait();
  sl::pdl_trigger();
  const int m_tiles = M_total / 128;
  const int num_items = ws_hdr[WS_NUM_ITEMS];
  const int n_hit = ws_hdr[WS_NUM_HIT_ITEMS];
  const int item_lo = phase == 1 ? n_hit : 0;
  const int item_hi = phase == 0 ? n_hit : num_items;
  const int num_tiles = (item_hi > item_lo ? item_hi - item_lo : 0) * m_tiles;
  const int k_blocks = K / F8_BK;
  const int kscale = K / 128;
  if (static_cast<int>(blockIdx.x) >= num_tiles) return;
  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) {
      sl::mbar_init(&full[s], 1);
      sl::mbar_init(&empty[s], 1 + F8W_NP);  // the MMAs' commit + every promotion warp
    }
    for (int b = 0; b < NB; ++b) {
      sl::mbar_init(&tfull[b], 1);
      sl::mbar_init(&tempty[b], F8W_NP);
    }
    sl::mbar_init(mma_done, 1);
    *abort_flag = 0;
    sl::fence_barrier_init();
    sl::tma_prefetch_desc(&tm_w);
    sl::tma_prefetch_desc(&tm_wsh);
    sl::tma_prefetch_desc(&tm_b);
  }
  if (warp == 1) sl::tmem_alloc(tmem_slot, NB * F8W_TSTRIDE);
  sl::tc_fence_before();
  __syncthreads();
  sl::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    if (sl::elect_one()) {
      int s = 0;
      uint32_t ph = 0;
      uint32_t issued_mask = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int4 it = items[item_lo + tile / m_tiles];
        const int mt = tile % m_tiles;
        const bool sh = it.x >= S;
        const CUtensorMap* tw = sh ? &tm_wsh : &tm_w;
        const int e = sh ? it.x - S : it.x;
        const int row0 = e * M_total + mt * 128;  // weight rows in the view [experts * rows, K]
        const int nb32 = (it.z + 31) >> 5;        // 32-row boxes holding tokens
        const uint32_t tx = F8W_ABYTES + nb32 * (32 * F8_BK + 32 * 4);
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (*abort_flag || !sl::mbar_wait(&empty[s], ph ^ 1)) {
            ok = false;
            break;
          }
          sl::mbar_arrive_expect_tx(&full[s], tx);
          uint8_t* a0 = sAB + s * F8W_STAGE;
          sl::tma_load_2d_nohint(a0, tw, &full[s], kb * F8_BK, row0);
          for (int j = 0; j < nb32; ++j)
            sl::tma_load_2d_nohint(a0 + F8W_ABYTES + j * 32 * F8_BK, &tm_b, &full[s], kb * F8_BK,
                                   it.y + 32 * j);
          sl::bulk_load(sS + s * F8W_BN, b_scale + static_cast<size_t>(kb) * max_rows + it.y,
                        nb32 * 32 * 4, &full[s]);
          issued_mask = (issued_mask & ~(1u << s)) | (ph << s);
          if (++s == ST) {
            s = 0;
            ph ^= 1;
          }
        }
      }
      if (!ok) {
        atomicExch(status, SL_ERR_TIMEOUT);
        *abort_flag = 1;
        for (int i = 0; i < ST; ++i) (void)sl::mbar_wait(&full[i], (issued_mask >> i) & 1u);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------- MMA issuer
    if (sl::elect_one()) {
      int s = 0, b = 0;
      uint32_t ph = 0, bph = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int n = items[item_lo + tile / m_tiles].z;
        const uint32_t idesc = sl::umma_idesc_e4m3(128, (n + 15) & ~15);
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (*abort_flag || !sl::mbar_wait(&tempty[b], bph ^ 1) ||
              !sl::mbar_wait(&full[s], ph)) {
            ok = false;
            break;
          }
          sl::tc_fence_after();
          const uint32_t d0 = tmem_base + b * F8W_TSTRIDE;
          const uint32_t a_addr = sl::smem_u32(sAB + s * F8W_STAGE);
          const uint32_t b_addr = a_addr + F8W_ABYTES;
#pragma unroll
          for (int k = 0; k < F8_BK / 32; ++k)
            sl::umma_e4m3(d0, sl::umma_desc_sw128(a_addr + k * 32),
                          sl::umma_desc_sw128(b_addr + k * 32), idesc, k != 0);
          sl::umma_commit(&empty[s]);
          sl::umma_commit(&tfull[b]);
          if (++s == ST) {
            s = 0;
            ph ^= 1;
          }
          if (++b == NB) {
            b = 0;
            bph ^= 1;
          }
        }
      }
      if (!ok) {
        atomicExch(status, SL_ERR_TIMEOUT);
        *abort_flag = 1;
      }
      sl::umma_commit(mma_done);
      (void)sl::mbar_wait(mma_done, 0);
    }
  } else {
    // ------------------------------------------- promotion and epilogue
    const int q = warp & 3;               // TMEM lane quadrant of this warp
    const int c0 = ((warp - 2) >> 2) * 16;  // first token column of this warp
    const int row = q * 32 + lane;        // weight row within the 128-row tile
    int s = 0, b = 0;
    uint32_t ph = 0, bph = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      const int4 it = items[item_lo + tile / m_tiles];
      const int mt = tile % m_tiles;
      const bool sh = it.x >= S;
      const int e = sh ? it.x - S : it.x;
      const float* sc = (sh ? wsh_scale : w_scale) +
                        (static_cast<size_t>(e) * m_tiles + mt) * kscale;
      const int ncol = it.z - c0;  // <= 0: no chunk of this warp holds a token
      float2 acc[CW / 2];
#pragma unroll
      for (int i = 0; i < CW / 2; ++i) acc[i] = make_float2(0.f, 0.f);
      float wsk_next = __ldg(sc);  // weight block scales, one K block ahead
      for (int kb = 0; kb < k_blocks; ++kb) {
        const float wsk = wsk_next;  // weight block scale of this K block
        if (kb + 1 < k_blocks) wsk_next = __ldg(sc + kb + 1);
        ok = ok && !*abort_flag && sl::mbar_wait(&tfull[b], bph) && sl::mbar_wait(&full[s], ph);
        if (ok && ncol > 0) {
          sl::tc_fence_after();
          const uint32_t taddr = tmem_base + b * F8W_TSTRIDE +
                                 (static_cast<uint32_t>(q * 32) << 16) + c0;
          const float* ts = sS + s * F8W_BN + c0;
#pragma unroll
          for (int j = 0; j < CW / 16; ++j) {
            const int cc = j * 16 * F8W_NG;  // chunk j of this warp: columns c0 + cc ..
            if (cc < ncol) {
              uint32_t v[16];
              sl::tmem_ld16_nowait(taddr + cc, v);
              sl::tmem_wait_ld(v);
              // acc += v x (weight block scale x token group scale), per column
#pragma unroll
              for (int i = 0; i < 8; i += 2) {
                const float4 t4 = *reinterpret_cast<const float4*>(ts + cc + 2 * i);
                const float2 c01 = __fmul2_rn(make_float2(wsk, wsk), make_float2(t4.x, t4.y));
                const float2 c23 = __fmul2_rn(make_float2(wsk, wsk), make_float2(t4.z, t4.w));
                acc[j * 8 + i] = __ffma2_rn(
                    make_float2(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1])), c01,
                    acc[j * 8 + i]);
                acc[j * 8 + i + 1] = __ffma2_rn(
                    make_float2(__uint_as_float(v[2 * i + 2]), __uint_as_float(v[2 * i + 3])),
                    c23, acc[j * 8 + i + 1]);
              }
            }
          }
          sl::tc_fence_before();
        }
        __syncwarp();
        if (ok && lane == 0) {
          sl::mbar_arrive(&tempty[b]);
          sl::mbar_arrive(&empty[s]);
        }
        if (++s == ST) {
          s = 0;
          ph ^= 1;
        }
        if (++b == NB) {
          b = 0;
          bph ^= 1;
        }
      }
      if (!ok) {
        atomicExch(status, SL_ERR_TIMEOUT);
        *abort_flag = 1;
      }
      if (ok && ncol > 0) {
        __nv_bfloat16* dst = out + static_cast<size_t>(it.y + c0) * M_total + mt * 128 + row;
#pragma unroll
        for (int i = 0; i < CW / 2; ++i) {
          const int col = (i >> 3) * 16 * F8W_NG + 2 * (i & 7);  // column of acc[i].x - c0
          if (col < ncol) dst[static_cast<size_t>(col) * M_total] = __float2bfloat16(acc[i].x);
          if (col + 1 < ncol)
            dst[static_cast<size_t>(col + 1) * M_total] = __float2bfloat16(acc[i].y);
        }
      }
    }
  }
  sl::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    sl::tc_fence_after();
    sl::tmem_dealloc(tmem_base, NB * F8W_TSTRIDE);
  }
}

// vLLM's SiLU-and-mul chain on the wide gate/up output (bf16 g and u rows of
// 2I columns), then per-token 128-column quantisation for the down GEMM: the
// same arithmetic as the narrow gate/up epilogue. A warp takes four groups of
// one row (eight independent 8-byte loads per lane in flight).
__global__ void __launch_bounds__(256) swiglu_quant_kernel(
    const int32_t* __restrict__ ws_hdr, const int4* __restrict__ items, int BN,
    const __nv_bfloat16* __restrict__ gu, int I, uint8_t* __restrict__ Aq,
    float* __restrict__ As, int max_rows, int phase) {
  sl::pdl_wait();
  sl::pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int num_items = ws_hdr[WS_NUM_ITEMS];
  const int n_hit = ws_hdr[WS_NUM_HIT_ITEMS];
  const int item_lo = phase == 1 ? n_hit : 0;
  const int item_hi = phase == 0 ? n_hit : num_items;
  const int G = I / 128;
  const int GU = (G + kQuantGroups - 1) / kQuantGroups;
  const long n_units = static_cast<long>(item_hi > item_lo ? item_hi - item_lo : 0) * BN * GU;
  const long nwarps = static_cast<long>(gridDim.x) * (blockDim.x >> 5);
  for (long u = static_cast<long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
       u < n_units; u += nwarps) {
    const int g0 = static_cast<int>(u % GU) * kQuantGroups;
    const long rr = u / GU;
    const int4 it = items[item_lo + static_cast<int>(rr / BN)];
    const int r = static_cast<int>(rr % BN);
    if (r >= it.z) continue;  // the same for the whole warp
    const size_t row = static_cast<size_t>(it.y) + r;
    const __nv_bfloat16* gr = gu + row * 2 * I + lane * 4;
    uint2 graw[kQuantGroups], uraw[kQuantGroups];
#pragma unroll
    for (int g = 0; g < kQuantGroups; ++g)
      if (g0 + g < G) {
        graw[g] = *reinterpret_cast<const uint2*>(gr + (g0 + g) * 128);
        uraw[g] = *reinterpret_cast<const uint2*>(gr + I + (g0 + g) * 128);
      }
#pragma unroll
    for (int g = 0; g < kQuantGroups; ++g) {
      const int grp = g0 + g;
      if (grp >= G) break;
      const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&graw[g]);
      const __nv_bfloat162* u2 = reinterpret_cast<const __nv_bfloat162*>(&uraw[g]);
      float a[4];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float2 gg = __bfloat1622float2(g2[h]);
        const float2 uu = __bfloat1622float2(u2[h]);
        a[2 * h] = sl::bf16_round(sl::bf16_round(gg.x / (1.0f + expf(-gg.x))) * uu.x);
        a[2 * h + 1] = sl::bf16_round(sl::bf16_round(gg.y / (1.0f + expf(-gg.y))) * uu.y);
      }
      float m = fmaxf(fmaxf(fabsf(a[0]), fabsf(a[1])), fmaxf(fabsf(a[2]), fabsf(a[3])));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      const float scv = group_scale(m);
      *reinterpret_cast<uint32_t*>(Aq + row * I + grp * 128 + lane * 4) =
          e4m3x4(q_clamp(a[0], scv), q_clamp(a[1], scv), q_clamp(a[2], scv), q_clamp(a[3], scv));
      if (lane == 0) As[static_cast<size_t>(grp) * max_rows + row] = scv;
    }
  }
}

// ---------------------------------------------------------------- combine
// OUT_F32 = false: out = bf16(shared + bf16(scale * bf16(sum_j w z)))  (vLLM
//   torch-native rounding chain, runner tail in bf16)
// OUT_F32 = true:  out = scale * sum_j w z + shared, fp32, no rounding (the
//   per-rank partial of expert parallelism, summed across ranks afterwards);
//   ACCUMULATE adds it to what `out` holds (the expert waves of one step)
template <bool OUT_F32, bool ACCUMULATE = false>
__global__ void __launch_bounds__(256) combine_kernel(
    const int32_t* __restrict__ ws_hdr, const int32_t* __restrict__ pair_pos,
    const float* __restrict__ tw, const __nv_bfloat16* __restrict__ Z, int T, int topk, int H,
    int n_sh, int sh_t0, int sh_nt, float scale, void* __restrict__ out) {
  sl::pdl_wait();
  sl::pdl_trigger();
  const int t = blockIdx.y;
  const int h0 = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (h0 >= H || ws_hdr[WS_STATUS] != SL_OK) return;
  float r[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) r[i] = 0.f;
  for (int j0 = 0; j0 < topk; j0 += 8) {
    uint4 zv[8];
    float wj[8];
    uint32_t valid = 0;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int j = j0 + u;
      const int pos = j < topk ? pair_pos[t * topk + j] : -1;
      wj[u] = 0.f;
      if (pos >= 0) {
        valid |= 1u << u;
        wj[u] = tw[t * topk + j];
        zv[u] = *reinterpret_cast<const uint4*>(Z + static_cast<size_t>(pos) * H + h0);
      }
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      if (!((valid >> u) & 1u)) continue;
      const __nv_bfloat162* z2 = reinterpret_cast<const __nv_bfloat162*>(&zv[u]);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(z2[i]);
        r[2 * i] = __fadd_rn(r[2 * i], __fmul_rn(f.x, wj[u]));
        r[2 * i + 1] = __fadd_rn(r[2 * i + 1], __fmul_rn(f.y, wj[u]));
      }
    }
  }
  float o[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if constexpr (OUT_F32) {
      o[i] = r[i] * scale;
    } else {
      float routed = sl::bf16_round(r[i]);
      if (scale != 1.f) routed = sl::bf16_round(routed * scale);
      o[i] = routed;
    }
  }
  if (n_sh > 0 && t >= sh_t0 && t < sh_t0 + sh_nt) {
    float sv[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) sv[i] = 0.f;
    for (int e = 0; e < n_sh; ++e) {
      const int pos = ws_hdr[WS_SH_BASE + e] + (t - sh_t0);
      const uint4 zv = *reinterpret_cast<const uint4*>(Z + static_cast<size_t>(pos) * H + h0);
      const __nv_bfloat162* z2 = reinterpret_cast<const __nv_bfloat162*>(&zv);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(z2[i]);
        sv[2 * i] += f.x;
        sv[2 * i + 1] += f.y;
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = (OUT_F32 ? sv[i] : sl::bf16_round(sv[i])) + o[i];
  }
  if constexpr (OUT_F32) {
    float4* dst = reinterpret_cast<float4*>(static_cast<float*>(out) + static_cast<size_t>(t) * H + h0);
    if constexpr (ACCUMULATE) {
      const float4 a = dst[0], b = dst[1];
      o[0] += a.x, o[1] += a.y, o[2] += a.z, o[3] += a.w;
      o[4] += b.x, o[5] += b.y, o[6] += b.z, o[7] += b.w;
    }
    dst[0] = make_float4(o[0], o[1], o[2], o[3]);
    dst[1] = make_float4(o[4], o[5], o[6], o[7]);
  } else {
    uint4 ov;
    __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&ov);
#pragma unroll
    for (int i = 0; i < 4; ++i) o2[i] = __floats2bfloat162_rn(o[2 * i], o[2 * i + 1]);
    *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(out) + static_cast<size_t>(t) * H + h0) = ov;
  }
}

// ------------------------------------------------------------------- host
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D view [rows, inner] (inner contiguous), 128B swizzle (the MMA operand
// layout): bf16 with a 64-element box, or e4m3 (fp8) with a 128-byte box,
// box_rows rows.
bool make_map(CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows, uint32_t box_rows,
              bool fp8 = false) {
  auto fn = encode_fn();
  if (!fn || (reinterpret_cast<uintptr_t>(base) & 15) || rows == 0) return false;
  const uint64_t esz = fp8 ? 1 : 2;
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {inner * esz};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(fp8 ? F8_BK : BK), box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, fp8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
            const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN, bool GATED>
int launch_gemm_f8(const CUtensorMap& tw, const CUtensorMap& twsh, const CUtensorMap& tb,
                   const float* bscale, const float* wscale, const float* wshscale,
                   const int32_t* hdr, const int4* items, uint8_t* out_q, float* out_s,
                   __nv_bfloat16* out_z, int S, int K, int M_total, int max_rows,
                   int32_t* status, int max_items, cudaStream_t st, int phase,
                   const void* w_raw, const void* wsh_raw) {
  using Cfg = F8Cfg<BN, GATED>;
  auto kern = moe_gemm_f8_kernel<BN, GATED>;
  static std::atomic<uint64_t> smem_set{0};
  SL_CUDA_TRY(sl::ensure_smem_limit(kern, Cfg::kSmemBytes, smem_set));
  const int max_tiles = max_items * (M_total / 128);
  int grid = sl_device_sm_count();
  if (grid <= 0) return SL_ERR_CUDA;
  if (max_tiles < grid) grid = max_tiles > 0 ? max_tiles : 1;
  SL_CUDA_TRY(sl::launch(kern, dim3(grid), dim3(Cfg::kThreads), Cfg::kSmemBytes, st, tw, twsh,
                         tb, bscale, wscale, wshscale, hdr, items, out_q, out_s, out_z, S, K,
                         M_total, max_rows, status, phase, static_cast<const uint8_t*>(w_raw),
                         static_cast<const uint8_t*>(wsh_raw ? wsh_raw : w_raw)));
  return SL_OK;
}

int launch_gemm_f8w(const CUtensorMap& tw, const CUtensorMap& twsh, const CUtensorMap& tb,
                    const float* bscale, const float* wscale, const float* wshscale,
                    const int32_t* hdr, const int4* items, __nv_bfloat16* out, int S, int K,
                    int M_total, int max_rows, int32_t* status, int max_items, cudaStream_t st,
                    int phase) {
  static std::atomic<uint64_t> smem_set{0};
  SL_CUDA_TRY(sl::ensure_smem_limit(moe_gemm_f8w_kernel, F8W_SMEM, smem_set));
  const long max_tiles = static_cast<long>(max_items) * (M_total / 128);
  int grid = sl_device_sm_count();
  if (grid <= 0) return SL_ERR_CUDA;
  if (max_tiles < grid) grid = max_tiles > 0 ? static_cast<int>(max_tiles) : 1;
  SL_CUDA_TRY(sl::launch(moe_gemm_f8w_kernel, dim3(grid), dim3(F8W_THREADS), F8W_SMEM, st, tw,
                         twsh, tb, bscale, wscale, wshscale, hdr, items, out, S, K, M_total,
                         max_rows, status, phase));
  return SL_OK;
}

template <int BN, int STAGES, bool GATED>
int launch_gemm(const CUtensorMap& tw, const CUtensorMap& twsh, const CUtensorMap& tb,
                const int32_t* hdr, const int4* items, __nv_bfloat16* out, int S, int K,
                int M_total, int out_ld, int32_t* status, int max_items, cudaStream_t st,
                int phase, const void* w_raw, const void* wsh_raw) {
  using Cfg = GemmCfg<BN, STAGES, GATED>;
  auto kern = moe_gemm_kernel<BN, STAGES, GATED>;
  static std::atomic<uint64_t> smem_set{0};
  SL_CUDA_TRY(sl::ensure_smem_limit(kern, Cfg::kSmemBytes, smem_set));
  const int max_tiles = max_items * (M_total / TileShape<BN, GATED>::kRowsOut);
  int grid = sl_device_sm_count();
  if (grid <= 0) return SL_ERR_CUDA;
  if (max_tiles < grid) grid = max_tiles > 0 ? max_tiles : 1;
  SL_CUDA_TRY(sl::launch(kern, dim3(grid), dim3(kThreads), Cfg::kSmemBytes, st, tw, twsh, tb,
                         hdr, items, out, S, K, M_total, out_ld, status, phase,
                         static_cast<const uint8_t*>(w_raw),
                         static_cast<const uint8_t*>(wsh_raw ? wsh_raw : w_raw)));
  return SL_OK;
}

}  // namespace

extern "C" size_t sl_fused_experts_workspace_bytes(int T, int topk, int H, int I,
                                                   int num_slots, int n_shared) {
  if (T < 0 || topk <= 0 || H <= 0 || I <= 0 || num_slots <= 0 || n_shared < 0) return 0;
  // large enough for either weight dtype's token tiles
  const size_t a = ws_layout(T, topk, H, I, num_slots, n_shared, choose_bn(T, topk, num_slots)).total;
  const int bn8 = choose_bn(T, topk, num_slots, true);
  const size_t b = ws_layout(T, topk, H, I, num_slots, n_shared, bn8, bn8 == kF8WideBN).total;
  return a > b ? a : b;
}

// Argument checks of every fused-experts entry point, made before anything is
// enqueued (see common.cuh).
int sl::fused_experts_check(const void* hidden, int T, int H, int I, const sl_expert_weights& w,
                            const float* topk_weights, const int32_t* topk_ids, int topk,
                            const int32_t* expert_map, int global_n, int sh_t0, int sh_nt,
                            const void* out, int out_mode, const void* workspace,
                            size_t workspace_bytes, const void* fill_state, int phase) {
  if (out_mode < 0 || out_mode > 2) return SL_ERR_INVALID;
  const int num_slots = w.num_slots, n_shared = w.n_shared;
  const bool fp8 = w.dtype == SL_WEIGHTS_FP8_BLOCK128;
  if (w.dtype != SL_WEIGHTS_BF16 && !fp8) return SL_ERR_UNSUPPORTED;
  if (T < 0 || topk <= 0 || num_slots <= 0 || n_shared < 0) return SL_ERR_INVALID;
  if (H % BM || I % BM || H <= 0 || I <= 0) return SL_ERR_UNSUPPORTED;
  if (num_slots + n_shared > kMaxCode || n_shared > kMaxShared) return SL_ERR_UNSUPPORTED;
  if (phase < -1 || phase > SL_PHASE_COMBINE || (phase >= 0 && !fill_state))
    return SL_ERR_INVALID;
  if (T == 0) return SL_OK;
  if (!hidden || !w.w13 || !w.w2 || !topk_weights || !topk_ids || !out || !workspace)
    return SL_ERR_INVALID;
  if (fp8 && (!w.w13_scale || !w.w2_scale)) return SL_ERR_INVALID;
  if (n_shared > 0 && (!w.shared_w13 || !w.shared_w2)) return SL_ERR_INVALID;
  if (fp8 && n_shared > 0 && (!w.shared_w13_scale || !w.shared_w2_scale)) return SL_ERR_INVALID;
  if (n_shared > 0 && (sh_t0 < 0 || sh_nt < 0 || sh_t0 + sh_nt > T)) return SL_ERR_INVALID;
  if (expert_map && global_n <= 0) return SL_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255) ||
      ((reinterpret_cast<uintptr_t>(hidden) | reinterpret_cast<uintptr_t>(out)) & 15))
    return SL_ERR_INVALID;
  if (fp8 && (H / 128 > kF8MaxKBlocks || I / 128 > kF8MaxKBlocks)) return SL_ERR_UNSUPPORTED;
  const int BN = choose_bn(T, topk, num_slots, fp8);
  if (workspace_bytes < ws_layout(T, topk, H, I, num_slots, n_shared, BN,
                                  fp8 && BN == kF8WideBN).total)
    return SL_ERR_INVALID;
  return SL_OK;
}

namespace {

int run_fused(const void* hidden, int T, int H, int I, const sl_expert_weights& w,
              const float* topk_weights, const int32_t* topk_ids, int topk,
              const int32_t* expert_map, int global_n, int sh_t0, int sh_nt,
              float routed_scaling_factor, void* out, int out_mode, void* workspace,
              size_t workspace_bytes, cudaStream_t st, const void* fill_state = nullptr,
              int phase = -1) {
  // out_mode: 0 bf16 out; 1 fp32 partial written; 2 fp32 partial added to out
  const int rc0 = sl::fused_experts_check(hidden, T, H, I, w, topk_weights, topk_ids, topk,
                                          expert_map, global_n, sh_t0, sh_nt, out, out_mode,
                                          workspace, workspace_bytes, fill_state, phase);
  if (rc0 != SL_OK || T == 0) return rc0;
  const bool out_f32 = out_mode != 0, accumulate = out_mode == 2;
  const int num_slots = w.num_slots, n_shared = w.n_shared;
  const bool fp8 = w.dtype == SL_WEIGHTS_FP8_BLOCK128;
  const int BN = choose_bn(T, topk, num_slots, fp8);
  const WsLayout L = ws_layout(T, topk, H, I, num_slots, n_shared, BN, fp8 && BN == kF8WideBN);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int32_t* hdr = reinterpret_cast<int32_t*>(ws);
  int4* items = reinterpret_cast<int4*>(ws + L.items);
  int32_t* pair_pos = reinterpret_cast<int32_t*>(ws + L.pair_pos);
  __nv_bfloat16* X = reinterpret_cast<__nv_bfloat16*>(ws + L.x);
  __nv_bfloat16* A = reinterpret_cast<__nv_bfloat16*>(ws + L.act);
  __nv_bfloat16* Z = reinterpret_cast<__nv_bfloat16*>(ws + L.z);

  // fp8: the gathered rows and the gate/up output are quantised per
  // 128-column group: e4m3 rows [max_rows, H or I] followed by fp32 scales
  // [H/128 or I/128, max_rows], inside the bf16 regions
  uint8_t* Xq = ws + L.x;
  float* Xs = reinterpret_cast<float*>(ws + L.x + r256(size_t(L.max_rows) * H));
  uint8_t* Aq = ws + L.act;
  float* As = reinterpret_cast<float*>(ws + L.act + r256(size_t(L.max_rows) * I));

  CUtensorMap m_w13, m_w13sh, m_x, m_w2, m_w2sh, m_a;
  const int nsh = n_shared > 0 ? n_shared : 0;
  // bf16 gate/up weight boxes are 64 gate + 64 up rows; fp8 ones 128 + 128
  const uint32_t w13_box = fp8 ? 128 : 64;
  bool ok = make_map(&m_w13, w.w13, H, uint64_t(num_slots) * 2 * I, w13_box, fp8) &&
            make_map(&m_w2, w.w2, I, uint64_t(num_slots) * H, BM, fp8) &&
            make_map(&m_x, fp8 ? static_cast<void*>(Xq) : X, H, uint64_t(L.max_rows), BN, fp8) &&
            make_map(&m_a, fp8 ? static_cast<void*>(Aq) : A, I, uint64_t(L.max_rows), BN, fp8);
  if (ok && nsh) {
    ok = make_map(&m_w13sh, w.shared_w13, H, uint64_t(nsh) * 2 * I, w13_box, fp8) &&
         make_map(&m_w2sh, w.shared_w2, I, uint64_t(nsh) * H, BM, fp8);
  } else {
    m_w13sh = m_w13;
    m_w2sh = m_w2;
  }
  if (!ok) return SL_ERR_INVALID;

  // decode-sized steps: a small grid groups and gathers at once; larger ones
  // group in one CTA and gather with a grid-wide kernel
  const int P = T * topk;
  const bool small = P <= kSmallP && (num_slots + nsh) <= kMaxCode;
  // phase -1: everything; 0 = grouping + resident experts' GEMMs; 1 =
  // streamed experts' GEMMs + combine; 2..5: one of those four parts alone
  const bool do_group = phase == -1 || phase == 0 || phase == SL_PHASE_GROUP;
  const bool do_gemms = phase != SL_PHASE_GROUP && phase != SL_PHASE_COMBINE;
  const bool do_combine = phase == -1 || phase == 1 || phase == SL_PHASE_COMBINE;
  // the GEMM kernels' item range: -1 all, 0 resident experts, 1 streamed ones
  const int gphase = phase == -1 ? -1
                     : (phase == 0 || phase == SL_PHASE_RESIDENT_GEMMS) ? 0 : 1;
  if (do_group) {
    if (small) {
      SL_CUDA_TRY(sl::launch(align_small_kernel, dim3(kAlignSmallCtas), dim3(kAlignSmallThreads),
                             0, st, topk_ids, T, topk, expert_map, global_n, num_slots, nsh,
                             nsh ? sh_t0 : 0, nsh ? sh_nt : 0, BN,
                             static_cast<const __nv_bfloat16*>(hidden), H, hdr, items, pair_pos,
                             fp8 ? nullptr : X, L.max_items,
                             static_cast<const uint8_t*>(fill_state)));
    } else {
      SL_CUDA_TRY(sl::launch(align_kernel, dim3(1), dim3(1024), 0, st, topk_ids, T, topk,
                             expert_map, global_n, num_slots, nsh, nsh ? sh_t0 : 0,
                             nsh ? sh_nt : 0, BN, static_cast<const __nv_bfloat16*>(hidden), H,
                             hdr, items, pair_pos, X, L.max_items,
                             static_cast<const uint8_t*>(fill_state), 0));
      if (!fp8)
        SL_CUDA_TRY(sl::launch(gather_kernel, dim3(2 * sl_device_sm_count()), dim3(256), 0, st,
                               static_cast<const int32_t*>(hdr),
                               static_cast<const int32_t*>(pair_pos), P, topk, nsh,
                               nsh ? sh_t0 : 0, nsh ? sh_nt : 0,
                               static_cast<const __nv_bfloat16*>(hidden), H, X));
    }
    if (fp8) {
      // one unit = four 128-column groups of one token, quantised once and
      // written to every row the token feeds
      const long units = static_cast<long>(T) * ((H / 128 + kQuantGroups - 1) / kQuantGroups);
      long ctas = (units + 7) / 8;  // 8 warps per CTA, one unit each
      const long cap = 8L * sl_device_sm_count();
      if (ctas > cap) ctas = cap;
      if (ctas < 1) ctas = 1;
      SL_CUDA_TRY(sl::launch(gather_quant_kernel, dim3(static_cast<unsigned>(ctas)), dim3(256),
                             0, st,
                             static_cast<const int32_t*>(hdr),
                             static_cast<const int32_t*>(pair_pos), T, topk, nsh,
                             nsh ? sh_t0 : 0, nsh ? sh_nt : 0,
                             static_cast<const __nv_bfloat16*>(hidden), H, Xq, Xs, L.max_rows));
    }
  }
  int rc = SL_OK;
#define SL_GEMMS_BF16(BNV, S1, S2)                                                              \
  rc = launch_gemm<BNV, S1, true>(m_w13, m_w13sh, m_x, hdr, items, A, num_slots, H, I, I, hdr,   \
                                  L.max_items, st, gphase, w.w13, w.shared_w13);                  \
  if (rc == SL_OK)                                                                               \
    rc = launch_gemm<BNV, S2, false>(m_w2, m_w2sh, m_a, hdr, items, Z, num_slots, I, H, H, hdr,  \
                                     L.max_items, st, gphase, w.w2, w.shared_w2);
#define SL_GEMMS_F8(BNV)                                                                         \
  rc = launch_gemm_f8<BNV, true>(m_w13, m_w13sh, m_x, Xs, w.w13_scale, w.shared_w13_scale, hdr,  \
                                 items, Aq, As, nullptr, num_slots, H, I, L.max_rows, hdr,      \
                                 L.max_items, st, gphase, w.w13, w.shared_w13);                   \
  if (rc == SL_OK)                                                                               \
    rc = launch_gemm_f8<BNV, false>(m_w2, m_w2sh, m_a, As, w.w2_scale, w.shared_w2_scale, hdr,   \
                                    items, nullptr, nullptr, Z, num_slots, I, H, L.max_rows,    \
                                    hdr, L.max_items, st, gphase, w.w2, w.shared_w2);
  if (!do_gemms) {
    // grouping or combine alone
  } else if (fp8 && BN == kF8WideBN) {
    // gate/up over the 2I rows into bf16 g | u rows, SwiGLU + quantisation,
    // then down; the token tiles are read in 32-row boxes
    CUtensorMap m_xw, m_aw;
    if (!make_map(&m_xw, Xq, H, uint64_t(L.max_rows), 32, true) ||
        !make_map(&m_aw, Aq, I, uint64_t(L.max_rows), 32, true))
      return SL_ERR_INVALID;
    __nv_bfloat16* GU = reinterpret_cast<__nv_bfloat16*>(ws + L.gu);
    rc = launch_gemm_f8w(m_w13, m_w13sh, m_xw, Xs, w.w13_scale, w.shared_w13_scale, hdr, items,
                         GU, num_slots, H, 2 * I, L.max_rows, hdr, L.max_items, st, gphase);
    if (rc == SL_OK) {
      const long units = static_cast<long>(L.max_items) * BN *
                         ((I / 128 + kQuantGroups - 1) / kQuantGroups);
      long ctas = (units + 7) / 8;
      const long cap = 8L * sl_device_sm_count();
      if (ctas > cap) ctas = cap;
      if (ctas < 1) ctas = 1;
      SL_CUDA_TRY(sl::launch(swiglu_quant_kernel, dim3(static_cast<unsigned>(ctas)), dim3(256),
                             0, st, static_cast<const int32_t*>(hdr),
                             static_cast<const int4*>(items), BN,
                             static_cast<const __nv_bfloat16*>(GU), I, Aq, As, L.max_rows,
                             gphase));
      rc = launch_gemm_f8w(m_w2, m_w2sh, m_aw, As, w.w2_scale, w.shared_w2_scale, hdr, items, Z,
                           num_slots, I, H, L.max_rows, hdr, L.max_items, st, gphase);
    }
  } else if (fp8) {
    SL_GEMMS_F8(16)
  } else if (BN == 16) {
    SL_GEMMS_BF16(16, 12, 12)
  } else if (BN == 64) {
    SL_GEMMS_BF16(64, 9, 9)
  } else {
    SL_GEMMS_BF16(128, 6, 6)
  }
#undef SL_GEMMS_BF16
#undef SL_GEMMS_F8
  if (rc != SL_OK) return rc;
  if (!do_combine) return SL_OK;
  dim3 cgrid((H / 8 + 255) / 256, T);
  SL_CUDA_TRY(sl::launch(accumulate ? combine_kernel<true, true>
                         : out_f32  ? combine_kernel<true>
                                    : combine_kernel<false>,
                         cgrid, dim3(256), 0, st, static_cast<const int32_t*>(hdr),
                         static_cast<const int32_t*>(pair_pos), topk_weights,
                         static_cast<const __nv_bfloat16*>(Z), T, topk, H, nsh, sh_t0, sh_nt,
                         routed_scaling_factor, out));
  return SL_OK;
}

sl_expert_weights bf16_weights(const void* w13, const void* w2, int num_slots,
                               const void* shared_w13, const void* shared_w2, int n_shared) {
  sl_expert_weights w = {};
  w.w13 = w13;
  w.w2 = w2;
  w.num_slots = num_slots;
  w.shared_w13 = shared_w13;
  w.shared_w2 = shared_w2;
  w.n_shared = n_shared;
  w.dtype = SL_WEIGHTS_BF16;
  return w;
}

}  // namespace

extern "C" int sl_fused_experts(const void* hidden, int T, int H, int I, const void* w13,
                                const void* w2, int num_slots, int weight_dtype,
                                const float* topk_weights, const int32_t* topk_ids, int topk,
                                const int32_t* expert_map, int global_n,
                                const void* shared_w13, const void* shared_w2, int n_shared,
                                float routed_scaling_factor, void* out, void* workspace,
                                size_t workspace_bytes, sl_stream_t stream) {
  if (weight_dtype != SL_WEIGHTS_BF16) return SL_ERR_UNSUPPORTED;
  const sl_expert_weights w = bf16_weights(w13, w2, num_slots, shared_w13, shared_w2, n_shared);
  return run_fused(hidden, T, H, I, w, topk_weights, topk_ids, topk, expert_map, global_n, 0,
                   T, routed_scaling_factor, out, 0, workspace, workspace_bytes,
                   reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int sl_fused_experts_partial(const void* hidden, int T, int H, int I,
                                        const void* w13, const void* w2, int num_slots,
                                        int weight_dtype, const float* topk_weights,
                                        const int32_t* topk_ids, int topk,
                                        const int32_t* expert_map, int global_n,
                                        const void* shared_w13, const void* shared_w2,
                                        int n_shared, int shared_t0, int shared_nt,
                                        float routed_scaling_factor, float* out_f32,
                                        void* workspace, size_t workspace_bytes,
                                        sl_stream_t stream) {
  if (weight_dtype != SL_WEIGHTS_BF16) return SL_ERR_UNSUPPORTED;
  const sl_expert_weights w = bf16_weights(w13, w2, num_slots, shared_w13, shared_w2, n_shared);
  return run_fused(hidden, T, H, I, w, topk_weights, topk_ids, topk, expert_map, global_n,
                   shared_t0, shared_nt, routed_scaling_factor, out_f32, 1, workspace,
                   workspace_bytes, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int sl_fused_experts_phase(const void* hidden, int T, int H, int I, const void* w13,
                                      const void* w2, int num_slots, int weight_dtype,
                                      const float* topk_weights, const int32_t* topk_ids,
                                      int topk, const int32_t* expert_map, int global_n,
                                      const void* shared_w13, const void* shared_w2,
                                      int n_shared, float routed_scaling_factor,
                                      const void* slot_state, int phase, void* out,
                                      void* workspace, size_t workspace_bytes,
                                      sl_stream_t stream) {
  if (weight_dtype != SL_WEIGHTS_BF16) return SL_ERR_UNSUPPORTED;
  if (phase < 0 || phase > SL_PHASE_COMBINE) return SL_ERR_INVALID;
  const sl_expert_weights w = bf16_weights(w13, w2, num_slots, shared_w13, shared_w2, n_shared);
  return run_fused(hidden, T, H, I, w, topk_weights, topk_ids, topk, expert_map, global_n, 0,
                   T, routed_scaling_factor, out, 0, workspace, workspace_bytes,
                   reinterpret_cast<cudaStream_t>(stream), slot_state, phase);
}

extern "C" int sl_fused_experts_ex(const void* hidden, int T, int H, int I,
                                   const sl_expert_weights* weights, const float* topk_weights,
                                   const int32_t* topk_ids, int topk, const int32_t* expert_map,
                                   int global_n, float routed_scaling_factor, int shared_t0,
                                   int shared_nt, const void* slot_state, int phase, int out_f32,
                                   void* out, void* workspace, size_t workspace_bytes,
                                   sl_stream_t stream) {
  if (!weights) return SL_ERR_INVALID;
  if (shared_nt < 0) {  // default: every token
    shared_t0 = 0;
    shared_nt = T;
  }
  return run_fused(hidden, T, H, I, *weights, topk_weights, topk_ids, topk, expert_map,
                   global_n, shared_t0, shared_nt, routed_scaling_factor, out, out_f32,
                   workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream),
                   slot_state, phase);
}
