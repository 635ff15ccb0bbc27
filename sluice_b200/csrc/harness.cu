// Decoder-harness kernels for the DeepSeek-V2-Lite-shaped decoder that wraps
// the MoE layers in the benchmark (not part of the reference's MoE operator
// surface): the absorbed multi-head latent attention (MLA) of one decode step
// in one launch (it replaces a dozen small PyTorch kernels per layer: norm,
// rotary embedding, cache write, the absorbed query, scores, softmax, the
// weighted latent sum and the value map), the residual add + RMSNorm, and a
// skinny linear for single-sequence projections.
//
// MLA:
// One CTA per (head, sequence), sixteen warps. Inputs per sequence: the fused
// projection row [q (heads x (nope + rope)) | c_kv (rank) | k_pe (rope)] of
// this step, its position P; the latent cache [B, max_len, rank + rope]. The
// CTA:
//   1. normalises c_kv (RMSNorm, fp32, one bf16 rounding) and rotates k_pe
//      (RoPE on adjacent pairs) for position P; CTA head 0 writes them to the
//      cache (the other heads use their own copy for position P);
//   2. forms the absorbed query [q_nope W_uk | rope(q_pe)] (fp32 sums, bf16
//      rounding, as the bf16 GEMM it replaces);
//   3. scores every cached position 0..P and sums the latents weighted by
//      their softmax probabilities in one pass (a running max and sum per
//      warp, merged across the warps at the end);
//   4. maps the weighted latent through W_uv.
// Everything the CTA reads in bulk -- the head's W_uk rows, the sequence's
// cached rows 0..P-1, the head's W_uv rows -- arrives in 32-row chunks by
// 1-D bulk copies (cp.async.bulk) into a ring of four shared-memory slots,
// issued up to four chunks ahead of the warps that consume them, so the
// DRAM latency is paid about once per four chunks instead of once per row
// batch. Each lane owns 16 of the 512 latent columns (two 8-column chunks);
// the warps split a chunk's rows. The rank is fixed at 512 (the DeepSeek-V2 /
// V3 latent width) and rope at most 64; other shapes are refused by the host.
#include "common.cuh"

namespace {

constexpr int kMlaThreads = 512;
constexpr int kMlaWarps = kMlaThreads / 32;
constexpr int kRank = 512;
constexpr int kRingRows = 32;    // rows per bulk-copied chunk
constexpr int kRingSlots = 4;    // chunks in flight
constexpr int kMaxRowBytes = (512 + 64) * 2;
constexpr int kSlotBytes = kRingRows * kMaxRowBytes;  // 36864, a multiple of 16

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < nw; ++i) t += red[i];
  return t;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// The lane's 16 columns of a 512-wide bf16 row: columns 8*lane.. and
// 256 + 8*lane.., as two 16-byte loads.
struct Row16 {
  uint4 a, b;
};
__device__ __forceinline__ Row16 load_row16(const __nv_bfloat16* row, int lane) {
  Row16 r;
  r.a = *reinterpret_cast<const uint4*>(row + 8 * lane);
  r.b = *reinterpret_cast<const uint4*>(row + 256 + 8 * lane);
  return r;
}
// ... as eight column pairs: v[i] holds columns col16(lane, 2i), col16(lane, 2i + 1)
// (the arithmetic on them is packed fp32x2, two columns per instruction)
__device__ __forceinline__ void unpack16(const Row16& r, float2 (&v)[8]) {
  const __nv_bfloat162* a = reinterpret_cast<const __nv_bfloat162*>(&r.a);
  const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&r.b);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[i] = __bfloat1622float2(a[i]);
    v[4 + i] = __bfloat1622float2(b[i]);
  }
}
__device__ __forceinline__ int col16(int lane, int i) {
  return i < 8 ? 8 * lane + i : 256 + 8 * lane + (i - 8);
}

__global__ void __launch_bounds__(kMlaThreads) mla_decode_kernel(
    const __nv_bfloat16* __restrict__ qkv, int ld_qkv, const __nv_bfloat16* __restrict__ kv_norm,
    float eps, const __nv_bfloat16* __restrict__ w_uk, const __nv_bfloat16* __restrict__ w_uv,
    const float2* __restrict__ rope_cs, const int64_t* __restrict__ pos,
    __nv_bfloat16* __restrict__ cache, int nh, int nope, int rope, int vdim, int max_len,
    float scale, __nv_bfloat16* __restrict__ out) {
  extern __shared__ __align__(16) uint8_t sm_raw[];
  const int h = blockIdx.x, b = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int dk = kRank + rope;
  uint8_t* ring = sm_raw;                                            // [slots][kSlotBytes]
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + kRingSlots * kSlotBytes);
  float* q = reinterpret_cast<float*>(full + kRingSlots);            // [dk] absorbed query
  float* kv = q + dk;                      // [dk] this position's latent | rotated k_pe
  float* part = kv + dk;                   // [warps][rank] per-warp partial sums
  float* qn = part + kMlaWarps * kRank;    // [nope] q_nope of this head
  float* wm = qn + nope;                   // [warps] running max per warp
  float* wl = wm + kMlaWarps;              // [warps] running sum per warp
  float* red = wl + kMlaWarps;             // [32]
  int* slot_done = reinterpret_cast<int*>(red + 32);  // [slots] warps done with a slot

  // the chunk jobs, in consumption order: W_uk rows, cached rows 0..P-1,
  // W_uv rows
  const int nk = (nope + kRingRows - 1) / kRingRows;
  const int nv = (vdim + kRingRows - 1) / kRingRows;
  int P = 0, nc = 0;
  auto issue = [&](int j) {
    const __nv_bfloat16* src;
    int rows;
    size_t row_bytes;
    if (j < nk) {
      src = w_uk + (static_cast<size_t>(h) * nope + j * kRingRows) * kRank;
      rows = min(kRingRows, nope - j * kRingRows);
      row_bytes = kRank * 2;
    } else if (j < nk + nc) {
      const int c = j - nk;
      src = cache + (static_cast<size_t>(b) * max_len + c * kRingRows) * dk;
      rows = min(kRingRows, P - c * kRingRows);
      row_bytes = static_cast<size_t>(dk) * 2;
    } else {
      const int v = j - nk - nc;
      src = w_uv + (static_cast<size_t>(h) * vdim + v * kRingRows) * kRank;
      rows = min(kRingRows, vdim - v * kRingRows);
      row_bytes = kRank * 2;
    }
    const uint32_t bytes = static_cast<uint32_t>(rows * row_bytes);
    uint64_t* bar = &full[j % kRingSlots];
    sl::mbar_arrive_expect_tx(bar, bytes);
    sl::bulk_load(ring + (j % kRingSlots) * kSlotBytes, src, bytes, bar);
  };
  if (tid == 0) {
    for (int i = 0; i < kRingSlots; ++i) {
      sl::mbar_init(&full[i], 1);
      slot_done[i] = 0;
    }
    sl::fence_barrier_init();
    // the weights are constants of the step: their chunks may be fetched
    // before waiting on the kernel that wrote this step's projections
    for (int j = 0; j < nk && j < kRingSlots; ++j) issue(j);
  }
  sl::pdl_wait();
  sl::pdl_trigger();
  P = static_cast<int>(pos[b]);
  P = P < 0 ? 0 : (P >= max_len ? max_len - 1 : P);
  nc = (P + kRingRows - 1) / kRingRows;
  const int J = nk + nc + nv;
  if (tid == 0) {
    // the rest of the first ring's chunks (fewer weight chunks than slots)
    for (int j = min(nk, kRingSlots); j < min(J, kRingSlots); ++j) issue(j);
    // everything the ring will fetch later is asked into L2 now, so those
    // chunks land at L2 rather than DRAM latency
    auto prefetch = [&](const void* src, size_t bytes) {
      for (size_t o = 0; o < bytes; o += 65536) {
        const uint32_t n = static_cast<uint32_t>(bytes - o < 65536 ? bytes - o : 65536);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(
                         reinterpret_cast<const uint8_t*>(src) + o),
                     "r"(n)
                     : "memory");
      }
    };
    prefetch(cache + static_cast<size_t>(b) * max_len * dk, static_cast<size_t>(P) * dk * 2);
    prefetch(w_uv + static_cast<size_t>(h) * vdim * kRank, static_cast<size_t>(vdim) * kRank * 2);
  }
  const __nv_bfloat16* row = qkv + static_cast<size_t>(b) * ld_qkv;
  const __nv_bfloat16* qh = row + h * (nope + rope);
  const __nv_bfloat16* ckv = row + nh * (nope + rope);
  const float2* cs = rope_cs + static_cast<size_t>(P) * (rope / 2);

  // 1. RMSNorm of c_kv and the rotated k_pe for position P; q_nope to shared
  float ss = 0.f;
  for (int i = tid; i < kRank; i += blockDim.x) {
    const float v = __bfloat162float(ckv[i]);
    kv[i] = v;
    ss += v * v;
  }
  for (int d = tid; d < nope; d += blockDim.x) qn[d] = __bfloat162float(qh[d]);
  const float r = rsqrtf(block_sum(ss, red) / kRank + eps);
  for (int i = tid; i < kRank; i += blockDim.x)
    kv[i] = sl::bf16_round(kv[i] * r * __bfloat162float(kv_norm[i]));
  for (int j = tid; j < rope / 2; j += blockDim.x) {
    const float x0 = __bfloat162float(ckv[kRank + 2 * j]);
    const float x1 = __bfloat162float(ckv[kRank + 2 * j + 1]);
    const float2 c = cs[j];
    kv[kRank + 2 * j] = sl::bf16_round(x0 * c.x - x1 * c.y);
    kv[kRank + 2 * j + 1] = sl::bf16_round(x1 * c.x + x0 * c.y);
    const float y0 = __bfloat162float(qh[nope + 2 * j]), y1 = __bfloat162float(qh[nope + 2 * j + 1]);
    q[kRank + 2 * j] = sl::bf16_round(y0 * c.x - y1 * c.y);
    q[kRank + 2 * j + 1] = sl::bf16_round(y1 * c.x + y0 * c.y);
  }
  __syncthreads();  // barriers initialised, kv / q rope / q_nope written

  const int rp = rope / 32;  // rope columns per lane
  float2 acc[8];              // absorbed query, then the weighted latent
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = make_float2(0.f, 0.f);
  float2 qr[8];
  float qp0 = 0.f, qp1 = 0.f;
  float m_w = -INFINITY, l_w = 0.f;  // this warp's running max and sum
  float2 o16[8];
  auto store_part = [&]() {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      part[warp * kRank + col16(lane, 2 * i)] = acc[i].x;
      part[warp * kRank + col16(lane, 2 * i + 1)] = acc[i].y;
    }
  };
  auto load_pairs = [&](const float* src, float2 (&d)[8]) {
#pragma unroll
    for (int i = 0; i < 8; ++i) d[i] = make_float2(src[col16(lane, 2 * i)], src[col16(lane, 2 * i + 1)]);
  };
  // online softmax step of one row: score s, latent values v
  auto absorb = [&](float s, const float2 (&v)[8]) {
    if (s > m_w) {
      const float corr = __expf(m_w - s);
      l_w *= corr;
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = __fmul2_rn(make_float2(corr, corr), acc[i]);
      m_w = s;
    }
    const float pe = __expf(s - m_w);
    l_w += pe;
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = __ffma2_rn(make_float2(pe, pe), v[i], acc[i]);
  };
  auto dot = [&](const float2 (&v)[8]) {
    float2 t = make_float2(0.f, 0.f);
#pragma unroll
    for (int i = 0; i < 8; ++i) t = __ffma2_rn(qr[i], v[i], t);
    return t.x + t.y;
  };

  for (int j = 0; j < J; ++j) {
    // a chunk is a bulk copy of this GPU's own memory, which always lands;
    // the wait is bounded (2 s) only so that no fault elsewhere can hang it
    (void)sl::mbar_wait(&full[j % kRingSlots], (j / kRingSlots) & 1);
    const uint8_t* slot = ring + (j % kRingSlots) * kSlotBytes;
    if (j < nk) {
      // 2. absorbed query: q_lat[c] += q_nope[d] W_uk[h][d][c] over this
      // chunk's rows (warp w: rows w, w + 16, ...)
      const int d0 = j * kRingRows;
      const int rows = min(kRingRows, nope - d0);
      for (int rr = warp; rr < rows; rr += kMlaWarps) {
        float2 v[8];
        unpack16(load_row16(reinterpret_cast<const __nv_bfloat16*>(slot) + rr * kRank, lane), v);
        const float qd = qn[d0 + rr];
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = __ffma2_rn(make_float2(qd, qd), v[i], acc[i]);
      }
    } else if (j < nk + nc) {
      // 3. scores and the weighted latent of this chunk's cached rows
      const int l0 = (j - nk) * kRingRows;
      const int rows = min(kRingRows, P - l0);
      const __nv_bfloat16* base = reinterpret_cast<const __nv_bfloat16*>(slot);
      for (int rr = warp; rr < rows; rr += kMlaWarps) {
        const __nv_bfloat16* key = base + rr * dk;
        float2 v[8];
        unpack16(load_row16(key, lane), v);
        float sdot = dot(v);
        if (rp > 0) sdot = fmaf(qp0, __bfloat162float(key[kRank + lane * rp]), sdot);
        if (rp > 1) sdot = fmaf(qp1, __bfloat162float(key[kRank + lane * rp + 1]), sdot);
        absorb(warp_sum(sdot) * scale, v);
      }
    } else {
      // 4. value map: out[d] = sum_c o_lat[c] W_uv[h][d][c] (warp w: rows
      // w, w + 16, ... of this chunk)
      const int d0 = (j - nk - nc) * kRingRows;
      const int rows = min(kRingRows, vdim - d0);
      __nv_bfloat16* dst = out + static_cast<size_t>(b) * nh * vdim + h * vdim;
      for (int rr = warp; rr < rows; rr += kMlaWarps) {
        float2 v[8];
        unpack16(load_row16(reinterpret_cast<const __nv_bfloat16*>(slot) + rr * kRank, lane), v);
        float2 t2 = make_float2(0.f, 0.f);
#pragma unroll
        for (int i = 0; i < 8; ++i) t2 = __ffma2_rn(o16[i], v[i], t2);
        const float t = warp_sum(t2.x + t2.y);
        if (lane == 0) dst[d0 + rr] = __float2bfloat16(t);
      }
    }
    // this warp is done with the slot: the last warp to finish refills it,
    // so the warps do not wait for one another between chunks
    __syncwarp();
    if (lane == 0) {
      __threadfence_block();
      const int si = j % kRingSlots;
      if (atomicAdd(&slot_done[si], 1) == kMlaWarps - 1) {
        slot_done[si] = 0;
        if (j + kRingSlots < J) {
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          issue(j + kRingSlots);
        }
      }
    }
    if (j == nk - 1) {
      // the absorbed query from the warps' partial sums; CTA head 0 writes
      // position P's row to the cache
      store_part();
      __syncthreads();
      for (int c = tid; c < kRank; c += blockDim.x) {
        float t = 0.f;
#pragma unroll
        for (int w = 0; w < kMlaWarps; ++w) t += part[w * kRank + c];
        q[c] = sl::bf16_round(t);
      }
      if (h == 0) {
        __nv_bfloat16* dst = cache + (static_cast<size_t>(b) * max_len + P) * dk;
        for (int i = tid; i < dk; i += blockDim.x) dst[i] = __float2bfloat16(kv[i]);
      }
      __syncthreads();
      load_pairs(q, qr);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = make_float2(0.f, 0.f);
      qp0 = rp > 0 ? q[kRank + lane * rp] : 0.f;
      qp1 = rp > 1 ? q[kRank + lane * rp + 1] : 0.f;
    }
    if (j == nk + nc - 1) {
      // position P from this CTA's own copy of the new row (warp 0), then
      // the warps' running sums merged into the weighted latent
      if (warp == 0) {
        float2 v[8];
        load_pairs(kv, v);
        float sdot = dot(v);
        if (rp > 0) sdot = fmaf(qp0, kv[kRank + lane * rp], sdot);
        if (rp > 1) sdot = fmaf(qp1, kv[kRank + lane * rp + 1], sdot);
        absorb(warp_sum(sdot) * scale, v);
      }
      store_part();
      if (lane == 0) {
        wm[warp] = m_w;
        wl[warp] = l_w;
      }
      __syncthreads();
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kMlaWarps; ++w) M = fmaxf(M, wm[w]);
      float L = 0.f, f[kMlaWarps];
#pragma unroll
      for (int w = 0; w < kMlaWarps; ++w) {
        f[w] = __expf(wm[w] - M);
        L = fmaf(f[w], wl[w], L);
      }
      const float invL = 1.f / L;
      for (int c = tid; c < kRank; c += blockDim.x) {
        float t = 0.f;
#pragma unroll
        for (int w = 0; w < kMlaWarps; ++w) t = fmaf(f[w], part[w * kRank + c], t);
        q[c] = sl::bf16_round(t * invL);  // the query is no longer needed
      }
      __syncthreads();
      load_pairs(q, o16);
    }
  }
}

// Residual add + RMSNorm, one CTA per row: h = bf16(h + delta), then
// out = bf16(h * rsqrt(mean(h^2) + eps) * w), fp32 arithmetic. Each thread
// holds 8 consecutive columns (one 16-byte load of h, of delta and of w).
constexpr int kNormThreads = 256;

__global__ void __launch_bounds__(kNormThreads) add_rmsnorm_kernel(
    __nv_bfloat16* __restrict__ h, const __nv_bfloat16* __restrict__ delta,
    const __nv_bfloat16* __restrict__ w, float eps, __nv_bfloat16* __restrict__ out, int H) {
  __shared__ float red[32];
  sl::pdl_wait();
  sl::pdl_trigger();
  const size_t base = static_cast<size_t>(blockIdx.x) * H;
  float v[4][8];
  float ss = 0.f;
#pragma unroll
  for (int nv = 0; nv < 4; ++nv) {
    const int c = (threadIdx.x + nv * blockDim.x) * 8;
    if (c >= H) break;
    uint4 hv = *reinterpret_cast<const uint4*>(h + base + c);
    const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&hv);
    if (delta != nullptr) {
      const uint4 dv = *reinterpret_cast<const uint4*>(delta + base + c);
      const __nv_bfloat162* d2 = reinterpret_cast<const __nv_bfloat162*>(&dv);
      uint4 sv;
      __nv_bfloat162* s2 = reinterpret_cast<__nv_bfloat162*>(&sv);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 a = __bfloat1622float2(h2[i]), b = __bfloat1622float2(d2[i]);
        s2[i] = __floats2bfloat162_rn(a.x + b.x, a.y + b.y);
      }
      *reinterpret_cast<uint4*>(h + base + c) = sv;
      hv = sv;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 a = __bfloat1622float2(h2[i]);
      v[nv][2 * i] = a.x;
      v[nv][2 * i + 1] = a.y;
      ss = fmaf(a.x, a.x, ss);
      ss = fmaf(a.y, a.y, ss);
    }
  }
  const float r = rsqrtf(block_sum(ss, red) / H + eps);
#pragma unroll
  for (int nv = 0; nv < 4; ++nv) {
    const int c = (threadIdx.x + nv * blockDim.x) * 8;
    if (c >= H) break;
    const uint4 wv = *reinterpret_cast<const uint4*>(w + c);
    const __nv_bfloat162* w2 = reinterpret_cast<const __nv_bfloat162*>(&wv);
    uint4 ov;
    __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&ov);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 g = __bfloat1622float2(w2[i]);
      o2[i] = __floats2bfloat162_rn(v[nv][2 * i] * r * g.x, v[nv][2 * i + 1] * r * g.y);
    }
    *reinterpret_cast<uint4*>(out + base + c) = ov;
  }
}

// Skinny linear for single-sequence decode (T <= 4 rows): y[T, N] =
// x[T, K] W[N, K]^T (bf16 in and out, fp32 sums). The token rows sit in
// shared memory; each warp streams one weight row with 16-byte loads (eight
// in flight per lane) and keeps its lane's T partial sums in registers. A
// warp's first weight loads are issued before waiting on the kernel that
// wrote x. (From about 8 rows on, cuBLAS's tensor-core kernels are faster.)
constexpr int kLinThreads = 256;
constexpr int kLinMaxT = 4;
constexpr int kLinUnroll = 8;

__global__ void __launch_bounds__(kLinThreads) linear_small_kernel(
    const __nv_bfloat16* __restrict__ x, int T, int K, const __nv_bfloat16* __restrict__ w, int N,
    __nv_bfloat16* __restrict__ y) {
  extern __shared__ uint4 xs[];  // [T][K / 8]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int kv = K >> 3;
  const int row = blockIdx.x * (kLinThreads / 32) + warp;
  const uint4* wr = reinterpret_cast<const uint4*>(w) + static_cast<size_t>(row < N ? row : 0) * kv;
  uint4 wb[kLinUnroll];
#pragma unroll
  for (int u = 0; u < kLinUnroll; ++u) {
    const int v = lane + 32 * u;
    if (row < N && v < kv) wb[u] = __ldg(wr + v);
  }
  sl::pdl_wait();
  sl::pdl_trigger();
  const uint4* xg = reinterpret_cast<const uint4*>(x);
  for (int i = threadIdx.x; i < T * kv; i += blockDim.x) xs[i] = xg[i];
  __syncthreads();
  if (row >= N) return;
  float2 acc[kLinMaxT];
#pragma unroll
  for (int t = 0; t < kLinMaxT; ++t) acc[t] = make_float2(0.f, 0.f);
  for (int v0 = 0; v0 < kv; v0 += 32 * kLinUnroll) {
    if (v0 > 0) {
#pragma unroll
      for (int u = 0; u < kLinUnroll; ++u) {
        const int v = v0 + lane + 32 * u;
        if (v < kv) wb[u] = __ldg(wr + v);
      }
    }
#pragma unroll
    for (int u = 0; u < kLinUnroll; ++u) {
      const int v = v0 + lane + 32 * u;
      if (v >= kv) break;
      const __nv_bfloat162* w2 = reinterpret_cast<const __nv_bfloat162*>(&wb[u]);
      float2 wf[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) wf[i] = __bfloat1622float2(w2[i]);
#pragma unroll
      for (int t = 0; t < kLinMaxT; ++t) {
        if (t >= T) break;
        const uint4 xv = xs[t * kv + v];
        const __nv_bfloat162* x2 = reinterpret_cast<const __nv_bfloat162*>(&xv);
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[t] = __ffma2_rn(wf[i], __bfloat1622float2(x2[i]), acc[t]);
      }
    }
  }
#pragma unroll
  for (int t = 0; t < kLinMaxT; ++t) {
    if (t >= T) break;
    const float sum = warp_sum(acc[t].x + acc[t].y);
    if (lane == 0) y[static_cast<size_t>(t) * N + row] = __float2bfloat16(sum);
  }
}

}  // namespace

extern "C" int sl_linear_small(const void* x, int T, int K, const void* w, int N, void* y,
                               sl_stream_t stream) {
  if (T < 0 || T > kLinMaxT || K <= 0 || K % 8 || N <= 0) return SL_ERR_INVALID;
  if (T == 0) return SL_OK;
  if (!x || !w || !y) return SL_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w)) & 15) return SL_ERR_INVALID;
  const size_t smem = static_cast<size_t>(T) * K * 2;
  if (smem > 200 * 1024) return SL_ERR_UNSUPPORTED;
  static std::atomic<uint64_t> smem_set{0};
  if (smem > 48 * 1024)
    SL_CUDA_TRY(sl::ensure_smem_limit(linear_small_kernel, 200 * 1024, smem_set));
  const int rows_per_cta = kLinThreads / 32;
  SL_CUDA_TRY(sl::launch(linear_small_kernel, dim3((N + rows_per_cta - 1) / rows_per_cta),
                         dim3(kLinThreads), smem, reinterpret_cast<cudaStream_t>(stream),
                         static_cast<const __nv_bfloat16*>(x), T, K,
                         static_cast<const __nv_bfloat16*>(w), N,
                         static_cast<__nv_bfloat16*>(y)));
  return SL_OK;
}

extern "C" int sl_add_rmsnorm(void* h, const void* delta, const void* w, float eps, void* out,
                              int rows, int H, sl_stream_t stream) {
  if (rows < 0 || H <= 0 || H % 8 || H > 8 * kNormThreads * 4) return SL_ERR_INVALID;
  if (rows == 0) return SL_OK;
  if (!h || !w || !out || rows > 65535 * 32) return SL_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(h) | reinterpret_cast<uintptr_t>(delta) |
       reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(out)) & 15)
    return SL_ERR_INVALID;
  SL_CUDA_TRY(sl::launch(add_rmsnorm_kernel, dim3(rows), dim3(kNormThreads), 0,
                         reinterpret_cast<cudaStream_t>(stream), static_cast<__nv_bfloat16*>(h),
                         static_cast<const __nv_bfloat16*>(delta),
                         static_cast<const __nv_bfloat16*>(w), eps,
                         static_cast<__nv_bfloat16*>(out), H));
  return SL_OK;
}

extern "C" int sl_mla_decode(const void* qkv, int ld_qkv, const void* kv_norm, float eps,
                             const void* w_uk, const void* w_uv, const float* rope_cos_sin,
                             const int64_t* pos, void* cache, int B, int nh, int nope, int rope,
                             int rank, int vdim, int max_len, float scale, void* out,
                             sl_stream_t stream) {
  if (B < 0 || nh <= 0 || nope <= 0 || rope <= 0 || rope % 2 || rank <= 0 || vdim <= 0 ||
      max_len <= 0 || ld_qkv < nh * (nope + rope) + rank + rope)
    return SL_ERR_INVALID;
  // the kernel's lane layout: a 512-wide latent, 16-byte aligned rows, at
  // most two rope columns per lane
  if (rank != kRank || rope > 64 || rope % 32 || nope % 8 || ld_qkv % 8)
    return SL_ERR_UNSUPPORTED;
  if (B == 0) return SL_OK;
  if (!qkv || !kv_norm || !w_uk || !w_uv || !rope_cos_sin || !pos || !cache || !out)
    return SL_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(w_uk) | reinterpret_cast<uintptr_t>(w_uv) |
       reinterpret_cast<uintptr_t>(cache)) & 15)
    return SL_ERR_INVALID;
  const size_t smem = static_cast<size_t>(kRingSlots) * kSlotBytes + kRingSlots * 8 +
      sizeof(float) * (2 * static_cast<size_t>(rank + rope) + kMlaWarps * kRank + nope +
                       2 * kMlaWarps + 32) + sizeof(int) * kRingSlots;
  if (smem > 220 * 1024 || B > 65535) return SL_ERR_UNSUPPORTED;
  static std::atomic<uint64_t> smem_set{0};
  if (smem > 48 * 1024) SL_CUDA_TRY(sl::ensure_smem_limit(mla_decode_kernel, static_cast<int>(smem), smem_set));
  SL_CUDA_TRY(sl::launch(mla_decode_kernel, dim3(nh, B), dim3(kMlaThreads), smem,
                         reinterpret_cast<cudaStream_t>(stream),
                         static_cast<const __nv_bfloat16*>(qkv), ld_qkv,
                         static_cast<const __nv_bfloat16*>(kv_norm), eps,
                         static_cast<const __nv_bfloat16*>(w_uk),
                         static_cast<const __nv_bfloat16*>(w_uv),
                         reinterpret_cast<const float2*>(rope_cos_sin), pos,
                         static_cast<__nv_bfloat16*>(cache), nh, nope, rope, vdim, max_len, scale,
                         static_cast<__nv_bfloat16*>(out)));
  return SL_OK;
}
