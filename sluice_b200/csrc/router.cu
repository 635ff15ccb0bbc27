// Router: gate GEMV (bf16 logits) and select_experts (softmax / sigmoid,
// optional score bias, grouped top-k, renormalisation, routed scaling).
//
// Reference semantics: vLLM 0.22 fused_moe/router/grouped_topk_router.py:81-166
// and the topk_softmax contract of router/fused_topk_router.py:69-118, as
// called by kfirtoledo/sluice src/sluice/offloader.py:2582-2585.
//
// Two kernels:
//  * gate_kernel: one CTA per expert and tile of 16 tokens; threads split the
//    hidden dimension in 16-byte chunks (fp32 accumulate, CTA reduction);
//    logits rounded to bf16 like the bf16 gate linear.
//  * select_kernel: one warp per token; each lane owns E/32 contiguous
//    experts; scores, group mask and top-k by warp arg-max reductions with
//    ties to the lower expert id.
#include "common.cuh"

namespace {

constexpr int kTokTile = 16;
constexpr int kMaxE = 512;
constexpr int kMaxEPL = kMaxE / 32;

__device__ __forceinline__ void bf16x8_to_f32(const uint4& v, float (&f)[8]) {
  const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(p[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

// One CTA per expert (x a tile of up to kTokTile tokens): the CTA's threads
// split the hidden dimension into 16-byte chunks, so the expert's weight row
// is read once and every token row once per expert, with all loads of a
// thread independent; per-token sums reduce across the CTA.
constexpr int kGateThreads = 128;

__global__ void __launch_bounds__(kGateThreads) gate_kernel(
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
    const float* __restrict__ logit_bias, int T, int H, int E,
    __nv_bfloat16* __restrict__ logits) {
  __shared__ float part[kGateThreads / 32][kTokTile];
  sl::pdl_wait();
  sl::pdl_trigger();
  const int e = blockIdx.x;
  const int t0 = blockIdx.y * kTokTile;
  const int nt = min(kTokTile, T - t0);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float acc[kTokTile];
#pragma unroll
  for (int t = 0; t < kTokTile; ++t) acc[t] = 0.f;
  const uint4* wrow = reinterpret_cast<const uint4*>(w + static_cast<size_t>(e) * H);
  const uint4* xb = reinterpret_cast<const uint4*>(x + static_cast<size_t>(t0) * H);
  const int nvec = H >> 3;
  for (int v = threadIdx.x; v < nvec; v += kGateThreads) {
    float wf[8];
    bf16x8_to_f32(__ldg(wrow + v), wf);
    uint4 xv[kTokTile];
#pragma unroll
    for (int t = 0; t < kTokTile; ++t)
      if (t < nt) xv[t] = __ldg(xb + static_cast<size_t>(t) * nvec + v);
#pragma unroll
    for (int t = 0; t < kTokTile; ++t) {
      if (t < nt) {
        float xf[8];
        bf16x8_to_f32(xv[t], xf);
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[t] = fmaf(wf[i], xf[i], acc[t]);
      }
    }
  }
#pragma unroll
  for (int t = 0; t < kTokTile; ++t) {
    float s = acc[t];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) part[warp][t] = s;
  }
  __syncthreads();
  if (threadIdx.x < nt) {
    float s = 0.f;
#pragma unroll
    for (int q = 0; q < kGateThreads / 32; ++q) s += part[q][threadIdx.x];
    const float b = logit_bias ? logit_bias[e] : 0.f;
    logits[static_cast<size_t>(t0 + threadIdx.x) * E + e] = __float2bfloat16(s + b);
  }
}

// Warp arg-max over (value, id): larger value wins, lower id on ties.
__device__ __forceinline__ void warp_argmax(float& v, int& id) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, id, o);
    if (ov > v || (ov == v && oi < id)) {
      v = ov;
      id = oi;
    }
  }
}

__global__ void __launch_bounds__(128) select_kernel(
    const __nv_bfloat16* __restrict__ logits, int T, int E, int topk, int scoring,
    int n_group, int topk_group, int renorm, float scale,
    const float* __restrict__ score_bias, float* __restrict__ out_w,
    int32_t* __restrict__ out_ids) {
  __shared__ float s_sel[4][kMaxE];
  sl::pdl_wait();
  sl::pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * 4 + warp;
  if (t >= T) return;
  const int epl = E >> 5;  // experts per lane, contiguous
  const int e0 = lane * epl;
  float lg[kMaxEPL], sc[kMaxEPL], sel[kMaxEPL];
  const __nv_bfloat16* row = logits + static_cast<size_t>(t) * E;
#pragma unroll
  for (int i = 0; i < kMaxEPL; ++i)
    lg[i] = (i < epl) ? __bfloat162float(row[e0 + i]) : -INFINITY;

  if (scoring == 0) {  // softmax in fp32
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < kMaxEPL; ++i)
      if (i < epl) m = fmaxf(m, lg[i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxEPL; ++i) {
      sc[i] = (i < epl) ? expf(lg[i] - m) : 0.f;
      s += sc[i];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
#pragma unroll
    for (int i = 0; i < kMaxEPL; ++i) sc[i] = sc[i] / s;
  } else {  // sigmoid
#pragma unroll
    for (int i = 0; i < kMaxEPL; ++i) sc[i] = (i < epl) ? 1.f / (1.f + expf(-lg[i])) : 0.f;
  }
#pragma unroll
  for (int i = 0; i < kMaxEPL; ++i) {
    if (i < epl) {
      // Softmax is monotone in the logit, so rank softmax selections by the
      // exact bf16 logit; biased / sigmoid selections rank by the fp32 score.
      float base = (scoring == 0 && score_bias == nullptr) ? lg[i] : sc[i];
      sel[i] = score_bias ? sc[i] + score_bias[e0 + i] : base;
    } else {
      sel[i] = -INFINITY;
    }
  }

  if (n_group > 1) {
    // group scores: max, or (with a score bias) the sum of the top-2
    float* ss = s_sel[warp];
#pragma unroll
    for (int i = 0; i < kMaxEPL; ++i)
      if (i < epl) ss[e0 + i] = sel[i];
    __syncwarp();
    const int gs = E / n_group;
    float gscore = -INFINITY;
    if (lane < n_group) {
      float b1 = -INFINITY, b2 = -INFINITY;
      for (int j = 0; j < gs; ++j) {
        const float v = ss[lane * gs + j];
        if (v > b1) {
          b2 = b1;
          b1 = v;
        } else if (v > b2) {
          b2 = v;
        }
      }
      gscore = score_bias ? (b1 + b2) : b1;
    }
    uint32_t gmask = 0;
    float gv = gscore;
    for (int r = 0; r < topk_group; ++r) {
      float v = gv;
      int id = (lane < n_group) ? lane : 0x7fffffff;
      warp_argmax(v, id);
      gmask |= 1u << id;
      if (lane == id) gv = -INFINITY;
    }
#pragma unroll
    for (int i = 0; i < kMaxEPL; ++i)
      if (i < epl && !((gmask >> ((e0 + i) / gs)) & 1u)) sel[i] = -INFINITY;
  }

  // top-k, canonical order; lane r keeps the r-th choice
  uint32_t taken = 0;
  float my_w = 0.f;
  int my_id = 0;
  float wsum = 0.f;
  for (int r = 0; r < topk; ++r) {
    float v = -INFINITY;
    int id = 0x7fffffff;
    int li = -1;
#pragma unroll
    for (int i = 0; i < kMaxEPL; ++i) {
      if (i < epl && !((taken >> i) & 1u)) {
        if (li < 0 || sel[i] > v) {
          v = sel[i];
          id = e0 + i;
          li = i;
        }
      }
    }
    warp_argmax(v, id);
    float wv = 0.f;
    if (id >= e0 && id < e0 + epl) {
      const int i = id - e0;
      taken |= 1u << i;
#pragma unroll
      for (int q = 0; q < kMaxEPL; ++q)
        if (q == i) wv = sc[q];
    }
    const int owner = (id / epl) & 31;
    wv = __shfl_sync(0xffffffffu, wv, owner);
    if (lane == r) {
      my_w = wv;
      my_id = id;
    }
    wsum += wv;  // ascending r: the canonical order
  }
  if (lane < topk) {
    float wv = my_w;
    if (renorm) wv = wv / wsum;
    if (scale != 1.f) wv = wv * scale;
    out_w[static_cast<size_t>(t) * topk + lane] = wv;
    out_ids[static_cast<size_t>(t) * topk + lane] = my_id;
  }
}

int check_select_args(int T, int E, int topk, int scoring, int n_group,
                      int topk_group) {
  if (T < 0 || E <= 0 || E % 32 || E > kMaxE) return SL_ERR_UNSUPPORTED;
  if (topk <= 0 || topk > 32 || topk > E) return SL_ERR_INVALID;
  if (scoring != 0 && scoring != 1) return SL_ERR_INVALID;
  if (n_group < 1 || n_group > 32 || E % n_group) return SL_ERR_INVALID;
  if (topk_group < 1 || topk_group > n_group) return SL_ERR_INVALID;
  return SL_OK;
}

}  // namespace

extern "C" int sl_select_experts(const void* router_logits, int T, int E, int topk,
                                 int scoring, int num_expert_group, int topk_group,
                                 int renormalize, float routed_scaling_factor,
                                 const float* score_bias, float* topk_weights,
                                 int32_t* topk_ids, sl_stream_t stream) {
  int st = check_select_args(T, E, topk, scoring, num_expert_group, topk_group);
  if (st != SL_OK) return st;
  if (T == 0) return SL_OK;
  if (!router_logits || !topk_weights || !topk_ids) return SL_ERR_INVALID;
  SL_CUDA_TRY(sl::launch(select_kernel, dim3((T + 3) / 4), dim3(128), 0,
                         reinterpret_cast<cudaStream_t>(stream),
                         static_cast<const __nv_bfloat16*>(router_logits), T, E, topk, scoring,
                         num_expert_group, topk_group, renormalize, routed_scaling_factor,
                         score_bias, topk_weights, topk_ids));
  return SL_OK;
}

extern "C" int sl_gate(const void* hidden, const void* gate_w, const float* logit_bias, int T,
                       int H, int E, void* router_logits_out, sl_stream_t stream) {
  if (T < 0 || E <= 0 || E > 65535) return SL_ERR_INVALID;
  if (H <= 0 || H % 8) return SL_ERR_UNSUPPORTED;
  if (T == 0) return SL_OK;
  if (!hidden || !gate_w || !router_logits_out) return SL_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(hidden) | reinterpret_cast<uintptr_t>(gate_w)) & 15)
    return SL_ERR_INVALID;
  dim3 grid(E, (T + kTokTile - 1) / kTokTile);
  SL_CUDA_TRY(sl::launch(gate_kernel, grid, dim3(kGateThreads), 0,
                         reinterpret_cast<cudaStream_t>(stream),
                         static_cast<const __nv_bfloat16*>(hidden),
                         static_cast<const __nv_bfloat16*>(gate_w), logit_bias, T, H, E,
                         static_cast<__nv_bfloat16*>(router_logits_out)));
  return SL_OK;
}

extern "C" int sl_route(const void* hidden, const void* gate_w, const float* logit_bias,
                        int T, int H, int E, int topk, int scoring,
                        int num_expert_group, int topk_group, int renormalize,
                        float routed_scaling_factor, const float* score_bias,
                        float* topk_weights, int32_t* topk_ids,
                        void* router_logits_out, sl_stream_t stream) {
  int st = check_select_args(T, E, topk, scoring, num_expert_group, topk_group);
  if (st != SL_OK) return st;
  if (H <= 0 || H % 8) return SL_ERR_UNSUPPORTED;
  if (T == 0) return SL_OK;
  if (!hidden || !gate_w || !router_logits_out) return SL_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(hidden) | reinterpret_cast<uintptr_t>(gate_w)) & 15)
    return SL_ERR_INVALID;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  dim3 grid(E, (T + kTokTile - 1) / kTokTile);
  SL_CUDA_TRY(sl::launch(gate_kernel, grid, dim3(kGateThreads), 0, s,
                         static_cast<const __nv_bfloat16*>(hidden),
                         static_cast<const __nv_bfloat16*>(gate_w), logit_bias, T, H, E,
                         static_cast<__nv_bfloat16*>(router_logits_out)));
  return sl_select_experts(router_logits_out, T, E, topk, scoring, num_expert_group,
                           topk_group, renormalize, routed_scaling_factor, score_bias,
                           topk_weights, topk_ids, stream);
}
