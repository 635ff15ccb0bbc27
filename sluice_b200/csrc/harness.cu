// Decoder-harness kernel: the absorbed multi-head latent attention (MLA) of
// one decode step, for the DeepSeek-V2-Lite-shaped decoder that wraps the MoE
// layers in the benchmark. It is not part of the reference's MoE operator
// surface; it replaces a dozen small PyTorch kernels per layer (norm, rotary
// embedding, cache write, the absorbed query, scores, softmax, the weighted
// latent sum and the value map) with one launch.
//
// One CTA per (head, sequence). Inputs per sequence: the fused projection row
// [q (heads x (nope + rope)) | c_kv (rank) | k_pe (rope)] of this step, its
// position P; the latent cache [B, max_len, rank + rope]. The CTA:
//   1. normalises c_kv (RMSNorm, fp32, one bf16 rounding) and rotates k_pe
//      (RoPE on adjacent pairs) for position P; CTA head 0 writes them to the
//      cache (the other heads use their own copy for position P);
//   2. forms the absorbed query [q_nope W_uk | rope(q_pe)] (fp32 sums, bf16
//      rounding, as the bf16 GEMM it replaces);
//   3. scores every cached position 0..P (a warp per position), softmax;
//   4. sums the latents weighted by the probabilities, maps through W_uv.
#include "common.cuh"

namespace {

constexpr int kMlaThreads = 256;

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

__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = -INFINITY;
  for (int i = 0; i < nw; ++i) t = fmaxf(t, red[i]);
  return t;
}

__global__ void __launch_bounds__(kMlaThreads) mla_decode_kernel(
    const __nv_bfloat16* __restrict__ qkv, int ld_qkv, const __nv_bfloat16* __restrict__ kv_norm,
    float eps, const __nv_bfloat16* __restrict__ w_uk, const __nv_bfloat16* __restrict__ w_uv,
    const float2* __restrict__ rope_cs, const int64_t* __restrict__ pos,
    __nv_bfloat16* __restrict__ cache, int nh, int nope, int rope, int rank, int vdim,
    int max_len, float scale, __nv_bfloat16* __restrict__ out) {
  extern __shared__ float sm[];
  const int h = blockIdx.x, b = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
  const int dk = rank + rope;
  float* q = sm;            // [dk] absorbed query
  float* kv = q + dk;       // [dk] this position's latent | rotated k_pe
  float* p = kv + dk;       // [max_len] scores, then probabilities
  float* ol = p + max_len;  // [rank] probability-weighted latent
  float* red = ol + rank;   // [32]
  sl::pdl_wait();
  sl::pdl_trigger();
  int P = static_cast<int>(pos[b]);
  P = P < 0 ? 0 : (P >= max_len ? max_len - 1 : P);
  const __nv_bfloat16* row = qkv + static_cast<size_t>(b) * ld_qkv;
  const __nv_bfloat16* qh = row + h * (nope + rope);
  const __nv_bfloat16* ckv = row + nh * (nope + rope);
  const float2* cs = rope_cs + static_cast<size_t>(P) * (rope / 2);

  // 1. RMSNorm of c_kv and the rotated k_pe for position P
  float ss = 0.f;
  for (int i = tid; i < rank; i += blockDim.x) {
    const float v = __bfloat162float(ckv[i]);
    kv[i] = v;
    ss += v * v;
  }
  const float r = rsqrtf(block_sum(ss, red) / rank + eps);
  for (int i = tid; i < rank; i += blockDim.x)
    kv[i] = sl::bf16_round(kv[i] * r * __bfloat162float(kv_norm[i]));
  for (int j = tid; j < rope / 2; j += blockDim.x) {
    const float x0 = __bfloat162float(ckv[rank + 2 * j]), x1 = __bfloat162float(ckv[rank + 2 * j + 1]);
    const float2 c = cs[j];
    kv[rank + 2 * j] = sl::bf16_round(x0 * c.x - x1 * c.y);
    kv[rank + 2 * j + 1] = sl::bf16_round(x1 * c.x + x0 * c.y);
    const float y0 = __bfloat162float(qh[nope + 2 * j]), y1 = __bfloat162float(qh[nope + 2 * j + 1]);
    q[rank + 2 * j] = sl::bf16_round(y0 * c.x - y1 * c.y);
    q[rank + 2 * j + 1] = sl::bf16_round(y1 * c.x + y0 * c.y);
  }
  __syncthreads();
  if (h == 0) {
    __nv_bfloat16* dst = cache + (static_cast<size_t>(b) * max_len + P) * dk;
    for (int i = tid; i < dk; i += blockDim.x) dst[i] = __float2bfloat16(kv[i]);
  }
  // 2. absorbed query: q_lat[c] = sum_d q_nope[d] W_uk[h][d][c]
  const __nv_bfloat16* wk = w_uk + static_cast<size_t>(h) * nope * rank;
  for (int c = tid; c < rank; c += blockDim.x) {
    float acc = 0.f;
    for (int d = 0; d < nope; ++d)
      acc = fmaf(__bfloat162float(qh[d]), __bfloat162float(wk[static_cast<size_t>(d) * rank + c]),
                 acc);
    q[c] = sl::bf16_round(acc);
  }
  __syncthreads();
  // 3. scores over positions 0..P (a warp per position), softmax
  const __nv_bfloat16* cb = cache + static_cast<size_t>(b) * max_len * dk;
  for (int l = warp; l <= P; l += nw) {
    float acc = 0.f;
    if (l == P) {
      for (int i = lane; i < dk; i += 32) acc = fmaf(q[i], kv[i], acc);
    } else {
      const __nv_bfloat16* key = cb + static_cast<size_t>(l) * dk;
      for (int i = lane; i < dk; i += 32) acc = fmaf(q[i], __bfloat162float(key[i]), acc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) p[l] = acc * scale;
  }
  __syncthreads();
  float m = -INFINITY;
  for (int l = tid; l <= P; l += blockDim.x) m = fmaxf(m, p[l]);
  m = block_max(m, red);
  float se = 0.f;
  for (int l = tid; l <= P; l += blockDim.x) {
    const float e = __expf(p[l] - m);
    p[l] = e;
    se += e;
  }
  const float inv = 1.f / block_sum(se, red);
  // 4. probability-weighted latent, then the value map
  for (int c = tid; c < rank; c += blockDim.x) {
    float acc = 0.f;
    for (int l = 0; l < P; ++l)
      acc = fmaf(p[l], __bfloat162float(cb[static_cast<size_t>(l) * dk + c]), acc);
    acc = fmaf(p[P], kv[c], acc);
    ol[c] = sl::bf16_round(acc * inv);
  }
  __syncthreads();
  const __nv_bfloat16* wv = w_uv + static_cast<size_t>(h) * vdim * rank;
  for (int d = warp; d < vdim; d += nw) {
    float acc = 0.f;
    for (int c = lane; c < rank; c += 32)
      acc = fmaf(ol[c], __bfloat162float(wv[static_cast<size_t>(d) * rank + c]), acc);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) out[static_cast<size_t>(b) * nh * vdim + h * vdim + d] = __float2bfloat16(acc);
  }
}

}  // namespace

extern "C" int sl_mla_decode(const void* qkv, int ld_qkv, const void* kv_norm, float eps,
                             const void* w_uk, const void* w_uv, const float* rope_cos_sin,
                             const int64_t* pos, void* cache, int B, int nh, int nope, int rope,
                             int rank, int vdim, int max_len, float scale, void* out,
                             sl_stream_t stream) {
  if (B < 0 || nh <= 0 || nope <= 0 || rope <= 0 || rope % 2 || rank <= 0 || vdim <= 0 ||
      max_len <= 0 || ld_qkv < nh * (nope + rope) + rank + rope)
    return SL_ERR_INVALID;
  if (B == 0) return SL_OK;
  if (!qkv || !kv_norm || !w_uk || !w_uv || !rope_cos_sin || !pos || !cache || !out)
    return SL_ERR_INVALID;
  const size_t smem = sizeof(float) * (2 * static_cast<size_t>(rank + rope) + max_len + rank + 32);
  if (smem > 200 * 1024 || B > 65535) return SL_ERR_UNSUPPORTED;
  static std::atomic<uint64_t> smem_set{0};
  if (smem > 48 * 1024) SL_CUDA_TRY(sl::ensure_smem_limit(mla_decode_kernel, static_cast<int>(smem), smem_set));
  SL_CUDA_TRY(sl::launch(mla_decode_kernel, dim3(nh, B), dim3(kMlaThreads), smem,
                         reinterpret_cast<cudaStream_t>(stream),
                         static_cast<const __nv_bfloat16*>(qkv), ld_qkv,
                         static_cast<const __nv_bfloat16*>(kv_norm), eps,
                         static_cast<const __nv_bfloat16*>(w_uk),
                         static_cast<const __nv_bfloat16*>(w_uv),
                         reinterpret_cast<const float2*>(rope_cos_sin), pos,
                         static_cast<__nv_bfloat16*>(cache), nh, nope, rope, rank, vdim, max_len,
                         scale, static_cast<__nv_bfloat16*>(out)));
  return SL_OK;
}
