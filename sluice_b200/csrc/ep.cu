// Expert-parallel dispatch and combine over NVLink peer memory, routed.
//
// Experts are sharded in contiguous ranges (rank q owns global ids
// [q*G/world, (q+1)*G/world)). Ranks exchange through symmetric buffers (one
// allocation per rank, every rank holding every peer's address) and per-rank
// signal pads. Each exchange is one kernel per rank:
//   dispatch: a token goes to peer q only when one of its top-k ids is owned
//             by q. This rank packs each such token's row (hidden | top-k
//             weights | top-k ids | token index) into q's receive buffer at
//             slot `rank`, rows in token order, writes the row count, signals
//             every peer, waits for every peer's signal and unpacks: its own
//             T tokens first, then the rows each peer sent (rank order); the
//             unused tail rows get id -1 (no expert) and weight 0;
//   combine:  every received row's fp32 partial output goes back to its home
//             rank, at the token's row of slot `rank`; after the signal round
//             each rank sums, per token, its own partial and the partials of
//             the peers the token was sent to (rank order) and rounds once to
//             bf16 (optionally adding the decoder's residual).
// Receive buffers alternate between two halves by a device-side call counter
// (epoch), so a half is only rewritten after every peer has signalled the
// following call, i.e. finished reading it. Signals carry the epoch
// (monotonic, compared wrap-safe). The last CTA to finish pushing signals
// (counted with a monotonic device counter); every wait on a peer is bounded
// and records SL_ERR_TIMEOUT. No CTA waits on another CTA of its own grid.
#include "common.cuh"

namespace {

constexpr int kMaxRanks = 8;
constexpr int kEpThreads = 256;
constexpr int kMaxRoutedTokens = 1024;  // tokens per rank per call
constexpr int kRecvHeader = 128;        // bytes before the rows of a dispatch half

struct EpPeers {
  uint8_t* recv[kMaxRanks];     // each peer's receive buffer base (both halves)
  uint32_t* signal[kMaxRanks];  // each peer's signal pad
};

// per-rank device bookkeeping (a small local buffer, zeroed at set-up): how
// many CTAs finished pushing, summed over every call so far. Every call runs
// kEpCtas CTAs, so a CTA that has not yet counted itself reads
// floor(count / kEpCtas) = the number of completed calls, whatever the other
// CTAs of its own call have done: that is the call's epoch - 1.
enum { EP_DONE_DISPATCH = 0, EP_DONE_COMBINE = 1 };
constexpr int kEpCtas = 8;

__host__ __device__ inline int routed_row_bytes(int H, int topk) {
  return (2 * H + 8 * topk + 4 + 15) & ~15;
}
__host__ __device__ inline size_t dispatch_half_bytes(int world, int T, int H, int topk) {
  return kRecvHeader + static_cast<size_t>(world) * T * routed_row_bytes(H, topk);
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Signal every peer that this rank's pushes of `epoch` are complete, from the
// last CTA of the grid to finish pushing.
__device__ void signal_peers(const EpPeers& peers, uint32_t* book, int done_slot, int channel,
                             uint32_t epoch, int rank, int world) {
  __shared__ int last;
  __threadfence_system();  // every thread's pushes, before the count
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t old = atomicAdd(&book[done_slot], 1u);
    last = ((old + 1) % gridDim.x) == 0;
  }
  __syncthreads();
  if (last && threadIdx.x < world && threadIdx.x != rank) {
    __threadfence_system();
    st_release_sys(&peers.signal[threadIdx.x][channel * kMaxRanks + rank], epoch);
  }
}

// Wait until every peer has signalled `epoch` on `channel` (bounded).
__device__ void wait_peers(const uint32_t* my_signal, int channel, uint32_t epoch, int rank,
                           int world, int32_t* status) {
  __shared__ int timed_out;
  if (threadIdx.x == 0) timed_out = 0;
  __syncthreads();
  if (threadIdx.x < world && threadIdx.x != rank) {
    const uint32_t* p = &my_signal[channel * kMaxRanks + threadIdx.x];
    const uint64_t t0 = sl::globaltimer();
    while (static_cast<int32_t>(ld_acquire_sys(p) - epoch) < 0) {
      if (sl::globaltimer() - t0 > sl::kWaitLimitNs) {
        timed_out = 1;
        break;
      }
    }
  }
  __syncthreads();
  if (timed_out && threadIdx.x == 0) atomicExch(status, SL_ERR_TIMEOUT);
}

// Peers (other than `rank`) owning one of token t's ids, as a bit mask.
__device__ __forceinline__ uint32_t dest_mask(const int32_t* __restrict__ ti, int t, int topk,
                                              int G, int per, int rank) {
  uint32_t m = 0;
  for (int j = 0; j < topk; ++j) {
    const int g = ti[static_cast<size_t>(t) * topk + j];
    if (g >= 0 && g < G) m |= 1u << (g / per);
  }
  return m & ~(1u << rank);
}

// Per-token destination masks and each token's row position in every peer's
// slot (rows in token order), computed by every CTA in shared memory: warp q
// scans peer q's bit over the tokens with warp ballots. Returns via smem:
// mask[T], pos[q * T + t], count[q].
__device__ void route_tokens(const int32_t* __restrict__ ti, int T, int topk, int G, int per,
                             int rank, int world, uint32_t* mask, int* pos, int* count) {
  for (int t = threadIdx.x; t < T; t += blockDim.x) mask[t] = dest_mask(ti, t, topk, G, per, rank);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int q = warp; q < world; q += blockDim.x >> 5) {
    int run = 0;
    for (int t0 = 0; t0 < T; t0 += 32) {
      const int t = t0 + lane;
      const bool b = t < T && ((mask[t] >> q) & 1u);
      const uint32_t bal = __ballot_sync(0xffffffffu, b);
      if (t < T) pos[q * T + t] = b ? run + __popc(bal & ((1u << lane) - 1u)) : -1;
      run += __popc(bal);
    }
    if (lane == 0) count[q] = run;
  }
  __syncthreads();
}

// One 16-byte vector c of this rank's packed row for token r (hidden bf16 |
// top-k weights f32 | top-k ids i32 | token index i32 | zero pad).
__device__ __forceinline__ uint4 packed_vec(const __nv_bfloat16* __restrict__ x,
                                            const float* __restrict__ tw,
                                            const int32_t* __restrict__ ti, int r, int c,
                                            int H, int topk) {
  const int vec_x = H / 8;
  if (c < vec_x) return reinterpret_cast<const uint4*>(x + static_cast<size_t>(r) * H)[c];
  uint32_t w[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int word = (c - vec_x) * 4 + j;  // 4-byte word within the tail
    w[j] = word < topk       ? __float_as_uint(tw[static_cast<size_t>(r) * topk + word])
           : word < 2 * topk ? static_cast<uint32_t>(ti[static_cast<size_t>(r) * topk + word - topk])
           : word == 2 * topk ? static_cast<uint32_t>(r)
                              : 0u;
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

__global__ void __launch_bounds__(kEpThreads) ep_dispatch_kernel(
    const __nv_bfloat16* __restrict__ x, const float* __restrict__ tw,
    const int32_t* __restrict__ ti, int T, int H, int topk, int G, EpPeers peers,
    const uint32_t* my_signal, const uint8_t* my_recv,  // written by peers: no .nc loads
    uint32_t* __restrict__ book, int rank, int world, __nv_bfloat16* __restrict__ x_out,
    float* __restrict__ w_out, int32_t* __restrict__ id_out, int32_t* __restrict__ src_out,
    int32_t* __restrict__ status) {
  extern __shared__ int smem[];
  uint32_t* mask = reinterpret_cast<uint32_t*>(smem);
  int* pos = smem + T;
  __shared__ int count[kMaxRanks];
  __shared__ int base[kMaxRanks];
  sl::pdl_wait();
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(&book[EP_DONE_DISPATCH]) / kEpCtas + 1;
  const int per = G / world;
  const int row_bytes = routed_row_bytes(H, topk);
  const size_t half = dispatch_half_bytes(world, T, H, topk);
  const size_t hb = (epoch & 1u) * half;  // this call's half
  route_tokens(ti, T, topk, G, per, rank, world, mask, pos, count);
  // row counts for every peer (CTA 0), then the rows
  if (blockIdx.x == 0 && threadIdx.x < world && threadIdx.x != rank)
    reinterpret_cast<uint32_t*>(peers.recv[threadIdx.x] + hb)[rank] =
        static_cast<uint32_t>(count[threadIdx.x]);
  const int rvec = row_bytes / 16;
  const size_t slot0 = hb + kRecvHeader + static_cast<size_t>(rank) * T * row_bytes;
  for (int v = blockIdx.x * blockDim.x + threadIdx.x; v < T * rvec; v += gridDim.x * blockDim.x) {
    const int t = v / rvec, c = v % rvec;
    const uint32_t m = mask[t];
    if (!m) continue;
    const uint4 val = packed_vec(x, tw, ti, t, c, H, topk);
    for (int q = 0; q < world; ++q)
      if ((m >> q) & 1u)
        reinterpret_cast<uint4*>(peers.recv[q] + slot0 +
                                 static_cast<size_t>(pos[q * T + t]) * row_bytes)[c] = val;
  }
  signal_peers(peers, book, EP_DONE_DISPATCH, 0, epoch, rank, world);
  wait_peers(my_signal, 0, epoch, rank, world, status);
  // output rows: this rank's tokens, then each peer's rows in rank order
  const uint8_t* half_base = my_recv + hb;
  if (threadIdx.x == 0) {
    int b = T;
    for (int p = 0; p < world; ++p) {
      int n = 0;
      if (p != rank) {
        n = static_cast<int>(reinterpret_cast<const volatile uint32_t*>(half_base)[p]);
        n = n < 0 ? 0 : (n > T ? T : n);  // a peer never sends more than T rows
      }
      count[p] = n;
      base[p] = b;
      b += n;
    }
  }
  __syncthreads();
  const int n_rows = world * T;
  const int vec_x = H / 8;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n_rows * vec_x;
       i += gridDim.x * blockDim.x) {
    const int r = i / vec_x, c = i % vec_x;
    if (r < T) {
      reinterpret_cast<uint4*>(x_out)[i] = reinterpret_cast<const uint4*>(x)[i];
      continue;
    }
    for (int p = 0; p < world; ++p) {
      if (p == rank || r < base[p] || r >= base[p] + count[p]) continue;
      const uint8_t* row = half_base + kRecvHeader +
                           (static_cast<size_t>(p) * T + (r - base[p])) * row_bytes;
      reinterpret_cast<uint4*>(x_out)[i] = reinterpret_cast<const uint4*>(row)[c];
    }
  }
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n_rows * topk;
       i += gridDim.x * blockDim.x) {
    const int r = i / topk, j = i % topk;
    float wv = 0.f;
    int32_t idv = -1, src = -1;
    if (r < T) {
      wv = tw[i];
      idv = ti[i];
      src = (rank << 16) | r;
    } else {
      for (int p = 0; p < world; ++p) {
        if (p == rank || r < base[p] || r >= base[p] + count[p]) continue;
        const uint8_t* row = half_base + kRecvHeader +
                             (static_cast<size_t>(p) * T + (r - base[p])) * row_bytes;
        wv = reinterpret_cast<const float*>(row + 2 * H)[j];
        idv = reinterpret_cast<const int32_t*>(row + 2 * H + 4 * topk)[j];
        const int tok = reinterpret_cast<const int32_t*>(row + 2 * H + 8 * topk)[0];
        src = (p << 16) | (tok & 0xffff);
      }
    }
    w_out[i] = wv;
    id_out[i] = idv;
    if (j == 0) src_out[r] = src;
  }
  sl::pdl_trigger();
}

__global__ void __launch_bounds__(kEpThreads) ep_combine_kernel(
    const float* __restrict__ partial, const int32_t* __restrict__ src,
    const int32_t* __restrict__ ti, int T, int H, int topk, int G, EpPeers peers,
    const uint32_t* my_signal, const uint8_t* my_recv,  // written by peers: no .nc loads
    uint32_t* __restrict__ book, int rank, int world,
    const __nv_bfloat16* __restrict__ residual, __nv_bfloat16* __restrict__ out,
    int32_t* __restrict__ status) {
  sl::pdl_wait();
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(&book[EP_DONE_COMBINE]) / kEpCtas + 1;
  const size_t slot = static_cast<size_t>(T) * H * 4;  // one rank's rows for one peer
  const size_t half = static_cast<size_t>(world) * slot;
  const size_t hb = (epoch & 1u) * half;
  const int per = G / world;
  const int hvec = H / 4;  // float4 vectors per row
  // every received row's partial back to its home rank, at its token's row
  const int n_recv = (world - 1) * T;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n_recv * hvec;
       i += gridDim.x * blockDim.x) {
    const int r = T + i / hvec, c = i % hvec;
    const int s = src[r];
    if (s < 0) continue;
    const int p = s >> 16, tok = s & 0xffff;
    if (p == rank || p >= world || tok >= T) continue;
    reinterpret_cast<float4*>(peers.recv[p] + hb + rank * slot)[static_cast<size_t>(tok) * hvec + c] =
        reinterpret_cast<const float4*>(partial)[static_cast<size_t>(r) * hvec + c];
  }
  signal_peers(peers, book, EP_DONE_COMBINE, 1, epoch, rank, world);
  wait_peers(my_signal, 1, epoch, rank, world, status);
  const float* half_base = reinterpret_cast<const float*>(my_recv + hb);
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < T * hvec;
       i += gridDim.x * blockDim.x) {
    const int t = i / hvec;
    const uint32_t m = dest_mask(ti, t, topk, G, per, rank);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int q = 0; q < world; ++q) {  // rank order: deterministic
      float4 v;
      if (q == rank) {
        v = reinterpret_cast<const float4*>(partial)[i];
      } else if ((m >> q) & 1u) {
        v = reinterpret_cast<const float4*>(half_base + q * (slot / 4))[i];
      } else {
        continue;
      }
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    __nv_bfloat162* o = reinterpret_cast<__nv_bfloat162*>(out) + 2 * i;
    __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y);
    __nv_bfloat162 hi = __floats2bfloat162_rn(acc.z, acc.w);
    if (residual != nullptr) {
      // the decoder's residual add: bf16(h + bf16(moe)), as a bf16 tensor add
      const __nv_bfloat162* r2 = reinterpret_cast<const __nv_bfloat162*>(residual) + 2 * i;
      const float2 a = __bfloat1622float2(lo), b = __bfloat1622float2(hi);
      const float2 ra = __bfloat1622float2(r2[0]), rb = __bfloat1622float2(r2[1]);
      lo = __floats2bfloat162_rn(ra.x + a.x, ra.y + a.y);
      hi = __floats2bfloat162_rn(rb.x + b.x, rb.y + b.y);
    }
    o[0] = lo;
    o[1] = hi;
  }
  sl::pdl_trigger();
}

int fill_peers(EpPeers* p, int world, void* const* recv, void* const* signal) {
  if (world < 1 || world > kMaxRanks || !recv || !signal) return SL_ERR_INVALID;
  for (int q = 0; q < kMaxRanks; ++q) {
    p->recv[q] = q < world ? static_cast<uint8_t*>(recv[q]) : nullptr;
    p->signal[q] = q < world ? static_cast<uint32_t*>(signal[q]) : nullptr;
    if (q < world && (!p->recv[q] || !p->signal[q] ||
                      (reinterpret_cast<uintptr_t>(recv[q]) & 15)))
      return SL_ERR_INVALID;
  }
  return SL_OK;
}

int check_routing(int T, int H, int topk, int global_n, int rank, int world) {
  if (rank < 0 || rank >= world || T <= 0 || H <= 0 || H % 8 || topk <= 0 || global_n <= 0)
    return SL_ERR_INVALID;
  if (T > kMaxRoutedTokens || global_n % world) return SL_ERR_UNSUPPORTED;
  return SL_OK;
}

}  // namespace

extern "C" size_t sl_ep_dispatch_recv_bytes(int world, int T, int H, int topk) {
  if (world < 1 || T < 0 || H <= 0 || topk <= 0) return 0;
  return 2 * dispatch_half_bytes(world, T, H, topk);
}

extern "C" size_t sl_ep_combine_recv_bytes(int world, int T, int H) {
  if (world < 1 || T < 0 || H <= 0) return 0;
  return 2ull * world * T * H * 4ull;
}

extern "C" int sl_ep_dispatch(const void* hidden, const float* topk_weights,
                              const int32_t* topk_ids, int T, int H, int topk, int global_n,
                              int rank, int world, void* const* peer_recv,
                              void* const* peer_signal, void* book, void* x_out, float* w_out,
                              int32_t* id_out, int32_t* src_out, int32_t* status,
                              sl_stream_t stream) {
  EpPeers peers;
  int rc = fill_peers(&peers, world, peer_recv, peer_signal);
  if (rc != SL_OK) return rc;
  rc = check_routing(T, H, topk, global_n, rank, world);
  if (rc != SL_OK) return rc;
  if (!hidden || !topk_weights || !topk_ids || !book || !x_out || !w_out || !id_out ||
      !src_out || !status ||
      ((reinterpret_cast<uintptr_t>(hidden) | reinterpret_cast<uintptr_t>(x_out)) & 15))
    return SL_ERR_INVALID;
  const size_t smem = sizeof(int) * static_cast<size_t>(T) * (1 + world);
  SL_CUDA_TRY(sl::launch(ep_dispatch_kernel, dim3(kEpCtas), dim3(kEpThreads), smem,
                         reinterpret_cast<cudaStream_t>(stream),
                         static_cast<const __nv_bfloat16*>(hidden), topk_weights, topk_ids, T,
                         H, topk, global_n, peers,
                         static_cast<const uint32_t*>(peer_signal[rank]),
                         static_cast<const uint8_t*>(peer_recv[rank]),
                         static_cast<uint32_t*>(book), rank, world,
                         static_cast<__nv_bfloat16*>(x_out), w_out, id_out, src_out, status));
  return SL_OK;
}

extern "C" int sl_ep_combine(const float* partial, const int32_t* src,
                             const int32_t* topk_ids, int T, int H, int topk, int global_n,
                             int rank, int world, void* const* peer_recv,
                             void* const* peer_signal, void* book, const void* residual,
                             void* out, int32_t* status, sl_stream_t stream) {
  EpPeers peers;
  int rc = fill_peers(&peers, world, peer_recv, peer_signal);
  if (rc != SL_OK) return rc;
  rc = check_routing(T, H, topk, global_n, rank, world);
  if (rc != SL_OK) return rc;
  if (!partial || !src || !topk_ids || !book || !out || !status ||
      ((reinterpret_cast<uintptr_t>(partial) | reinterpret_cast<uintptr_t>(out) |
        reinterpret_cast<uintptr_t>(residual)) & 15))
    return SL_ERR_INVALID;
  SL_CUDA_TRY(sl::launch(ep_combine_kernel, dim3(kEpCtas), dim3(kEpThreads), 0,
                         reinterpret_cast<cudaStream_t>(stream), partial, src, topk_ids, T, H,
                         topk, global_n, peers,
                         static_cast<const uint32_t*>(peer_signal[rank]),
                         static_cast<const uint8_t*>(peer_recv[rank]),
                         static_cast<uint32_t*>(book), rank, world,
                         static_cast<const __nv_bfloat16*>(residual),
                         static_cast<__nv_bfloat16*>(out), status));
  return SL_OK;
}
