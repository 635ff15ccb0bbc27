// Expert-parallel dispatch and combine over NVLink peer memory.
//
// Ranks exchange through symmetric buffers (one allocation per rank, every
// rank holding every peer's address) and per-rank signal pads. Each exchange
// is one kernel per rank:
//   dispatch: push this rank's packed token rows [T, row] into every peer's
//             receive buffer at slot `rank`, signal the peers, wait for every
//             peer's signal, then unpack all ranks' rows into local outputs
//             (hidden rows, top-k weights, top-k ids);
//   combine:  push the fp32 partial rows of each peer's tokens into that
//             peer's receive buffer at slot `rank`, signal, wait, then sum
//             the world's partials for this rank's tokens in rank order and
//             round once to bf16.
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

// One 16-byte vector of this rank's packed row r (hidden bf16 | top-k weights
// f32 | top-k ids i32), read from the three inputs: the hidden part is whole
// vectors; the weight / id tail is assembled word by word (4*topk need not be
// a multiple of 16).
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
    w[j] = word < topk ? __float_as_uint(tw[static_cast<size_t>(r) * topk + word])
                       : static_cast<uint32_t>(ti[static_cast<size_t>(r) * topk + word - topk]);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

__global__ void __launch_bounds__(kEpThreads) ep_dispatch_kernel(
    const __nv_bfloat16* __restrict__ x, const float* __restrict__ tw,
    const int32_t* __restrict__ ti, int T, int row_bytes, EpPeers peers,
    const uint32_t* my_signal, const uint8_t* my_recv,  // written by peers: no .nc loads
    uint32_t* __restrict__ book, int rank, int world, __nv_bfloat16* __restrict__ x_out,
    float* __restrict__ w_out, int32_t* __restrict__ id_out, int H, int topk,
    int32_t* __restrict__ status) {
  sl::pdl_wait();
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(&book[EP_DONE_DISPATCH]) / kEpCtas + 1;
  const size_t half = static_cast<size_t>(world) * T * row_bytes;
  const size_t base = (epoch & 1u) * half + static_cast<size_t>(rank) * T * row_bytes;
  const int rvec = row_bytes / 16;
  const int nvec = T * rvec;
  // pack this rank's rows straight into every peer's receive half
  for (int v = blockIdx.x * blockDim.x + threadIdx.x; v < nvec; v += gridDim.x * blockDim.x) {
    const uint4 val = packed_vec(x, tw, ti, v / rvec, v % rvec, H, topk);
    for (int q = 0; q < world; ++q)
      if (q != rank) reinterpret_cast<uint4*>(peers.recv[q] + base)[v] = val;
  }
  signal_peers(peers, book, EP_DONE_DISPATCH, 0, epoch, rank, world);
  wait_peers(my_signal, 0, epoch, rank, world, status);
  // every rank's rows, this rank's own straight from its inputs
  const uint8_t* half_base = my_recv + (epoch & 1u) * half;
  const int xb = 2 * H, wb = 4 * topk;
  const int n_rows = world * T;
  const int vec_x = xb / 16;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n_rows * vec_x;
       i += gridDim.x * blockDim.x) {
    const int r = i / vec_x, c = i % vec_x;
    const int src_rank = r / T;
    reinterpret_cast<uint4*>(x_out)[i] =
        src_rank == rank
            ? reinterpret_cast<const uint4*>(x + static_cast<size_t>(r % T) * H)[c]
            : reinterpret_cast<const uint4*>(half_base + static_cast<size_t>(r) * row_bytes)[c];
  }
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n_rows * topk;
       i += gridDim.x * blockDim.x) {
    const int r = i / topk, j = i % topk;
    const int src_rank = r / T;
    if (src_rank == rank) {
      w_out[i] = tw[static_cast<size_t>(r % T) * topk + j];
      id_out[i] = ti[static_cast<size_t>(r % T) * topk + j];
    } else {
      const uint8_t* row = half_base + static_cast<size_t>(r) * row_bytes;
      w_out[i] = reinterpret_cast<const float*>(row + xb)[j];
      id_out[i] = reinterpret_cast<const int32_t*>(row + xb + wb)[j];
    }
  }
  sl::pdl_trigger();
}

__global__ void __launch_bounds__(kEpThreads) ep_combine_kernel(
    const float* __restrict__ partial, int T, int H, EpPeers peers,
    const uint32_t* my_signal, const uint8_t* my_recv,  // written by peers: no .nc loads
    uint32_t* __restrict__ book, int rank, int world,
    const __nv_bfloat16* __restrict__ residual, __nv_bfloat16* __restrict__ out,
    int32_t* __restrict__ status) {
  sl::pdl_wait();
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(&book[EP_DONE_COMBINE]) / kEpCtas + 1;
  const size_t slot = static_cast<size_t>(T) * H * 4;  // one rank's rows for one peer
  const size_t half = static_cast<size_t>(world) * slot;
  const int nvec = static_cast<int>(slot / 16);
  for (int q = 0; q < world; ++q) {
    if (q == rank) continue;
    const uint4* src = reinterpret_cast<const uint4*>(partial + static_cast<size_t>(q) * T * H);
    uint4* dst = reinterpret_cast<uint4*>(peers.recv[q] + (epoch & 1u) * half + rank * slot);
    for (int v = blockIdx.x * blockDim.x + threadIdx.x; v < nvec; v += gridDim.x * blockDim.x)
      dst[v] = src[v];
  }
  signal_peers(peers, book, EP_DONE_COMBINE, 1, epoch, rank, world);
  wait_peers(my_signal, 1, epoch, rank, world, status);
  const float* half_base = reinterpret_cast<const float*>(my_recv + (epoch & 1u) * half);
  const float* own = partial + static_cast<size_t>(rank) * T * H;
  const int n = T * H / 4;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int q = 0; q < world; ++q) {  // rank order: deterministic
      const float4 v = q == rank ? reinterpret_cast<const float4*>(own)[i]
                                 : reinterpret_cast<const float4*>(half_base + q * (slot / 4))[i];
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
    if (q < world && (!p->recv[q] || !p->signal[q])) return SL_ERR_INVALID;
  }
  return SL_OK;
}

}  // namespace

extern "C" size_t sl_ep_dispatch_recv_bytes(int world, int T, int H, int topk) {
  if (world < 1 || T < 0 || H <= 0 || topk <= 0) return 0;
  return 2ull * world * T * (2ull * H + 8ull * topk);
}

extern "C" size_t sl_ep_combine_recv_bytes(int world, int T, int H) {
  if (world < 1 || T < 0 || H <= 0) return 0;
  return 2ull * world * T * H * 4ull;
}

extern "C" int sl_ep_dispatch(const void* hidden, const float* topk_weights,
                              const int32_t* topk_ids, int T, int H, int topk, int rank,
                              int world, void* const* peer_recv, void* const* peer_signal,
                              void* book, void* x_out, float* w_out, int32_t* id_out,
                              int32_t* status, sl_stream_t stream) {
  EpPeers peers;
  int rc = fill_peers(&peers, world, peer_recv, peer_signal);
  if (rc != SL_OK) return rc;
  if (!hidden || !topk_weights || !topk_ids || !book || !x_out || !w_out || !id_out ||
      !status || rank < 0 || rank >= world || T <= 0 || H % 8 || topk <= 0 ||
      ((reinterpret_cast<uintptr_t>(hidden) | reinterpret_cast<uintptr_t>(x_out)) & 15))
    return SL_ERR_INVALID;
  const int row_bytes = 2 * H + 8 * topk;
  if (row_bytes % 16) return SL_ERR_UNSUPPORTED;
  SL_CUDA_TRY(sl::launch(ep_dispatch_kernel, dim3(kEpCtas), dim3(kEpThreads), 0,
                         reinterpret_cast<cudaStream_t>(stream),
                         static_cast<const __nv_bfloat16*>(hidden), topk_weights, topk_ids, T,
                         row_bytes, peers,
                         static_cast<const uint32_t*>(peer_signal[rank]),
                         static_cast<const uint8_t*>(peer_recv[rank]),
                         static_cast<uint32_t*>(book), rank, world,
                         static_cast<__nv_bfloat16*>(x_out), w_out, id_out, H, topk, status));
  return SL_OK;
}

extern "C" int sl_ep_combine(const float* partial, int T, int H, int rank, int world,
                             void* const* peer_recv, void* const* peer_signal, void* book,
                             const void* residual, void* out, int32_t* status,
                             sl_stream_t stream) {
  EpPeers peers;
  int rc = fill_peers(&peers, world, peer_recv, peer_signal);
  if (rc != SL_OK) return rc;
  if (!partial || !book || !out || !status || rank < 0 || rank >= world || T <= 0 || H % 8)
    return SL_ERR_INVALID;
  SL_CUDA_TRY(sl::launch(ep_combine_kernel, dim3(kEpCtas), dim3(kEpThreads), 0,
                         reinterpret_cast<cudaStream_t>(stream), partial, T, H, peers,
                         static_cast<const uint32_t*>(peer_signal[rank]),
                         static_cast<const uint8_t*>(peer_recv[rank]),
                         static_cast<uint32_t*>(book), rank, world,
                         static_cast<const __nv_bfloat16*>(residual),
                         static_cast<__nv_bfloat16*>(out), status));
  return SL_OK;
}
