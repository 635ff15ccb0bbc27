// fused_experts for callers that cannot allocate device memory.
//
// Some callers of this library have no way to obtain device scratch memory
// for a call: a host program binding the C ABI directly (cgo, JNI, ctypes
// without torch) has no caching allocator to borrow from, and a serving
// process that has already handed almost all of HBM to its own memory pool
// (KV cache, activation arena) sees cudaMalloc fail, or pays for the implicit
// device synchronisation cudaMalloc can cause in the middle of a decode step.
// This entry point gives them the same computation as sl_fused_experts with
// its scratch taken from one fixed, file-scope device array instead of a
// caller-provided workspace.
//
// Limits and sharing rules:
//  * The scratch is kNoAllocScratchBytes (32 MiB) per device; it exists on
//    every GPU that loads this library until the process exits. Problems whose
//    workspace (sl_fused_experts_workspace_bytes) exceeds it are rejected with
//    SL_ERR_NO_SCRATCH before anything is launched.
//  * All calls on a device share the one array. Calls that may overlap on the
//    GPU (different streams without ordering between them) race on it and
//    corrupt each other's results; order them on one stream.
//  * The array keeps the previous call's contents. The first 256 bytes (the
//    status word and work counts) are cleared with cudaMemsetAsync on the
//    caller's stream at the start of every call; the rest is rewritten by the
//    call before it is read (rows that are never consumed may keep old data).
//  * The first call on each device looks up the array's device address with
//    cudaGetSymbolAddress while that device is current; make that first call
//    before any stream capture. Nothing here calls cudaMalloc, cudaFree or an
//    allocating library routine.
#include <mutex>

#include "common.cuh"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;
constexpr int kNoAllocMaxDevices = 64;

// In host code this name is a host-side stand-in, not a device address: only
// the pointer from cudaGetSymbolAddress may be handed to kernels.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

void* g_scratch_dev[kNoAllocMaxDevices] = {nullptr};
std::mutex g_scratch_mu;

// Device address of this device's scratch array (looked up once per device).
int scratch_for_current_device(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return SL_ERR_CUDA;
  if (dev < 0 || dev >= kNoAllocMaxDevices) return SL_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_dev[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      (void)cudaGetLastError();
      return SL_ERR_CUDA;
    }
    g_scratch_dev[dev] = p;
  }
  *out = g_scratch_dev[dev];
  return SL_OK;
}

__global__ void copy_status_kernel(const int32_t* scratch_status, int32_t* status_out) {
  *status_out = *scratch_status;
}

}  // namespace

extern "C" int sl_fused_experts_noalloc(const void* hidden, int T, int H, int I,
                                        const void* w13, const void* w2, int num_slots,
                                        int weight_dtype, const float* topk_weights,
                                        const int32_t* topk_ids, int topk,
                                        const int32_t* expert_map, int global_n,
                                        const void* shared_w13, const void* shared_w2,
                                        int n_shared, float routed_scaling_factor, void* out,
                                        int32_t* status_out, sl_stream_t stream) {
  // Every argument is checked before anything is enqueued, so an error return
  // leaves the stream, the scratch and status_out untouched.
  if (weight_dtype != SL_WEIGHTS_BF16) return SL_ERR_UNSUPPORTED;
  const size_t need =
      sl_fused_experts_workspace_bytes(T, topk, H, I, num_slots, n_shared);
  if (need == 0) return SL_ERR_INVALID;
  if (need > kNoAllocScratchBytes) return SL_ERR_NO_SCRATCH;
  void* scratch = nullptr;
  int rc = scratch_for_current_device(&scratch);
  if (rc != SL_OK) return rc;
  sl_expert_weights w = {};
  w.w13 = w13;
  w.w2 = w2;
  w.num_slots = num_slots;
  w.shared_w13 = shared_w13;
  w.shared_w2 = shared_w2;
  w.n_shared = n_shared;
  w.dtype = SL_WEIGHTS_BF16;
  rc = sl::fused_experts_check(hidden, T, H, I, w, topk_weights, topk_ids, topk, expert_map,
                               global_n, 0, T, out, 0, scratch, kNoAllocScratchBytes, nullptr,
                               -1);
  if (rc != SL_OK) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (T == 0) {  // nothing to compute: report success
    if (status_out != nullptr && cudaMemsetAsync(status_out, 0, sizeof(int32_t), st) != cudaSuccess) {
      (void)cudaGetLastError();
      return SL_ERR_CUDA;
    }
    return SL_OK;
  }
  if (cudaMemsetAsync(scratch, 0, 256, st) != cudaSuccess) {
    (void)cudaGetLastError();
    return SL_ERR_CUDA;
  }
  rc = sl_fused_experts(hidden, T, H, I, w13, w2, num_slots, weight_dtype, topk_weights,
                        topk_ids, topk, expert_map, global_n, shared_w13, shared_w2, n_shared,
                        routed_scaling_factor, out, scratch, kNoAllocScratchBytes, stream);
  if (rc != SL_OK || status_out == nullptr) return rc;
  copy_status_kernel<<<1, 1, 0, st>>>(static_cast<const int32_t*>(scratch), status_out);
  SL_LAUNCH_CHECK();
  return SL_OK;
}
