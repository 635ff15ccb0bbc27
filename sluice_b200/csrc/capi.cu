// Library-level entry points: status strings, version, device properties.
#include <stdlib.h>

#include "common.cuh"

namespace {
constexpr int kMaxDevices = 64;
int g_sm_count[kMaxDevices] = {0};
}  // namespace

extern "C" const char* sl_status_string(int status) {
  switch (status) {
    case SL_OK: return "ok";
    case SL_ERR_OVERFLOW:
      return "Sluice router-split: working set exceeds slots on a decode-sized step; "
             "raise SLUICE_SLOTS.";
    case SL_ERR_INVALID: return "invalid argument";
    case SL_ERR_CUDA: return "CUDA runtime error";
    case SL_ERR_UNSUPPORTED: return "shape or dtype not supported by this build";
    case SL_ERR_TIMEOUT: return "a bounded device wait ran out";
    case SL_ERR_NO_SCRATCH:
      return "problem needs more than the 32 MiB static scratch of sl_fused_experts_noalloc; "
             "use sl_fused_experts with a caller workspace";
    default: return "unknown status";
  }
}

extern "C" int sl_version(void) { return 100; }

// PDL on unless SLUICE_PDL=0 in the environment (read once).
bool sl::pdl_enabled() {
  static const bool on = [] {
    const char* v = getenv("SLUICE_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

extern "C" int sl_device_sm_count(void) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 0;
  if (g_sm_count[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    g_sm_count[dev] = n;
  }
  return g_sm_count[dev];
}
