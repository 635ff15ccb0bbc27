// Layout of one layer's device slot-cache state block (see
// sl_slot_state_offsets in include/sluice_b200.h), shared by the planner,
// the streamer and the fused-experts align step (which reads the fill list).
#pragma once

#include <stddef.h>
#include <stdint.h>

#include "../../include/sluice_b200.h"

namespace {

__host__ __device__ inline size_t round16(size_t v) { return (v + 15) & ~size_t(15); }

__host__ __device__ inline void state_layout(int S, int G, int L, size_t* off) {
  size_t o = 0;
  off[0] = o; o += round16(16 * 4);           // header
  off[1] = o; o += round16(16 * 8);           // counters
  off[2] = o; o += round16(size_t(G) * 4);    // local_of
  off[3] = o; o += round16(size_t(L) * 4);    // global_of_local
  off[4] = o; o += round16(size_t(L) * 4);    // slot_of
  off[5] = o; o += round16(size_t(S) * 4);    // expert_in_slot
  off[6] = o; o += round16(size_t(S));        // seg
  off[7] = o; o += round16(size_t(S) * 4);    // stamp
  off[8] = o; o += round16(size_t(S) * 4);    // free_stack
  off[9] = o; o += round16(size_t(S) * 4);    // fill_local
  off[10] = o; o += round16(size_t(S) * 4);   // fill_slot
  off[11] = o; o += round16(size_t(L) * 4);   // freq (LFU counts)
  off[12] = o;
}

struct StateView {
  int32_t* hdr;
  unsigned long long* cnt;
  int32_t* local_of;
  int32_t* global_of_local;
  int32_t* slot_of;
  int32_t* eis;
  uint8_t* seg;
  uint32_t* stamp;
  int32_t* free_stack;
  int32_t* fill_local;
  int32_t* fill_slot;
  uint32_t* freq;
};

__device__ inline StateView view(uint8_t* base, int S, int G, int L) {
  size_t off[13];
  state_layout(S, G, L, off);
  StateView v;
  v.hdr = reinterpret_cast<int32_t*>(base + off[0]);
  v.cnt = reinterpret_cast<unsigned long long*>(base + off[1]);
  v.local_of = reinterpret_cast<int32_t*>(base + off[2]);
  v.global_of_local = reinterpret_cast<int32_t*>(base + off[3]);
  v.slot_of = reinterpret_cast<int32_t*>(base + off[4]);
  v.eis = reinterpret_cast<int32_t*>(base + off[5]);
  v.seg = base + off[6];
  v.stamp = reinterpret_cast<uint32_t*>(base + off[7]);
  v.free_stack = reinterpret_cast<int32_t*>(base + off[8]);
  v.fill_local = reinterpret_cast<int32_t*>(base + off[9]);
  v.fill_slot = reinterpret_cast<int32_t*>(base + off[10]);
  v.freq = reinterpret_cast<uint32_t*>(base + off[11]);
  return v;
}

__device__ inline StateView view_from_header(uint8_t* base, int& S, int& G, int& L) {
  const int32_t* h = reinterpret_cast<const int32_t*>(base);
  S = h[SL_HDR_NUM_SLOTS];
  G = h[SL_HDR_GLOBAL_N];
  L = h[SL_HDR_LOCAL_N];
  return view(base, S, G, L);
}

// Wave plan of a step beyond the envelope (sl_plan_waves), in int32 words:
// header, fill count per wave, fill lists per wave ([max_waves][S] locals and
// slots), one expert map per wave ([max_waves][G]). Fields start on 16 bytes.
__host__ __device__ inline void wave_layout(int S, int G, int MW, size_t* off) {
  const size_t r = ~size_t(3);
  size_t o = 0;
  off[0] = o; o += 16;                              // header (SL_WAVE_HDR_*)
  off[1] = o; o += (size_t(MW) + 3) & r;            // fill_count
  off[2] = o; o += (size_t(MW) * S + 3) & r;        // fill_local
  off[3] = o; o += (size_t(MW) * S + 3) & r;        // fill_slot
  off[4] = o; o += (size_t(MW) * G + 3) & r;        // map
  off[5] = o;
}

struct WaveView {
  int32_t* hdr;
  int32_t* count;
  int32_t* loc;   // wave k at loc + k * S
  int32_t* slot;
  int32_t* map;   // wave k at map + k * G
};

__host__ __device__ inline WaveView wave_view(int32_t* base, int S, int G, int MW) {
  size_t off[6];
  wave_layout(S, G, MW, off);
  return WaveView{base + off[0], base + off[1], base + off[2], base + off[3], base + off[4]};
}

}  // namespace
