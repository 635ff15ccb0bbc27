/* A C host of the library (what a cgo / JNI / plain C caller links against):
 * the calls that need no GPU — version, status text, state and wave-plan
 * layouts, workspace sizes and argument checks. Exits 0 when all hold. */
#include <stdio.h>
#include <string.h>

#include "sluice_b200.h"

#define EXPECT(cond)                                        \
  do {                                                      \
    if (!(cond)) {                                          \
      fprintf(stderr, "failed: %s (line %d)\n", #cond, __LINE__); \
      return 1;                                             \
    }                                                       \
  } while (0)

int main(void) {
  size_t st[SL_STATE_NFIELDS + 1], wv[SL_WAVE_NFIELDS + 1];
  EXPECT(sl_version() >= 100);
  EXPECT(strcmp(sl_status_string(SL_OK), "ok") == 0);
  EXPECT(sl_slot_state_offsets(48, 64, 64, st) == SL_OK);
  EXPECT(st[SL_STATE_NFIELDS] == sl_slot_state_bytes(48, 64, 64));
  EXPECT(sl_wave_plan_offsets(48, 64, 5, wv) == SL_OK);
  EXPECT(wv[SL_WAVE_NFIELDS] == sl_wave_plan_bytes(48, 64, 5));
  EXPECT(sl_fused_experts_workspace_bytes(8, 6, 2048, 1408, 48, 2) > 0);
  EXPECT(sl_ep_combine_recv_bytes(2, 8, 2048) == 2u * 2u * 8u * 2048u * 4u);
  /* refused before any device work */
  EXPECT(sl_plan_slots(NULL, NULL, 0, NULL, NULL) == SL_ERR_INVALID);
  EXPECT(sl_plan_waves(NULL, NULL, 8, 6, 0, NULL, NULL, NULL) == SL_ERR_INVALID);
  EXPECT(sl_stream_wave(NULL, 0, 2, NULL, NULL, NULL, NULL, 0, NULL) == SL_ERR_INVALID);
  EXPECT(sl_wave_plan_init(NULL, 48, 64, 5, NULL) == SL_ERR_INVALID);
  /* phased fused experts: parts 0..SL_PHASE_COMBINE only */
  EXPECT(sl_fused_experts_phase(NULL, 4, 2048, 1408, NULL, NULL, 8, SL_WEIGHTS_BF16, NULL, NULL,
                                2, NULL, 0, NULL, NULL, 0, 1.0f, NULL, SL_PHASE_COMBINE + 1,
                                NULL, NULL, 0, NULL) == SL_ERR_INVALID);
  printf("c host ok: library version %d\n", sl_version());
  return 0;
}
