/*
 * sluice_b200 — C ABI of the B200 (sm_100a) MoE expert-offload hot path.
 *
 * Every entry point takes plain device / host pointers and sizes, enqueues
 * its kernels on the caller's CUDA stream and returns an int status (SL_OK on
 * success). No call synchronises the stream, so every call can be captured in
 * a CUDA graph. Conditions found on the device (slot overflow, a bounded wait
 * that ran out) are written to a device status word that the caller reads
 * outside capture (sl_slot_state_offsets / the fused-experts workspace).
 *
 * Tensor layouts (row-major, last dim contiguous):
 *   hidden        bf16 [T, H]
 *   gate_w        bf16 [E, H]
 *   w13 slots     bf16 [num_slots, 2*I, H]   (gate rows, then up rows)
 *   w2 slots      bf16 [num_slots, H, I]
 *   topk_weights  f32  [T, topk];  topk_ids  i32 [T, topk]
 *   expert_map    i32  [global_n]  (global id -> slot, -1 = not resident)
 *
 * Each declaration names the reference interface it replaces
 * (kfirtoledo/sluice, paths inside that project; vLLM paths are the
 * third-party code the reference calls, vLLM 0.22 as installed here).
 */
#ifndef SLUICE_B200_H
#define SLUICE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* sl_stream_t; /* a cudaStream_t */

enum {
  SL_OK = 0,
  SL_ERR_OVERFLOW = 1,    /* working set exceeds slots (offloader.py:2456-2460) */
  SL_ERR_INVALID = 2,     /* bad argument */
  SL_ERR_CUDA = 3,        /* CUDA runtime error */
  SL_ERR_UNSUPPORTED = 4, /* shape / dtype this build does not cover */
  SL_ERR_TIMEOUT = 5,     /* a bounded device wait ran out */
  SL_ERR_NO_SCRATCH = 6   /* problem too large for sl_fused_experts_noalloc */
};

/* Human-readable text for a status code. */
const char* sl_status_string(int status);
/* Library ABI version (major*100 + minor). */
int sl_version(void);
/* Number of SMs of the current device (used to size persistent grids). */
int sl_device_sm_count(void);

/* ------------------------------------------------------------------ router
 * Replaces runner.gate(hs) + router.select_experts(...)
 *   src/sluice/offloader.py:2582-2585 (router-split entry);
 *   vLLM fused_moe/router/base_router.py:250-298 (select_experts),
 *   router/grouped_topk_router.py:81-166 (grouped_topk),
 *   router/fused_topk_router.py:69-118 (topk_softmax contract).
 * logits = bf16(hidden @ gate_w^T + logit_bias); scores = softmax or sigmoid
 * (fp32); optional score_bias (e_score_correction_bias) for selection only;
 * num_expert_group/topk_group group mask (1/1 = no grouping); top-k with
 * ties to the lower id; optional renormalisation; routed_scaling_factor.
 * Outputs are ordered by selection score descending, id ascending.
 * scoring: 0 = softmax, 1 = sigmoid. router_logits_out (bf16 [T,E]) receives
 * the logits. Limits: E % 32 == 0, E <= 512, H % 8 == 0, topk <= 32. */
int sl_route(const void* hidden, const void* gate_w, const float* logit_bias,
             int T, int H, int E, int topk, int scoring, int num_expert_group,
             int topk_group, int renormalize, float routed_scaling_factor,
             const float* score_bias, float* topk_weights, int32_t* topk_ids,
             void* router_logits_out, sl_stream_t stream);

/* The gate linear alone: router_logits_out (bf16 [T, E]) = bf16(hidden @
 * gate_w^T + logit_bias), the same logits sl_route computes. Replaces
 * `rl, _ = gate(hs)` of the router-split entry (offloader.py:2582; vLLM's
 * bf16 ReplicatedLinear gate). logit_bias may be NULL. Limits: H % 8 == 0,
 * 16-byte aligned hidden / gate_w. */
int sl_gate(const void* hidden, const void* gate_w, const float* logit_bias,
            int T, int H, int E, void* router_logits_out, sl_stream_t stream);

/* select_experts from given bf16 router logits [T, E]
 * (vLLM router/base_router.py:250-298). Same arithmetic as sl_route. */
int sl_select_experts(const void* router_logits, int T, int E, int topk,
                      int scoring, int num_expert_group, int topk_group,
                      int renormalize, float routed_scaling_factor,
                      const float* score_bias, float* topk_weights,
                      int32_t* topk_ids, sl_stream_t stream);

/* -------------------------------------------------------------- slot state
 * Device-resident state of one layer's slot cache: replaces the host-side
 * _ExpertLayerCache (offloader.py:121-169) fields slot_of, expert_in_slot,
 * free_slots, protected / probation (SLRU), protected_cap, local_of,
 * global_of_local, map_is_standing, plus the gap counters
 * (offloader.py:2367-2385) and the fill list of the last gap. */
enum {
  SL_SEG_FREE = 0, SL_SEG_PROBATION = 1, SL_SEG_PROTECTED = 2, SL_SEG_PINNED = 3
};
enum {
  SL_PLAN_FAST_HIT = 1, /* SLUICE_RS_FAST_HIT (offloader.py:2409-2424) */
  SL_PLAN_LFU = 2       /* SLUICE_LFU: popularity counts (_bump_freq 1993-2007,
                           halved every 256 calls) order the protected victims
                           (_coldest_protected 2023-2034, _acquire_slot 2056-2066) */
};

/* Field offsets (bytes) inside the state block, in this order:
 * 0 header (int32 x 16, see SL_HDR_*), 1 counters (uint64 x 16, SL_CNT_*),
 * 2 local_of[global_n], 3 global_of_local[local_n], 4 slot_of[local_n],
 * 5 expert_in_slot[S], 6 seg[S] (uint8), 7 stamp[S] (uint32),
 * 8 free_stack[S], 9 fill_local[S], 10 fill_slot[S], 11 freq[local_n]
 * (uint32 popularity counts, SL_PLAN_LFU); offsets[12] = total. */
enum { SL_STATE_NFIELDS = 12 };
enum {
  SL_HDR_NUM_SLOTS = 0, SL_HDR_GLOBAL_N, SL_HDR_LOCAL_N, SL_HDR_PROTECTED_CAP,
  SL_HDR_FLAGS, SL_HDR_MAP_IS_STANDING, SL_HDR_FREE_TOP, SL_HDR_PROTECTED_COUNT,
  SL_HDR_CLOCK, SL_HDR_STATUS, SL_HDR_FILL_COUNT, SL_HDR_LAST_MISSES,
  SL_HDR_LFU_STEPS, /* calls since the counts were last halved */
  SL_HDR_PREFETCH_FILLS /* experts filled by the last sl_prefetch_slots */
};
enum {
  SL_CNT_GAPS = 0, SL_CNT_FAST_HITS, SL_CNT_MISSES, SL_CNT_HITS,
  SL_CNT_OVERFLOWS, SL_CNT_FILLS /* every expert streamed, gaps and waves */,
  /* steps planned by sl_plan_waves (the classic hook's _StepStats steps,
   * hits, misses and waves, offloader.py:172-183) */
  SL_CNT_SCAN_STEPS, SL_CNT_SCAN_HITS, SL_CNT_SCAN_MISSES, SL_CNT_WAVES,
  SL_CNT_PREFETCHES /* experts filled by sl_prefetch_slots */
};
size_t sl_slot_state_bytes(int num_slots, int global_n, int local_n);
int sl_slot_state_offsets(int num_slots, int global_n, int local_n,
                          size_t* offsets /* [SL_STATE_NFIELDS + 1] */);

/* Initialise a state block from host arrays (replaces the state set-up of
 * _install_cache offloader.py:936-1003 and _apply_pins 1046-1083, which the
 * host computes). expert_in_slot / seg are [S]; free_stack lists the free
 * slots bottom first (the next slot taken is free_stack[n_free-1]). Copies
 * are enqueued on `stream` from the host arrays, which must stay valid until
 * the stream reaches them (the call itself copies them to a staging buffer,
 * so they may be freed on return). */
int sl_slot_state_init(void* state, int num_slots, int global_n, int local_n,
                       int protected_cap, int flags, const int32_t* local_of,
                       const int32_t* expert_in_slot, const uint8_t* seg,
                       const int32_t* free_stack, int n_free,
                       sl_stream_t stream);

/* The gap's slot planning, on the device: replaces the body of
 * _router_split_gap (offloader.py:2362-2467) minus the device-to-host id
 * sync: FAST_HIT check, sorted unique selected ids, SLRU touches of hits,
 * _acquire_slot / _evict_to for misses in ascending id order (the fill
 * list), and the standing expert map (_write_standing_map 2112-2123) written
 * in place into expert_map [global_n]. One CTA. Overflow sets the state's
 * status word to SL_ERR_OVERFLOW (the map is then left as it was). */
int sl_plan_slots(void* state, const int32_t* topk_ids, int num_ids,
                  int32_t* expert_map, sl_stream_t stream);

/* Opt-in cross-layer prefetch, no counterpart in the reference (which
 * measured its gate-ahead prefetch neutral on H100 and removed it,
 * docs/EVALUATION.md:94-97): fill this layer's slots with experts predicted
 * for its next step (e.g. the layer's router run on the previous layer's
 * input) while the previous layer still computes. Predicted owned experts
 * that are not resident, ascending id, at most max_fills, each into the free
 * list's next slot or the least recently used probation slot (never a
 * protected or pinned slot), as a new probation entry; no touches. The fills
 * become the state's fill list: stream them with sl_stream_experts, and order
 * the layer's next sl_plan_slots and its GEMMs after that stream. The
 * standing map, if standing, is rewritten. Changes the slot trajectory
 * relative to the reference's policy, so it is off unless called. */
int sl_prefetch_slots(void* state, const int32_t* topk_ids, int num_ids,
                      int max_fills, int32_t* expert_map, sl_stream_t stream);

/* ---------------------------------------------- steps beyond the envelope
 * A step whose working set can exceed the slots (a prefill, or a mixed
 * prefill + decode batch) runs in expert waves, as the reference's classic
 * hook does for prefill-sized steps under router-split: run_moe
 * (offloader.py:1452-1764) classifies the step, touches the hits and fills
 * what it can (wave 0), and _run_waves (1846-1933) rotates the remaining
 * misses through the probation slots in two ping-pong groups, one wave per
 * group; the step's output is the sum of the waves' outputs.
 *
 * Wave plan buffer (int32 words; field offsets from sl_wave_plan_offsets):
 * 0 header (SL_WAVE_HDR_*), 1 fill_count[max_waves], 2 fill_local
 * [max_waves][S], 3 fill_slot [max_waves][S], 4 map [max_waves][global_n]
 * (wave k's expert map: its experts -> their slots, -1 elsewhere). */
enum { SL_WAVE_NFIELDS = 5 };
enum {
  SL_WAVE_HDR_NUM_WAVES = 0, SL_WAVE_HDR_STATUS, SL_WAVE_HDR_MAX_WAVES,
  SL_WAVE_HDR_GLOBAL_N, SL_WAVE_HDR_NUM_SLOTS,
  SL_WAVE_HDR_LEFTOVER,   /* misses of the last plan past wave 0 */
  SL_WAVE_HDR_ROTATION    /* slots in the last plan's rotation groups */
};
size_t sl_wave_plan_bytes(int num_slots, int global_n, int max_waves);
int sl_wave_plan_offsets(int num_slots, int global_n, int max_waves,
                         size_t* offsets /* [SL_WAVE_NFIELDS + 1], bytes */);
/* Write the buffer's header (dimensions) and empty waves; synchronises
 * `stream`. */
int sl_wave_plan_init(void* waves, int num_slots, int global_n, int max_waves,
                      sl_stream_t stream);

/* Plan one step of num_tokens x topk ids in waves, on the device (one CTA):
 * decode_rows is the step's decode signal (_split_signal 1767-1800): > 0 —
 * rows [0, decode_rows) are single-token decodes (decode-class experts may
 * promote into / evict from the protected segment); 0 — no per-token signal,
 * so the step is decode-class as a whole when its owned working set fits
 * protected_cap + pinned slots (1629-1639); < 0 — every expert scan-class.
 * Wave 0 = hits + the misses that found a slot (decode-class misses first,
 * _acquire_slot 2036-2074); its fills are also the state's fill list, so
 * sl_fused_experts_phase can split wave 0 around its stream. The expert map
 * is left holding the last wave's map and the map stops being standing (the
 * next sl_plan_slots touches its hits and rewrites it), as _write_map
 * 2083-2110 leaves them. More waves than the buffer holds set
 * SL_ERR_OVERFLOW in both status words. */
int sl_plan_waves(void* state, const int32_t* topk_ids, int num_tokens, int topk,
                  int decode_rows, int32_t* expert_map, void* waves,
                  sl_stream_t stream);

/* Stream wave `wave`'s fills of the last sl_plan_waves (nothing for a wave
 * past its count), as sl_stream_experts_strided does for a gap. Order it
 * after the GEMMs that last read the wave's slots: wave k >= 1 reuses the
 * slots of wave k - 2 (ping-pong) or, with a single rotation group, of wave
 * k - 1; waves 1 and 2 also reuse slots wave 0 reads. */
int sl_stream_wave(const void* waves, int wave, int num_params,
                   const void* const* host_src, void* const* slot_dst,
                   const size_t* bytes_per_expert,
                   const size_t* host_stride_bytes, int num_ctas,
                   sl_stream_t stream);

/* Stream the last plan's fills: replaces _stream_in (offloader.py:2709-2723)
 * and its copy-stream events (1979-1991). For every fill (local, slot) and
 * every parameter p, copies bytes_per_expert[p] bytes from
 * host_src[p] + local*bytes_per_expert[p] (mapped pinned host memory) to
 * slot_dst[p] + slot*bytes_per_expert[p], as device-side 16-byte loads.
 * bytes_per_expert[p] % 16 == 0; num_params <= 8; num_ctas <= 0 picks a
 * default. */
int sl_stream_experts(const void* state, int num_params,
                      const void* const* host_src, void* const* slot_dst,
                      const size_t* bytes_per_expert, int num_ctas,
                      sl_stream_t stream);

/* The same for a host store whose experts are not packed per parameter:
 * expert `local` of parameter p starts at host_src[p] + local *
 * host_stride_bytes[p] (a multiple of 16, >= bytes_per_expert[p]). With one
 * packed record per expert ([w13 | w2 | scales], record-sized strides) every
 * fill reads one contiguous host range: the layout a checkpoint loader can
 * fill directly. */
int sl_stream_experts_strided(const void* state, int num_params,
                              const void* const* host_src, void* const* slot_dst,
                              const size_t* bytes_per_expert,
                              const size_t* host_stride_bytes, int num_ctas,
                              sl_stream_t stream);

/* Page-locked host memory mapped into the device address space
 * (cudaHostAlloc Mapped|Portable): the host store of offloaded experts
 * (replaces cpu.pin_memory(), offloader.py:965-967). */
int sl_host_alloc_mapped(size_t bytes, void** host_ptr);
int sl_host_free(void* host_ptr);

/* ----------------------------------------------------------- fused experts
 * Replaces torch.ops.vllm.fused_experts(h, w13, w2, tw, ti, activation=
 * "silu", global_num_experts, expert_map) (offloader.py:2590-2599; vLLM
 * fused_moe.py:1587-1869) plus the shared-expert MLP (offloader.py:2602) and
 * the runner tail (vLLM runner/moe_runner.py:350-366, 663-680):
 *   out[t] = bf16( shared(t) + bf16(scale * bf16(sum_j w[t,j] * z(t,j))) )
 * with z(t,j) = W2[e] (silu(W1g[e] x_t) * W1u[e] x_t) through
 * e = expert_map[topk_ids[t,j]] (a -1 entry contributes nothing) and shared
 * experts given as n_shared experts of the same I (shared_w13 [n_shared,2I,H],
 * shared_w2 [n_shared,H,I]; NULL/0 for none). expert_map NULL means ids are
 * slot indices. weight_dtype must be SL_WEIGHTS_BF16 here (fp8 block-scaled
 * weights go through sl_fused_experts_ex).
 * Tensor-core GEMMs (tcgen05, TMEM accumulators, TMA-fed). Limits:
 * H % 128 == 0, I % 128 == 0, num_slots + n_shared <= 1024.
 * workspace: device memory of at least sl_fused_experts_workspace_bytes(...),
 * 256-byte aligned; its first int32 is the device status word. */
size_t sl_fused_experts_workspace_bytes(int T, int topk, int H, int I,
                                        int num_slots, int n_shared);
int sl_fused_experts(const void* hidden, int T, int H, int I,
                     const void* w13, const void* w2, int num_slots,
                     int weight_dtype, const float* topk_weights,
                     const int32_t* topk_ids, int topk,
                     const int32_t* expert_map, int global_n,
                     const void* shared_w13, const void* shared_w2,
                     int n_shared, float routed_scaling_factor, void* out,
                     void* workspace, size_t workspace_bytes,
                     sl_stream_t stream);

/* Expert weights of one layer for sl_fused_experts_ex. */
enum { SL_WEIGHTS_BF16 = 0, SL_WEIGHTS_FP8_BLOCK128 = 1 };
typedef struct sl_expert_weights {
  const void* w13;                /* [num_slots, 2I, H] bf16 or fp8 e4m3 */
  const void* w2;                 /* [num_slots, H, I] */
  const float* w13_scale;         /* fp8: [num_slots, 2I/128, H/128] */
  const float* w2_scale;          /* fp8: [num_slots, H/128, I/128] */
  int num_slots;
  const void* shared_w13;         /* [n_shared, 2I, H] or NULL */
  const void* shared_w2;          /* [n_shared, H, I] or NULL */
  const float* shared_w13_scale;  /* fp8 */
  const float* shared_w2_scale;   /* fp8 */
  int n_shared;
  int dtype;                      /* SL_WEIGHTS_* */
} sl_expert_weights;

/* The general form of fused_experts (offloader.py:2590-2602 with vLLM's
 * block-fp8 MoE layout, fused_moe.py:1587-1632 w1_scale / w2_scale /
 * block_shape=[128,128]): bf16 or fp8 e4m3 weights with fp32 128x128 block
 * scales (dequantised per tile into bf16 for the tensor cores; activations
 * stay bf16), shared experts on tokens [shared_t0, shared_t0 + shared_nt)
 * (shared_nt < 0: every token), optional phase split around the expert
 * stream (phase -1: whole call; 0 / 1 or the parts SL_PHASE_* as
 * sl_fused_experts_phase, slot_state required), and out_f32 = 1 for the
 * expert-parallel fp32 partial (as
 * sl_fused_experts_partial), 2 for the same partial added to the fp32 `out`
 * (the expert waves of one step, sl_plan_waves). */
int sl_fused_experts_ex(const void* hidden, int T, int H, int I,
                        const sl_expert_weights* weights,
                        const float* topk_weights, const int32_t* topk_ids,
                        int topk, const int32_t* expert_map, int global_n,
                        float routed_scaling_factor, int shared_t0,
                        int shared_nt, const void* slot_state, int phase,
                        int out_f32, void* out, void* workspace,
                        size_t workspace_bytes, sl_stream_t stream);

/* Parts of a phased fused-experts call (phase 0 = GROUP then
 * RESIDENT_GEMMS, phase 1 = STREAMED_GEMMS then COMBINE). */
enum {
  SL_PHASE_GROUP = 2,           /* token grouping only */
  SL_PHASE_RESIDENT_GEMMS = 3,  /* both GEMMs over the resident experts' items */
  SL_PHASE_STREAMED_GEMMS = 4,  /* both GEMMs over the streamed experts' items */
  SL_PHASE_COMBINE = 5          /* the combine only (output written here) */
};

/* sl_fused_experts in two phases, so the gap's expert stream can overlap
 * with the experts that were already resident (the reference serialises the
 * copy stream and the GEMM with events, offloader.py:2443-2464):
 *   phase 0 — token grouping (items of the slots in the state's current fill
 *             list are ordered last) and both GEMMs over the resident
 *             experts' items;
 *   phase 1 — both GEMMs over the streamed experts' items, then the
 *             combine (output written here).
 * Order sl_stream_experts (e.g. on a second stream) before phase 1 and after
 * sl_plan_slots; phase 0 only reads slots the streamer does not write. Both
 * calls take the same workspace. Phases 2..5 (SL_PHASE_*) run one part each,
 * in that order, so the streamed experts' GEMMs can follow the stream on its
 * own stream while the resident ones run: STREAMED_GEMMS after GROUP and
 * after the stream, COMBINE after both GEMM parts. */
int sl_fused_experts_phase(const void* hidden, int T, int H, int I,
                           const void* w13, const void* w2, int num_slots,
                           int weight_dtype, const float* topk_weights,
                           const int32_t* topk_ids, int topk,
                           const int32_t* expert_map, int global_n,
                           const void* shared_w13, const void* shared_w2,
                           int n_shared, float routed_scaling_factor,
                           const void* slot_state, int phase, void* out,
                           void* workspace, size_t workspace_bytes,
                           sl_stream_t stream);

/* Expert-parallel half of fused_experts: this rank's experts only, fp32, no
 * rounding, so partial outputs of all ranks can be summed (reduce-scatter)
 * before the final bf16 rounding:
 *   out_f32[t] = scale * sum_{j: expert_map[ids[t,j]] >= 0} w[t,j] z(t,j)
 *              + (shared_t0 <= t < shared_t0 + shared_nt ? shared(t) : 0)
 * Replaces the per-rank expert computation of vLLM's EP path under the
 * reference (non-owned experts are -1 in the map: offloader.py:974-986,
 * 2432-2435); shared experts run once per token, on the token's home rank.
 * Same workspace as sl_fused_experts. */
int sl_fused_experts_partial(const void* hidden, int T, int H, int I,
                             const void* w13, const void* w2, int num_slots,
                             int weight_dtype, const float* topk_weights,
                             const int32_t* topk_ids, int topk,
                             const int32_t* expert_map, int global_n,
                             const void* shared_w13, const void* shared_w2,
                             int n_shared, int shared_t0, int shared_nt,
                             float routed_scaling_factor, float* out_f32,
                             void* workspace, size_t workspace_bytes,
                             sl_stream_t stream);

/* ------------------------------------------------ expert-parallel exchange
 * Replaces vLLM's EP dispatch / combine around the reference's per-rank
 * experts (offloader.py:690-699, 1192-1201: every rank plans the ids it owns
 * after the dispatch) with one routed kernel each over NVLink peer memory:
 * a token travels only to the ranks that own one of its top-k experts, and
 * only those ranks' partial outputs come back. Experts are sharded in
 * contiguous ranges (rank q owns global ids [q*G/world, (q+1)*G/world),
 * global_n % world == 0). peer_recv[q] / peer_signal[q] are rank q's receive
 * buffer (16-byte aligned) and signal words (16 x u32, zeroed before first
 * use), mapped into every rank (symmetric memory); book is 16 bytes of this
 * rank's device memory, zeroed once; status a device int32. T <= the T the
 * buffers were sized for, T <= 1024. Receive buffers hold two halves used
 * alternately (sized by the _bytes queries). All ranks must make the same
 * sequence of calls; every wait on a peer is bounded (SL_ERR_TIMEOUT in
 * *status).
 * dispatch: this rank's hidden bf16 [T, H] (16-byte aligned), top-k weights
 *   f32 [T, topk] and ids i32 [T, topk]. Outputs world*T rows: rows [0, T)
 *   are this rank's tokens, then the rows each peer sent (peers in rank
 *   order, each peer's tokens in token order); the remaining rows carry id
 *   -1 and weight 0 (no expert) and an unwritten hidden row. x_out bf16
 *   [world*T, H], w_out [world*T, topk], id_out [world*T, topk], src_out
 *   i32 [world*T]: (home rank << 16) | token index of each row, -1 for an
 *   empty row.
 * combine: partial fp32 [world*T, H] (this rank's experts over the rows the
 *   dispatch produced, in its order), the dispatch's src_out, and this rank's
 *   own topk_ids [T, topk]; out = bf16(sum over the ranks each token was
 *   sent to, and this rank, in rank order) for this rank's T tokens, or
 *   bf16(residual + that) when residual (bf16 [T, H]) is not NULL: the
 *   decoder's residual add folded in. */
size_t sl_ep_dispatch_recv_bytes(int world, int T, int H, int topk);
size_t sl_ep_combine_recv_bytes(int world, int T, int H);
int sl_ep_dispatch(const void* hidden, const float* topk_weights, const int32_t* topk_ids,
                   int T, int H, int topk, int global_n, int rank, int world,
                   void* const* peer_recv, void* const* peer_signal, void* book,
                   void* x_out, float* w_out, int32_t* id_out, int32_t* src_out,
                   int32_t* status, sl_stream_t stream);
int sl_ep_combine(const float* partial, const int32_t* src, const int32_t* topk_ids,
                  int T, int H, int topk, int global_n, int rank, int world,
                  void* const* peer_recv, void* const* peer_signal, void* book,
                  const void* residual, void* out, int32_t* status, sl_stream_t stream);

/* ---------------------------------------------------- decoder harness
 * Not part of the reference's MoE operator surface: the attention of the
 * DeepSeek-V2-Lite-shaped decoder that wraps the MoE layers in this build's
 * benchmark (the reference runs inside vLLM, whose attention this stands in
 * for). One decode step of absorbed multi-head latent attention for B
 * sequences: qkv bf16 [B, ld_qkv] rows [q (nh x (nope + rope)) | c_kv (rank)
 * | k_pe (rope)]; c_kv RMSNormed (kv_norm bf16 [rank], eps) and k_pe / q_pe
 * rotated by rope_cos_sin (f32 [max_len, rope/2, 2], adjacent pairs) at
 * position pos[b] (int64 [B]); the position's [c_kv | k_pe] is written to
 * cache bf16 [B, max_len, rank + rope]; scores of [q_nope W_uk | q_pe]
 * (w_uk bf16 [nh, nope, rank]) against positions 0..pos[b], times scale,
 * softmax; out bf16 [B, nh * vdim] = (sum_l p_l c_l) W_uv^T per head (w_uv
 * bf16 [nh, vdim, rank]). */
int sl_mla_decode(const void* qkv, int ld_qkv, const void* kv_norm, float eps,
                  const void* w_uk, const void* w_uv, const float* rope_cos_sin,
                  const int64_t* pos, void* cache, int B, int nh, int nope, int rope,
                  int rank, int vdim, int max_len, float scale, void* out,
                  sl_stream_t stream);

/* Not part of the reference's MoE operator surface: the residual add and
 * RMSNorm between the decoder's sublayers in this build's benchmark harness
 * (vLLM's fused add + RMSNorm, which the reference's model runs). For each of
 * `rows` rows of width H (bf16): h = bf16(h + delta) in place (delta NULL:
 * h unchanged), then out = bf16(h * rsqrt(mean(h^2) + eps) * w) (fp32
 * arithmetic, w bf16 [H]). H a multiple of 8, at most 8192; rows 16-byte
 * aligned. */
int sl_add_rmsnorm(void* h, const void* delta, const void* w, float eps, void* out, int rows,
                   int H, sl_stream_t stream);

/* Not part of the reference's MoE operator surface: the projections of the
 * decoder in this build's benchmark harness for single-sequence decode. y
 * bf16 [T, N] = x bf16 [T, K] times w bf16 [N, K] transposed, fp32 sums; T <= 4,
 * K a multiple of 8 with T * K * 2 bytes <= 200 KB; x and w 16-byte
 * aligned. */
int sl_linear_small(const void* x, int T, int K, const void* w, int N, void* y,
                    sl_stream_t stream);

/* sl_fused_experts without any device allocation. No counterpart in the
 * reference: it serves callers that cannot allocate device scratch memory for
 * a call -- a host program binding this C ABI directly (cgo, JNI, ctypes
 * without torch) has no caching allocator to draw on, and a serving process
 * that has handed nearly all HBM to its own pool sees cudaMalloc fail or
 * stall the device mid-step. Same arguments and result as sl_fused_experts,
 * minus the workspace; the scratch is one file-scope device array of 32 MiB
 * per device, held from library load until process exit.
 *   - Problems whose sl_fused_experts_workspace_bytes(...) exceeds 32 MiB
 *     return SL_ERR_NO_SCRATCH and launch nothing.
 *   - Every call on a device shares the array: calls that can overlap on the
 *     GPU (unordered streams) race and corrupt each other.
 *   - The array keeps the last call's contents; each call clears its status
 *     word and work counts first and rewrites every row it reads.
 *   - The first call on a device looks up the array's device address
 *     (cudaGetSymbolAddress) with that device current: make it before any
 *     stream capture.
 *   - status_out (device int32, may be NULL) receives the device status word
 *     (SL_OK or SL_ERR_TIMEOUT) on the same stream, and only when the call
 *     returns SL_OK. Every argument is checked before anything is enqueued:
 *     any other return leaves the stream, the scratch and status_out
 *     untouched (SL_ERR_CUDA from a failed launch excepted).
 *   - bf16 weights only (weight_dtype SL_WEIGHTS_BF16; others return
 *     SL_ERR_UNSUPPORTED).
 * Calls no cudaMalloc / cudaFree / allocating library routine. */
int sl_fused_experts_noalloc(const void* hidden, int T, int H, int I,
                             const void* w13, const void* w2, int num_slots,
                             int weight_dtype, const float* topk_weights,
                             const int32_t* topk_ids, int topk,
                             const int32_t* expert_map, int global_n,
                             const void* shared_w13, const void* shared_w2,
                             int n_shared, float routed_scaling_factor,
                             void* out, int32_t* status_out,
                             sl_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* SLUICE_B200_H */
