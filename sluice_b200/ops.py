"""The reference's operator surface, backed by the sm_100a library.

* ``Router.select_experts(hidden_states, router_logits, *, input_ids=None)``
  mirrors vLLM's ``BaseRouter.select_experts`` (``router/base_router.py``
  250-298) as called at ``offloader.py:2583-2585``; ``Router.gate`` is the
  bf16 gate linear (``offloader.py:2582``) and ``Router.route`` the gate
  fused with the selection.
* ``sluice_stream_gap(hidden_states, topk_ids, layer_idx)`` mirrors the
  custom op ``vllm::sluice_stream_gap`` (``offloader.py:2311-2331``): it runs
  the slot planner and the expert streamer of the registered layer and
  returns ``hidden_states.clone()`` (``mutates_args=[]``; the fake returns
  ``empty_like``). Registered as ``torch.ops.sluice.sluice_stream_gap``.
* ``fused_experts(hidden_states, w1, w2, topk_weights, topk_ids,
  activation="silu", global_num_experts=-1, expert_map=None, ...)`` mirrors
  ``torch.ops.vllm.fused_experts`` as called at ``offloader.py:2590-2599``,
  with the shared experts and routed scaling fused into its combine.
  Registered as ``torch.ops.sluice.fused_experts``.
* ``register_reference_names()`` registers the same ops under the names the
  reference's router-split entry calls, ``torch.ops.vllm.sluice_stream_gap``
  and ``torch.ops.vllm.fused_experts``, so that entry runs unedited.

All calls enqueue on the current CUDA stream and never synchronise, so they
can be captured in a CUDA graph.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import check, lib, ptr
from .configs import RoutingConfig


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _need_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("sluice_b200 ops take CUDA tensors")


class Router:
    """Gate linear + expert selection for one MoE layer."""

    def __init__(self, routing: RoutingConfig, gate_weight: torch.Tensor | None = None,
                 logit_bias: torch.Tensor | None = None,
                 score_bias: torch.Tensor | None = None):
        self.routing = routing
        self.gate_weight = gate_weight
        self.logit_bias = logit_bias
        self.score_bias = score_bias
        if routing.has_score_bias and score_bias is None:
            raise ValueError("this routing mode needs e_score_correction_bias")

    @property
    def num_experts(self) -> int:
        return self.gate_weight.shape[0]

    def _groups(self):
        r = self.routing
        if r.use_grouped_topk:
            return r.num_expert_group, r.topk_group
        return 1, 1

    def select_experts(self, hidden_states: torch.Tensor, router_logits: torch.Tensor, *,
                       input_ids: torch.Tensor | None = None):
        """(topk_weights fp32 [T,k], topk_ids int32 [T,k]) from bf16 logits."""
        _need_cuda(router_logits)
        r = self.routing
        T, E = router_logits.shape
        lg = router_logits.contiguous()
        if lg.dtype != torch.bfloat16:
            lg = lg.to(torch.bfloat16)
        w = torch.empty(T, r.topk, dtype=torch.float32, device=lg.device)
        ids = torch.empty(T, r.topk, dtype=torch.int32, device=lg.device)
        ng, tg = self._groups()
        check(lib().sl_select_experts(ptr(lg), T, E, r.topk, r.scoring, ng, tg,
                                      int(r.renormalize), 1.0, ptr(self.score_bias),
                                      ptr(w), ptr(ids), _stream()), "sl_select_experts")
        return w, ids

    def gate(self, hidden_states: torch.Tensor):
        """The gate linear: ``(router_logits bf16 [T, E], None)``, the
        ``(output, bias)`` pair of vLLM's gate module that the router-split
        entry unpacks as ``rl, _ = gate(hs)`` (offloader.py:2582)."""
        _need_cuda(hidden_states, self.gate_weight)
        hs = hidden_states.contiguous()
        T, H = hs.shape
        E = self.gate_weight.shape[0]
        logits = torch.empty(T, E, dtype=torch.bfloat16, device=hs.device)
        check(lib().sl_gate(ptr(hs), ptr(self.gate_weight), ptr(self.logit_bias), T, H, E,
                            ptr(logits), _stream()), "sl_gate")
        return logits, None

    def route(self, hidden_states: torch.Tensor, logits_out: torch.Tensor | None = None):
        """Fused gate GEMV + selection: (topk_weights, topk_ids, router_logits)."""
        _need_cuda(hidden_states, self.gate_weight)
        r = self.routing
        hs = hidden_states.contiguous()
        T, H = hs.shape
        E = self.gate_weight.shape[0]
        dev = hs.device
        logits = logits_out if logits_out is not None else torch.empty(
            T, E, dtype=torch.bfloat16, device=dev)
        w = torch.empty(T, r.topk, dtype=torch.float32, device=dev)
        ids = torch.empty(T, r.topk, dtype=torch.int32, device=dev)
        ng, tg = self._groups()
        check(lib().sl_route(ptr(hs), ptr(self.gate_weight), ptr(self.logit_bias), T, H, E,
                             r.topk, r.scoring, ng, tg, int(r.renormalize), 1.0,
                             ptr(self.score_bias), ptr(w), ptr(ids), ptr(logits),
                             _stream()), "sl_route")
        return w, ids, logits


def _expert_weights(w1, w2, w1_scale, w2_scale, shared_w13, shared_w2,
                    shared_w13_scale, shared_w2_scale) -> _lib.ExpertWeights:
    fp8 = w1.dtype == torch.float8_e4m3fn
    if fp8:
        if w1_scale is None or w2_scale is None:
            raise ValueError("fp8 expert weights need w1_scale / w2_scale (128x128 blocks)")
        for t in (w1_scale, w2_scale, shared_w13_scale, shared_w2_scale):
            if t is not None and (t.dtype != torch.float32 or not t.is_contiguous()):
                raise ValueError("block scales must be contiguous fp32")
    elif w1.dtype != torch.bfloat16:
        raise ValueError(f"unsupported expert weight dtype {w1.dtype}")
    if w2.dtype != w1.dtype or (shared_w13 is not None and shared_w13.dtype != w1.dtype):
        raise ValueError("all expert weights must share one dtype")
    n_sh = 0 if shared_w13 is None else shared_w13.shape[0]
    return _lib.ExpertWeights(ptr(w1), ptr(w2), ptr(w1_scale), ptr(w2_scale), w1.shape[0],
                              ptr(shared_w13), ptr(shared_w2), ptr(shared_w13_scale),
                              ptr(shared_w2_scale), n_sh,
                              _lib.WEIGHTS_FP8_BLOCK128 if fp8 else _lib.WEIGHTS_BF16)


def fused_experts_workspace(T: int, topk: int, H: int, I: int, slots: int, n_shared: int,
                            device) -> torch.Tensor:
    n = lib().sl_fused_experts_workspace_bytes(T, topk, H, I, slots, n_shared)
    return torch.empty(max(n, 256), dtype=torch.uint8, device=device)


def _fused_ex(hs, w1, w2, topk_weights, topk_ids, expert_map, global_n, *, w1_scale=None,
              w2_scale=None, shared_w13=None, shared_w2=None, shared_w13_scale=None,
              shared_w2_scale=None, routed_scaling_factor=1.0, shared_t0=0, shared_nt=-1,
              slot_state=None, phase=-1, out_f32=0, out=None, workspace=None):
    # out_f32: 0 bf16 output; 1 fp32 partial written to `out`; 2 fp32 partial
    # added to `out` (sl_fused_experts_ex)
    _need_cuda(hs, w1, w2, topk_weights, topk_ids, expert_map)
    hs = hs.contiguous()
    if hs.dtype != torch.bfloat16:
        raise ValueError("bf16 activations expected")
    T, H = hs.shape
    S, two_i, H1 = w1.shape
    I = two_i // 2
    if H1 != H or tuple(w2.shape) != (S, H, I):
        raise ValueError(f"weight shapes {tuple(w1.shape)} / {tuple(w2.shape)} do not match H={H}")
    if expert_map is not None and expert_map.dtype != torch.int32:
        raise ValueError("expert_map must be int32")
    w = _expert_weights(w1, w2, w1_scale, w2_scale, shared_w13, shared_w2, shared_w13_scale,
                        shared_w2_scale)
    k = topk_ids.shape[1]
    if workspace is None:
        workspace = fused_experts_workspace(T, k, H, I, S, w.n_shared, hs.device)
    if out is None:
        out = torch.empty(T, H, dtype=torch.float32 if out_f32 else torch.bfloat16,
                          device=hs.device)
    tw = topk_weights if topk_weights.dtype == torch.float32 and topk_weights.is_contiguous() \
        else topk_weights.contiguous().float()
    ti = topk_ids if topk_ids.dtype == torch.int32 and topk_ids.is_contiguous() \
        else topk_ids.contiguous().to(torch.int32)
    check(lib().sl_fused_experts_ex(ptr(hs), T, H, I, ctypes.byref(w), ptr(tw), ptr(ti), k,
                                    ptr(expert_map), global_n, float(routed_scaling_factor),
                                    int(shared_t0), int(shared_nt), ptr(slot_state), int(phase),
                                    int(out_f32), ptr(out), ptr(workspace), workspace.numel(),
                                    _stream()), "sl_fused_experts_ex")
    fused_experts.last_workspace = workspace
    return out


def fused_experts(hidden_states: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor,
                  topk_weights: torch.Tensor, topk_ids: torch.Tensor,
                  activation: str = "silu", global_num_experts: int = -1,
                  expert_map: torch.Tensor | None = None,
                  w1_scale: torch.Tensor | None = None, w2_scale: torch.Tensor | None = None,
                  block_shape: list | None = None,
                  shared_w13: torch.Tensor | None = None,
                  shared_w2: torch.Tensor | None = None,
                  shared_w13_scale: torch.Tensor | None = None,
                  shared_w2_scale: torch.Tensor | None = None,
                  routed_scaling_factor: float = 1.0,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """Routed (+ shared) expert output [T, H] bf16.

    ``w1`` is [slots, 2I, H] (gate rows then up rows), ``w2`` [slots, H, I],
    bf16 or fp8 e4m3 with fp32 ``w1_scale`` [slots, 2I/128, H/128] /
    ``w2_scale`` [slots, H/128, I/128] (``block_shape`` [128, 128]);
    ``expert_map`` int32 [global_num_experts] maps a global id to its slot
    (-1: contributes nothing). Without a map, ids index ``w1`` directly.
    """
    if activation != "silu":
        raise ValueError("only activation='silu' (SwiGLU) is on this path")
    if block_shape is not None and list(block_shape) != [128, 128]:
        raise ValueError("only 128x128 weight blocks are supported")
    G = expert_map.numel() if expert_map is not None else (
        global_num_experts if global_num_experts > 0 else w1.shape[0])
    return _fused_ex(hidden_states, w1, w2, topk_weights, topk_ids, expert_map, G,
                     w1_scale=w1_scale, w2_scale=w2_scale, shared_w13=shared_w13,
                     shared_w2=shared_w2, shared_w13_scale=shared_w13_scale,
                     shared_w2_scale=shared_w2_scale,
                     routed_scaling_factor=routed_scaling_factor, out=out)


fused_experts.last_workspace = None


def fused_experts_phase(hidden_states, w1, w2, topk_weights, topk_ids, expert_map, slot_state,
                        phase: int, workspace: torch.Tensor, out: torch.Tensor,
                        w1_scale=None, w2_scale=None, shared_w13=None, shared_w2=None,
                        shared_w13_scale=None, shared_w2_scale=None,
                        routed_scaling_factor: float = 1.0) -> torch.Tensor:
    """One phase of ``fused_experts`` split around the expert stream: phase 0
    computes the already-resident experts, phase 1 the streamed ones and the
    combine into ``out``. Both phases take the same ``workspace``. Phases
    2..5 (``_lib.PHASE_*``: grouping, resident experts' GEMMs, streamed
    experts' GEMMs, combine) run one part each, in that order, so the
    streamed experts' GEMMs can be ordered after the stream on its own
    stream."""
    return _fused_ex(hidden_states, w1, w2, topk_weights, topk_ids, expert_map,
                     expert_map.numel(), w1_scale=w1_scale, w2_scale=w2_scale,
                     shared_w13=shared_w13, shared_w2=shared_w2,
                     shared_w13_scale=shared_w13_scale, shared_w2_scale=shared_w2_scale,
                     routed_scaling_factor=routed_scaling_factor, slot_state=slot_state,
                     phase=phase, out=out, workspace=workspace)


def fused_experts_partial(hidden_states, w1, w2, topk_weights, topk_ids, expert_map,
                          shared_w13=None, shared_w2=None, shared_t0: int = 0,
                          shared_nt: int = 0, routed_scaling_factor: float = 1.0,
                          out=None, w1_scale=None, w2_scale=None, shared_w13_scale=None,
                          shared_w2_scale=None, slot_state=None, phase: int = -1,
                          workspace=None) -> torch.Tensor:
    """Expert-parallel partial output [T, H] fp32: this rank's experts (the
    ones ``expert_map`` maps) scaled by ``routed_scaling_factor``, plus the
    shared experts on rows [shared_t0, shared_t0 + shared_nt). ``phase`` 0 / 1
    (or its four parts 2..5) split the call around the gap's expert stream as
    ``fused_experts_phase`` does (every part: the same ``slot_state``,
    ``workspace`` and ``out``)."""
    return _fused_ex(hidden_states, w1, w2, topk_weights, topk_ids, expert_map,
                     expert_map.numel(), w1_scale=w1_scale, w2_scale=w2_scale,
                     shared_w13=shared_w13, shared_w2=shared_w2,
                     shared_w13_scale=shared_w13_scale, shared_w2_scale=shared_w2_scale,
                     routed_scaling_factor=routed_scaling_factor, shared_t0=shared_t0,
                     shared_nt=shared_nt, out_f32=1, out=out, slot_state=slot_state,
                     phase=phase, workspace=workspace)


fused_experts_partial.last_workspace = None


def fused_experts_accumulate(hidden_states, w1, w2, topk_weights, topk_ids, expert_map,
                             out: torch.Tensor, workspace: torch.Tensor,
                             routed_scaling_factor: float = 1.0, w1_scale=None,
                             w2_scale=None) -> torch.Tensor:
    """``out`` [T, H] fp32 += the routed experts ``expert_map`` maps, scaled
    by ``routed_scaling_factor`` (no shared experts): one expert wave of a
    step beyond the envelope, whose waves sum to the step's output
    (``_run_waves``, offloader.py:1920-1933)."""
    if out.dtype != torch.float32:
        raise ValueError("the wave accumulator is fp32")
    return _fused_ex(hidden_states, w1, w2, topk_weights, topk_ids, expert_map,
                     expert_map.numel(), w1_scale=w1_scale, w2_scale=w2_scale,
                     routed_scaling_factor=routed_scaling_factor, out_f32=2, out=out,
                     workspace=workspace)


def workspace_status(ws: torch.Tensor) -> int:
    """Device status word of a fused_experts workspace (synchronises)."""
    return int(ws[:4].view(torch.int32)[0].item())


# --------------------------------------------------------------- torch ops
# The gap registry: layer_idx -> SlotCache (the reference's _rs_caches).
_GAP_CACHES: list = []


def register_gap_layer(cache) -> int:
    _GAP_CACHES.append(cache)
    return len(_GAP_CACHES) - 1


def sluice_stream_gap(hidden_states: torch.Tensor, topk_ids: torch.Tensor,
                      layer_idx: int) -> torch.Tensor:
    _GAP_CACHES[int(layer_idx)].gap(topk_ids)
    return hidden_states.clone()


_lib_def = torch.library.Library("sluice", "DEF")
_lib_def.define("sluice_stream_gap(Tensor hidden_states, Tensor topk_ids, int layer_idx) -> Tensor")
_lib_def.define(
    "fused_experts(Tensor hidden_states, Tensor w1, Tensor w2, Tensor topk_weights, "
    "Tensor topk_ids, str activation='silu', int global_num_experts=-1, "
    "Tensor? expert_map=None, Tensor? w1_scale=None, Tensor? w2_scale=None, "
    "Tensor? shared_w13=None, Tensor? shared_w2=None, float routed_scaling_factor=1.0) "
    "-> Tensor")
_lib_def.impl("sluice_stream_gap", sluice_stream_gap, "CUDA")
_lib_def.impl(
    "fused_experts",
    lambda hs, w1, w2, tw, ti, activation="silu", global_num_experts=-1, expert_map=None,
    w1_scale=None, w2_scale=None, shared_w13=None, shared_w2=None,
    routed_scaling_factor=1.0: fused_experts(
        hs, w1, w2, tw, ti, activation=activation, global_num_experts=global_num_experts,
        expert_map=expert_map, w1_scale=w1_scale, w2_scale=w2_scale, shared_w13=shared_w13,
        shared_w2=shared_w2, routed_scaling_factor=routed_scaling_factor),
    "CUDA")


@torch.library.register_fake("sluice::sluice_stream_gap")
def _gap_fake(hidden_states, topk_ids, layer_idx):
    return torch.empty_like(hidden_states)


@torch.library.register_fake("sluice::fused_experts")
def _fe_fake(hidden_states, w1, w2, topk_weights, topk_ids, activation="silu",
             global_num_experts=-1, expert_map=None, w1_scale=None, w2_scale=None,
             shared_w13=None, shared_w2=None, routed_scaling_factor=1.0):
    return torch.empty_like(hidden_states)


# ------------------------------------------- the reference's own op names
# The reference's router-split entry (offloader.py:2578-2603) calls
# torch.ops.vllm.sluice_stream_gap, which the reference registers itself
# (_register_stream_gap_op, offloader.py:2296-2331), and
# torch.ops.vllm.fused_experts, vLLM's fused-MoE op. Registering this build's
# ops under those names lets that entry run unedited on the sm_100a path.
_VLLM_LIB = None


def _vllm_op_exists(name: str) -> bool:
    try:
        getattr(torch.ops.vllm, name)
        return True
    except (AttributeError, RuntimeError):
        return False


def register_reference_names() -> list[str]:
    """Register ``vllm::sluice_stream_gap`` (the reference's schema:
    ``(Tensor hidden_states, Tensor topk_ids, int layer_idx) -> Tensor``,
    ``mutates_args=[]``, a fake returning ``empty_like``) and, where no
    ``vllm::fused_experts`` is loaded, ``vllm::fused_experts(hidden_states,
    w1, w2, topk_weights, topk_ids, activation='silu', global_num_experts=-1,
    expert_map=None, w1_scale=None, w2_scale=None)`` — the routed experts
    only, as the reference's entry expects (its caller adds the shared
    experts). Names already defined (the reference plugin's own gap op, or a
    vLLM build that has ``fused_experts``) are left alone. Returns the names
    this call registered; calling it again registers nothing."""
    global _VLLM_LIB
    done = []
    want = [n for n in ("sluice_stream_gap", "fused_experts") if not _vllm_op_exists(n)]
    if not want:
        return done
    if _VLLM_LIB is None:
        _VLLM_LIB = torch.library.Library("vllm", "FRAGMENT")
    lib_ = _VLLM_LIB
    if "sluice_stream_gap" in want:
        lib_.define("sluice_stream_gap(Tensor hidden_states, Tensor topk_ids, int layer_idx) "
                    "-> Tensor")
        lib_.impl("sluice_stream_gap", sluice_stream_gap, "CUDA")
        lib_._register_fake("sluice_stream_gap", _gap_fake)
        done.append("vllm::sluice_stream_gap")
    if "fused_experts" in want:
        lib_.define(
            "fused_experts(Tensor hidden_states, Tensor w1, Tensor w2, Tensor topk_weights, "
            "Tensor topk_ids, str activation='silu', int global_num_experts=-1, "
            "Tensor? expert_map=None, Tensor? w1_scale=None, Tensor? w2_scale=None) -> Tensor")
        lib_.impl(
            "fused_experts",
            lambda hs, w1, w2, tw, ti, activation="silu", global_num_experts=-1,
            expert_map=None, w1_scale=None, w2_scale=None: fused_experts(
                hs, w1, w2, tw, ti, activation=activation,
                global_num_experts=global_num_experts, expert_map=expert_map,
                w1_scale=w1_scale, w2_scale=w2_scale),
            "CUDA")
        lib_._register_fake(
            "fused_experts",
            lambda hs, w1, w2, tw, ti, activation="silu", global_num_experts=-1,
            expert_map=None, w1_scale=None, w2_scale=None: torch.empty_like(hs))
        done.append("vllm::fused_experts")
    return done
