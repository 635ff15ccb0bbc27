"""Generate the golden fixtures in this folder from the reference itself.

Run in a container that has the reference checkout and vLLM installed::

    SLUICE_REFERENCE=<path to kfirtoledo/sluice> python tests/golden/make_golden.py

It writes:

* ``slot_traces.json`` — per scenario, the flattened ``topk_ids`` of every
  step and the state after each call of the reference's own
  ``ExpertStreamOffloader._router_split_gap`` (``src/sluice/offloader.py``
  2362-2467) on a CPU ``_ExpertLayerCache`` built by the reference's own
  ``_install_cache`` (895-1044) and ``_apply_pins`` (1046-1083): the expert
  map, slot owners, slot contents, protected / probation order and counters.
* ``routing.npz`` — router logits and vLLM 0.22's CPU ``grouped_topk``
  (``fused_moe/cpu_fused_moe.py`` 59-115) outputs for the V2-Lite, Qwen3 and
  DeepSeek-V3 routing modes.
* ``moe.npz`` — a small ``fused_experts`` case through an expert map,
  evaluated by vLLM's ``cpu_fused_moe_torch`` (``cpu_fused_moe.py`` 428-482).
* ``fp8_quant.npz`` — bf16 activations through vLLM's torch-native
  per-token-group fp8 quantisation (``QuantFP8._quantize_group_native``).
* ``nonmla_rows.json`` — the reference's opt-in non-MLA decode-row
  classifier ``ExpertStreamOffloader._non_mla_decode_rows`` (1802-1844) on
  synthetic attention metadata (vLLM's forward context replaced for the call).
* ``wave_traces.json`` — steps beyond the envelope through the reference's
  classic hook ``ExpertStreamOffloader.run_moe`` (1452-1764) and
  ``_run_waves`` (1846-1933), some scenarios interleaved with router-split gap
  calls: per step the waves (each wave's expert map entries and the fills
  streamed before it, read off ``_write_map`` / ``_stream_in``) and the
  state after the step. CUDA events and the current stream are replaced by
  no-op stand-ins (there is no copy stream on a CPU cache, so every copy is
  made in place), and ``_split_signal`` returns the step's decode signal.

Nothing at test time reads the reference; the tests read these files.
"""

from __future__ import annotations

import json
import os
import sys

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get("SLUICE_REFERENCE", "")


def _ref_offloader(slots: int, fast_hit: bool, frac: float, no_static_full=False,
                   lfu=False):
    os.environ["SLUICE_RS_FAST_HIT"] = "1" if fast_hit else "0"
    os.environ["SLUICE_LFU"] = "1" if lfu else "0"
    os.environ["SLUICE_PROTECT_FRAC"] = str(frac)
    os.environ["SLUICE_NO_STATIC_FULL"] = "1" if no_static_full else "0"
    os.environ.pop("SLUICE_ROUTER_SPLIT", None)
    from sluice.offloader import ExpertStreamOffloader

    ExpertStreamOffloader._infer_device = staticmethod(lambda m: torch.device("cpu"))
    off = ExpertStreamOffloader(slots)
    off.pin_memory = False
    return off


class _FakeMoE(nn.Module):
    """Just enough of a FusedMoE layer for the reference's _install_cache."""

    def __init__(self, local_n: int, global_n: int, expert_map):
        super().__init__()
        self.local_num_experts = local_n
        self.global_num_experts = global_n
        self.quant_method = None
        # each local expert's payload is its own local index
        self.w = nn.Parameter(torch.arange(local_n, dtype=torch.float32).view(-1, 1),
                              requires_grad=False)
        self.expert_map = expert_map


def _zipf_ids(gen, steps, T, k, E, s=1.1, locality=0.6):
    """Top-k ids per token without replacement, Zipf popularity over a seeded
    permutation, 60% of tokens repeating their previous-step selection."""
    perm = torch.randperm(E, generator=gen)
    p = 1.0 / torch.arange(1, E + 1, dtype=torch.float64) ** s
    p = p / p.sum()
    prev = None
    out = []
    for _ in range(steps):
        rows = []
        for t in range(T):
            if prev is not None and torch.rand(1, generator=gen).item() < locality:
                rows.append(prev[t])
                continue
            pick = torch.multinomial(p, k, replacement=False, generator=gen)
            rows.append(perm[pick].tolist())
        prev = rows
        out.append([g for r in rows for g in r])
    return out


def _run_scenario(name, *, slots, global_n, local_n, owned_lo=0, steps_ids,
                  fast_hit=True, frac=0.5, pins=None, no_static_full=False, lfu=False):
    off = _ref_offloader(slots, fast_hit, frac, no_static_full, lfu)
    if pins is not None:
        off._pin_layers = {0: list(pins)}
    if local_n == global_n:
        emap = None
        local_of = list(range(global_n))
    else:
        lo = [-1] * global_n
        for i in range(local_n):
            lo[owned_lo + i] = i
        emap = torch.tensor(lo, dtype=torch.int32)
        local_of = lo
    mod = _FakeMoE(local_n, global_n, emap)
    off._install_cache(mod)
    cache = off._caches[id(mod)]
    assert not cache.static_full, name
    off._rs_caches.append(cache)
    trace = []
    overflow_step = -1
    for i, ids in enumerate(steps_ids):
        if lfu:
            # the popularity counts the reference's hook keeps for every real
            # step (_bump_freq over the step's selected owned experts), then
            # the gap's policy reads them
            pairs = [(g, local_of[g], True) for g in sorted(set(ids))
                     if 0 <= g < global_n and local_of[g] >= 0]
            off._bump_freq(cache, pairs)
        try:
            off._router_split_gap(0, torch.tensor(ids, dtype=torch.int32))
        except RuntimeError:
            overflow_step = i
        w = cache.gpu_cache["w"][:, 0]
        trace.append({
            "expert_map": cache.expert_map_buf.tolist(),
            "expert_in_slot": [-1 if v is None else int(v) for v in cache.expert_in_slot],
            "slot_payload": [int(w[s].item()) if cache.expert_in_slot[s] is not None
                             else -1 for s in range(cache.num_slots)],
            "protected": list(cache.protected),
            "probation": list(cache.probation),
            "map_is_standing": bool(cache.map_is_standing),
            "gaps": off._rs_gaps, "misses": off._rs_misses,
            "fast_hits": off._rs_fast_hits,
            "freq": [int(cache.freq.get(loc, 0)) for loc in range(local_n)],
        })
        if overflow_step >= 0:
            break
    return {
        "name": name, "num_slots": cache.num_slots, "global_n": global_n,
        "local_n": local_n, "local_of": local_of, "fast_hit": fast_hit, "lfu": lfu,
        "protect_frac": frac, "protected_cap": cache.protected_cap,
        "pins": list(pins) if pins is not None else None,
        "pinned_slots": sorted(cache.pinned_slots),
        "prefill_resident": bool(no_static_full and slots >= local_n),
        "steps": steps_ids[: len(trace)], "trace": trace,
        "overflow_step": overflow_step,
    }


def make_slot_traces():
    g = torch.Generator().manual_seed(1234)
    zipf = _zipf_ids(g, 64, 8, 6, 64)
    uni = [torch.randint(0, 64, (48,), generator=g).tolist() for _ in range(40)]
    qwen = _zipf_ids(g, 48, 12, 8, 128)
    v3 = _zipf_ids(g, 40, 8, 8, 256)
    noisy = []
    for ids in _zipf_ids(g, 30, 8, 6, 64):
        ids = list(ids)
        ids[3] = -1
        ids[7] = 64 + (len(noisy) % 5)
        noisy.append(ids)
    big = [torch.randperm(64, generator=g)[:48].tolist() for _ in range(12)]
    lfu_long = _zipf_ids(torch.Generator().manual_seed(4321), 300, 8, 6, 64, locality=0.3)
    exact = [torch.randperm(64, generator=g)[:48].tolist() for _ in range(12)]
    sc = [
        _run_scenario("v2lite_zipf_fasthit", slots=48, global_n=64, local_n=64,
                      steps_ids=zipf),
        _run_scenario("v2lite_zipf_nofasthit", slots=48, global_n=64, local_n=64,
                      steps_ids=zipf, fast_hit=False),
        _run_scenario("v2lite_uniform", slots=48, global_n=64, local_n=64,
                      steps_ids=uni),
        _run_scenario("v2lite_frac0", slots=48, global_n=64, local_n=64,
                      steps_ids=zipf, frac=0.0),
        _run_scenario("v2lite_frac09", slots=48, global_n=64, local_n=64,
                      steps_ids=uni, frac=0.9),
        _run_scenario("v2lite_pins", slots=48, global_n=64, local_n=64,
                      steps_ids=uni, pins=[5, 9, 9, 70, 2, 11]),
        _run_scenario("v2lite_invalid_ids", slots=40, global_n=64, local_n=64,
                      steps_ids=noisy),
        _run_scenario("ep_rank1_of2", slots=24, global_n=64, local_n=32,
                      owned_lo=32, steps_ids=uni),
        _run_scenario("qwen3_s96", slots=96, global_n=128, local_n=128,
                      steps_ids=qwen),
        _run_scenario("v3_ep4_rank2", slots=48, global_n=256, local_n=64,
                      owned_lo=128, steps_ids=v3),
        _run_scenario("overflow_s40", slots=40, global_n=64, local_n=64,
                      steps_ids=zipf[:10] + big[:2]),
        _run_scenario("uniques_equal_slots", slots=48, global_n=64, local_n=64,
                      steps_ids=exact),
        _run_scenario("prefill_resident", slots=64, global_n=64, local_n=64,
                      steps_ids=uni[:8], no_static_full=True),
        # LFU hybrid: frequency-ordered protected victims; 300 steps cross one
        # halving of the counts (every 256 steps)
        _run_scenario("v2lite_lfu_aging", slots=48, global_n=64, local_n=64,
                      steps_ids=lfu_long, lfu=True),
        _run_scenario("v2lite_lfu_uniform_frac09", slots=48, global_n=64, local_n=64,
                      steps_ids=uni, frac=0.9, lfu=True),
        _run_scenario("v2lite_lfu_pins_nofasthit", slots=40, global_n=64, local_n=64,
                      steps_ids=zipf, pins=[3, 17, 40], fast_hit=False, lfu=True),
        _run_scenario("v3_ep4_rank2_lfu", slots=48, global_n=256, local_n=64,
                      owned_lo=128, steps_ids=v3, lfu=True),
    ]
    with open(os.path.join(HERE, "slot_traces.json"), "w") as f:
        json.dump({"generator": "tests/golden/make_golden.py",
                   "scenarios": sc}, f, separators=(",", ":"))
    for s in sc:
        print(f"{s['name']}: steps={len(s['trace'])} misses={s['trace'][-1]['misses']} "
              f"fast_hits={s['trace'][-1]['fast_hits']} overflow={s['overflow_step']}")


def make_routing():
    from vllm.model_executor.layers.fused_moe import cpu_fused_moe as cfm

    g = torch.Generator().manual_seed(99)
    out = {}
    cases = {
        # name: (T, H, E, topk, renorm, groups, topk_group, scoring, scale, bias)
        "v2lite": (32, 2048, 64, 6, False, 1, 1, "softmax", 1.0, False),
        "qwen3": (32, 2048, 128, 8, True, 1, 1, "softmax", 1.0, False),
        "v3": (32, 7168, 256, 8, True, 8, 4, "sigmoid", 2.5, True),
    }
    for name, (T, H, E, k, renorm, G, TG, sf, scale, has_bias) in cases.items():
        x = torch.randn(T, H, generator=g).to(torch.bfloat16)
        w = (torch.randn(E, H, generator=g) * 0.02).to(torch.bfloat16)
        lb = 1.5 * torch.log(1.0 / (torch.randperm(E, generator=g) + 1).double()).float()
        logits = (x.float() @ w.float().t() + lb).to(torch.bfloat16)
        sb = (torch.rand(E, generator=g) * 0.1).float() if has_bias else None
        tw, ti = cfm.grouped_topk(x, logits, k, renorm, G, TG, sf, scale, sb)
        out[f"{name}_logits"] = logits.view(torch.int16).numpy()
        out[f"{name}_ids"] = ti.numpy()
        out[f"{name}_weights"] = tw.numpy()
        if sb is not None:
            out[f"{name}_score_bias"] = sb.numpy()
        out[f"{name}_meta"] = np.array([T, H, E, k, int(renorm), G, TG,
                                        1 if sf == "sigmoid" else 0], dtype=np.int64)
        out[f"{name}_scale"] = np.array([scale], dtype=np.float32)
    np.savez_compressed(os.path.join(HERE, "routing.npz"), **out)
    print("routing:", sorted(k for k in out if k.endswith("_ids")))


def make_fp8_quant():
    """``fp8_quant.npz``: activations through vLLM's torch-native per-token
    group quantisation (``QuantFP8._quantize_group_native``,
    ``layers/quantization/input_quant_fp8.py``; group 128, dynamic scales),
    the CPU-runnable twin of the CUDA op its fp8 MoE path calls."""
    import types

    from vllm.model_executor.layers.quantization.input_quant_fp8 import QuantFP8

    self_ = types.SimpleNamespace(group_size=128, use_ue8m0=False, column_major_scales=False)
    g = torch.Generator().manual_seed(2468)
    x = (torch.randn(96, 2048, generator=g) * torch.rand(96, 1, generator=g) * 4
         ).to(torch.bfloat16)
    xq, s = QuantFP8._quantize_group_native(self_, x)
    np.savez_compressed(os.path.join(HERE, "fp8_quant.npz"),
                        x=x.float().numpy(), q=xq.view(torch.uint8).numpy(),
                        scale=s.float().numpy())


def make_moe():
    from vllm.model_executor.layers.activation import SiluAndMul
    from vllm.model_executor.layers.fused_moe import cpu_fused_moe as cfm
    from vllm.model_executor.layers.fused_moe.activation import MoEActivation

    cfm._CPU_MOE_ACT_FN[MoEActivation.SILU] = SiluAndMul.forward_native
    g = torch.Generator().manual_seed(7)
    T, H, I, S, E, k = 6, 256, 128, 4, 8, 3
    hs = torch.randn(T, H, generator=g).to(torch.bfloat16)
    w13 = (torch.randn(S, 2 * I, H, generator=g) * 0.05).to(torch.bfloat16)
    w2 = (torch.randn(S, H, I, generator=g) * 0.05).to(torch.bfloat16)
    emap = torch.tensor([2, -1, 0, -1, 3, 1, -1, -1], dtype=torch.int32)
    ti = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).to(torch.int32)
    tw = torch.rand(T, k, generator=g).float()
    # vLLM's CPU path has no expert map: route unmapped pairs to a zero expert
    # (one zero expert per choice j, so no token sees the same expert twice)
    zero_slot = S + torch.arange(k, dtype=torch.int32).expand(T, k)
    slots = torch.where(emap[ti.long()] >= 0, emap[ti.long()], zero_slot)
    w13z = torch.cat([w13, torch.zeros(k, 2 * I, H, dtype=w13.dtype)])
    w2z = torch.cat([w2, torch.zeros(k, H, I, dtype=w2.dtype)])

    class _L:
        pass

    layer = _L()
    layer.gate_up_linear = [(lambda x, i=i: F.linear(x, w13z[i])) for i in range(S + k)]
    layer.down_linear = [(lambda x, i=i: F.linear(x, w2z[i])) for i in range(S + k)]
    cfm._CPU_MOE_LAYER_CACHE[12345] = lambda: layer
    out = torch.empty(T, H, dtype=torch.bfloat16)
    cfm.cpu_fused_moe_torch(12345, out, hs, tw, slots.to(torch.int32), "silu",
                            global_num_experts=S + k)
    np.savez_compressed(
        os.path.join(HERE, "moe.npz"),
        hs=hs.view(torch.int16).numpy(), w13=w13.view(torch.int16).numpy(),
        w2=w2.view(torch.int16).numpy(), expert_map=emap.numpy(),
        topk_ids=ti.numpy(), topk_weights=tw.numpy(),
        out=out.view(torch.int16).numpy())
    print("moe: out", out.float().abs().mean().item())


class _NoEvent:
    def record(self, *a):
        pass

    def synchronize(self):
        pass


def _split_signal_for(decode_rows: int):
    """``_split_signal`` of a real MLA step: rows [0, d) decode (d > 0), a
    pure prefill (0), or short prefills folded into the decode count (-1)."""
    if decode_rows > 0:
        return (decode_rows, decode_rows, True)
    if decode_rows == 0:
        return (0, 0, True)
    return (2, 1, True)


def _run_wave_scenario(name, *, slots, global_n, local_n, owned_lo=0, steps, frac=0.5,
                       pins=None, lfu=False, fast_hit=True):
    """``steps``: [("gap", ids) | ("moe", ids, topk, signal)]: an int signal is
    an MLA decode count (``_split_signal_for``); a list of row indices (or
    None: metadata that does not describe the batch) is what the opt-in
    non-MLA classifier ``_non_mla_decode_rows`` returns for the step."""
    torch.cuda.Event = _NoEvent
    torch.cuda.current_stream = lambda *a: None
    off = _ref_offloader(slots, fast_hit, frac, False, lfu)
    if pins is not None:
        off._pin_layers = {0: list(pins)}
    if local_n == global_n:
        emap, local_of = None, list(range(global_n))
    else:
        lo = [-1] * global_n
        for i in range(local_n):
            lo[owned_lo + i] = i
        emap, local_of = torch.tensor(lo, dtype=torch.int32), lo
    mod = _FakeMoE(local_n, global_n, emap)
    off._install_cache(mod)
    cache = off._caches[id(mod)]
    assert not cache.static_full, name
    off._rs_caches.append(cache)
    log = []
    wm, si = off._write_map, off._stream_in
    off._write_map = lambda c, wave, pinned: (log.append(("map", [list(x) for x in wave])),
                                              wm(c, wave, pinned))[1]
    off._stream_in = lambda c, local, slot, cs, on_stream=False: (
        log.append(("fill", [int(local), int(slot)])), si(c, local, slot, cs, on_stream))[1]
    signal = [(0, 0, True)]
    off._split_signal = lambda: signal[0]
    rows_now = [None]
    off._non_mla_decode_rows = lambda n: (None if rows_now[0] is None
                                          else torch.tensor(rows_now[0], dtype=torch.long))
    trace = []
    for st in steps:
        log.clear()
        rec = {"kind": st[0], "ids": list(st[1])}
        if st[0] == "gap":
            if lfu:
                pairs = [(g, local_of[g], True) for g in sorted(set(st[1]))
                         if 0 <= g < global_n and local_of[g] >= 0]
                off._bump_freq(cache, pairs)
            try:
                off._router_split_gap(0, torch.tensor(st[1], dtype=torch.int32))
                rec["overflow"] = False
            except RuntimeError:
                rec["overflow"] = True
        else:
            _, ids, topk, d = st
            rec["topk"] = topk
            if isinstance(d, int):
                rec["decode_rows"] = d
                off.nonmla_classifier = False
                signal[0] = _split_signal_for(d)
            else:
                # a non-MLA backend: no decode count, rows from query_start_loc
                rec["decode_row_index"] = d
                off.nonmla_classifier = True
                signal[0] = (None, None, True)
                rows_now[0] = d
            t = torch.tensor(ids, dtype=torch.int32).view(-1, topk)
            out = off.run_moe(lambda *a, **k: torch.ones(1), (), {}, mod, t)
            waves, pending = [], []
            for kind, v in log:
                if kind == "fill":
                    pending.append(v)
                else:
                    waves.append({"map": v, "fills": pending})
                    pending = []
            assert not pending and int(out.item()) == len(waves), name
            rec["waves"] = waves
        w = cache.gpu_cache["w"][:, 0]
        stats = off._stats
        rec.update({
            "expert_map": cache.expert_map_buf.tolist(),
            "expert_in_slot": [-1 if v is None else int(v) for v in cache.expert_in_slot],
            "slot_payload": [int(w[s].item()) if cache.expert_in_slot[s] is not None
                             else -1 for s in range(cache.num_slots)],
            "protected": list(cache.protected),
            "probation": list(cache.probation),
            "map_is_standing": bool(cache.map_is_standing),
            "gaps": off._rs_gaps, "misses": off._rs_misses, "fast_hits": off._rs_fast_hits,
            "scan_steps": stats["small"].steps + stats["scan"].steps,
            "scan_hits": stats["small"].hits + stats["scan"].hits,
            "scan_misses": stats["small"].misses + stats["scan"].misses,
            "scan_waves": stats["small"].waves + stats["scan"].waves,
            "freq": [int(cache.freq.get(loc, 0)) for loc in range(local_n)],
        })
        trace.append(rec)
        if rec.get("overflow"):
            break
    return {
        "name": name, "num_slots": cache.num_slots, "global_n": global_n,
        "local_n": local_n, "local_of": local_of, "fast_hit": fast_hit, "lfu": lfu,
        "protect_frac": frac, "protected_cap": cache.protected_cap,
        "pins": list(pins) if pins is not None else None,
        "pinned_slots": sorted(cache.pinned_slots), "trace": trace,
    }


def make_wave_traces():
    g = torch.Generator().manual_seed(2468)

    def prefill(T, k, E, d=0):
        # each token's k distinct ids, uniform
        ids = [i for _ in range(T) for i in torch.randperm(E, generator=g)[:k].tolist()]
        return ("moe", ids, k, d)

    def decode(T, k, E, s=1.1):
        return ("gap", _zipf_ids(g, 1, T, k, E, s=s)[0])

    def mixed(n, Tp, Td, k, E, every=4, d=0):
        out = []
        for i in range(n):
            out.append(prefill(Tp, k, E, d) if i % every == 0 else decode(Td, k, E))
        return out

    sc = [
        _run_wave_scenario("v2lite_prefill_scan", slots=48, global_n=64, local_n=64,
                           steps=[prefill(64, 6, 64) for _ in range(6)]),
        _run_wave_scenario("v2lite_mixed", slots=48, global_n=64, local_n=64,
                           steps=mixed(24, 40, 8, 6, 64)),
        _run_wave_scenario("v2lite_mixed_decode_rows", slots=48, global_n=64, local_n=64,
                           steps=mixed(16, 24, 8, 6, 64, every=3, d=4)
                           + [prefill(16, 6, 64, 16), prefill(30, 6, 64, -1)]),
        _run_wave_scenario("v2lite_frac09_small_groups", slots=48, global_n=64, local_n=64,
                           frac=0.9, steps=mixed(12, 64, 8, 6, 64, every=2)),
        _run_wave_scenario("s8_frac09_one_slot_rotation", slots=8, global_n=32, local_n=32,
                           frac=0.9, steps=[decode(1, 6, 32), prefill(12, 6, 32),
                                            decode(1, 6, 32), prefill(20, 6, 32)]),
        _run_wave_scenario("v2lite_pins_prefill", slots=40, global_n=64, local_n=64,
                           pins=[5, 9, 11, 2], steps=mixed(12, 48, 6, 6, 64, every=3)),
        _run_wave_scenario("v2lite_friendly_small_prefill", slots=48, global_n=64, local_n=64,
                           steps=[prefill(3, 6, 64), prefill(5, 6, 64), prefill(12, 6, 64),
                                  prefill(3, 6, 64)]),
        _run_wave_scenario("ep_rank1_of2_prefill", slots=24, global_n=64, local_n=32,
                           owned_lo=32, steps=mixed(12, 32, 4, 6, 64, every=2)),
        _run_wave_scenario("qwen3_s64_mixed", slots=64, global_n=128, local_n=128,
                           steps=mixed(12, 48, 8, 8, 128, every=3)),
        _run_wave_scenario("v2lite_lfu_mixed", slots=48, global_n=64, local_n=64, lfu=True,
                           steps=mixed(30, 32, 8, 6, 64, every=5)),
        _run_wave_scenario("no_owned_ids", slots=24, global_n=64, local_n=32, owned_lo=0,
                           steps=[("moe", [40, 41, 63, -1, 50, 33] * 8, 6, 0),
                                  decode(4, 6, 64)]),
    ]
    # the opt-in non-MLA classifier: decode rows anywhere in the batch
    rng = torch.Generator().manual_seed(97531)

    def rows_step(T, k, E, n_dec):
        rows = sorted(torch.randperm(T, generator=rng)[:n_dec].tolist())
        ids = [i for _ in range(T) for i in torch.randperm(E, generator=rng)[:k].tolist()]
        return ("moe", ids, k, rows)

    sc += [
        _run_wave_scenario("nonmla_scattered_decode_rows", slots=48, global_n=64, local_n=64,
                           steps=[decode(8, 6, 64), rows_step(40, 6, 64, 5), decode(8, 6, 64),
                                  rows_step(24, 6, 64, 24), rows_step(32, 6, 64, 0),
                                  ("moe", prefill(20, 6, 64)[1], 6, None),
                                  rows_step(48, 6, 64, 9), decode(8, 6, 64)]),
        _run_wave_scenario("nonmla_qwen3_lfu", slots=64, global_n=128, local_n=128, lfu=True,
                           steps=[rows_step(24, 8, 128, 6), decode(8, 8, 128),
                                  rows_step(40, 8, 128, 12), rows_step(16, 8, 128, 1),
                                  decode(8, 8, 128)]),
    ]
    with open(os.path.join(HERE, "wave_traces.json"), "w") as f:
        json.dump({"generator": "tests/golden/make_golden.py", "scenarios": sc}, f,
                  separators=(",", ":"))
    for s in sc:
        nw = [len(r["waves"]) for r in s["trace"] if r["kind"] == "moe"]
        print(f"{s['name']}: steps={len(s['trace'])} waves per moe step={nw}")
    return sc


def make_nonmla_rows():
    import types

    import vllm.forward_context as fc
    from sluice.offloader import ExpertStreamOffloader

    cases = [  # (query_start_loc, num_tokens, max_query_len, num_actual_tokens)
        ([0, 1, 2, 3, 4], 4, 1, 4),                 # pure decode
        ([0, 1, 5, 6, 10], 10, 4, 10),              # decodes at rows 0 and 5
        ([0, 4, 10], 10, 6, None),                  # pure prefill
        ([0, 3, 4, 5, 9, 10, 11], 11, 4, 11),       # decodes at 3, 4, 9, 10
        ([0, 2, 7], 8, 5, 8),                       # query lengths do not cover the batch
        ([0, 1, 2], 2, 1, 3),                       # a padded batch
        ([[0, 1], [1, 2]], 2, 2, 2),                # not a 1-D query_start_loc
        ([0], 0, 2, 0),                             # no requests
    ]
    out = []
    orig = fc.get_forward_context
    try:
        for qsl, T, mql, nat in cases:
            md = types.SimpleNamespace(max_query_len=mql, query_start_loc=torch.tensor(qsl),
                                       num_actual_tokens=nat)
            fc.get_forward_context = lambda md=md: types.SimpleNamespace(attn_metadata=md)
            r = ExpertStreamOffloader._non_mla_decode_rows(T)
            out.append({"query_start_loc": qsl, "num_tokens": T, "max_query_len": mql,
                        "num_actual_tokens": nat, "rows": None if r is None else r.tolist()})
    finally:
        fc.get_forward_context = orig
    with open(os.path.join(HERE, "nonmla_rows.json"), "w") as f:
        json.dump({"generator": "tests/golden/make_golden.py", "cases": out}, f, indent=1)
    print("nonmla rows:", [c["rows"] for c in out])


if __name__ == "__main__":
    if not REF:
        raise SystemExit("set SLUICE_REFERENCE to a checkout of kfirtoledo/sluice")
    sys.path.insert(0, os.path.join(REF, "src"))
    wanted = set(sys.argv[1:]) or {"slots", "routing", "moe", "fp8", "waves", "nonmla"}
    if "slots" in wanted:
        make_slot_traces()
    if "routing" in wanted:
        make_routing()
    if "moe" in wanted:
        make_moe()
    if "fp8" in wanted:
        make_fp8_quant()
    if "waves" in wanted:
        make_wave_traces()
    if "nonmla" in wanted:
        make_nonmla_rows()
