"""Benchmark: offloaded MoE decode on B200 (the reference's headline path).

Workload (the MoE path of a DeepSeek-V2-Lite-shaped
decoder): 26 MoE layers, hidden 2048, 64 routed experts of SwiGLU
intermediate 1408 (bf16, 17.3 MB each) plus 2 shared experts, softmax top-6,
48 GPU slots per layer (16 of 64 experts per layer live only in host RAM),
c = 8 decode tokens per step. Seeded synthetic weights and tokens (no
checkpoints): gate logit bias 1.5*log(1/rank) for Zipf-like popularity, 60%
of each step's tokens reuse the previous step's vector plus noise.

One step = one decode step through all 26 MoE layers (router -> device slot
planner -> GPU-initiated expert streaming -> tcgen05 fused experts with the
shared experts -> residual), replayed as one CUDA graph.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl sluice|reference]

``--impl reference`` times the reference's torch-native CPU path (the oracle
port of routing, the slot policy and the MoE layer) on the host cores.
Prints one JSON line on rank 0.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

METRIC = "decode tok/s"
UNIT = "tok/s"
# PCIe Gen5 x16 host link: 32 GT/s x 16 lanes x 128/130 encoding / 8 bits
PCIE_GEN5_X16_GBS = 63.0


def _args(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="sluice", choices=["sluice", "reference"])
    ap.add_argument("--config", default="deepseek-v2-lite")
    ap.add_argument("--slots", type=int, default=None,
                    help="GPU slots per layer and rank (default: --slots-frac of the local experts)")
    ap.add_argument("--slots-frac", type=float, default=0.75,
                    help="slots per layer as a fraction of each rank's local experts")
    ap.add_argument("--sweep", default="32,40,56",
                    help="slot counts of the one-GPU slots sweep (besides --slots and resident)")
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--tokens", type=int, default=8)
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--prefill-steps", type=int, default=24,
                    help="untimed steps that fill the slot caches before warm-up")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-resident", action="store_true")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--lfu", action="store_true",
                    help="SLUICE_LFU=1: popularity-ordered protected victims (opt-in policy)")
    ap.add_argument("--exchange", default="nvlink", choices=["nvlink", "nccl"],
                    help="expert-parallel dispatch/combine (N>1): peer-memory kernels or NCCL")
    ap.add_argument("--prefetch", type=int, default=0,
                    help="opt-in cross-layer prefetch: experts per layer predicted from the "
                         "previous layer's input and streamed ahead (one GPU; 0 = off)")
    ap.add_argument("--no-overlap", action="store_true",
                    help="serialise the expert stream and the GEMMs (A/B)")
    ap.add_argument("--workload", default="decoder",
                    choices=["decoder", "moe-stack", "grouped-gemm", "prefill"],
                    help="decoder: the DeepSeek-V2-Lite-shaped decoder (MoE layers on this "
                         "build's kernels, attention / dense layer / head in PyTorch); "
                         "moe-stack: the MoE layers alone; grouped-gemm: the fp8 grouped-GEMM "
                         "microbench (one JSON line per T); prefill: steps beyond the "
                         "envelope, expert waves and token chunks")
    ap.add_argument("--prompt-len", type=int, default=128,
                    help="decoder: prompt tokens per sequence (fed before warm-up)")
    ap.add_argument("--gen-len", type=int, default=256,
                    help="decoder: generated tokens per sequence (cache length budget)")
    ap.add_argument("--prefill-tokens", type=int, default=512,
                    help="tokens per step of the prefill workload")
    ap.add_argument("--prefill-modes", default="waves,chunks",
                    help="prefill workload modes to run, in order (waves, chunks)")
    ap.add_argument("--gemm-tokens", default="8,64,512,4096",
                    help="token counts of the grouped-GEMM microbench")
    ap.add_argument("--gemm-experts", type=int, default=256,
                    help="experts of the grouped-GEMM microbench (a smaller profiling case)")
    return ap.parse_args(argv)


def _slots_for(a, cfg, world=1) -> int:
    """GPU slots per layer on each rank: --slots, else --slots-frac of the
    rank's local experts (never more than them)."""
    local_n = cfg.num_experts // world
    s = a.slots if a.slots is not None else max(1, round(a.slots_frac * local_n))
    return min(s, local_n)


def _config(a, cfg, slots, T, layers, world):
    """The workload's config, identical in the GPU arm and the reference arm
    for the same arguments (facts about one arm's run go elsewhere)."""
    local_n = cfg.num_experts // world
    return {"workload": _workload_for(a, cfg, slots, T, layers, world), "model": cfg.name,
            "tokens_per_step": T, "slots": slots, "slots_frac": slots / local_n,
            "layers": layers, "global_batch": T * world, "seq_len": 1,
            "parallelism": f"ep{world}" if world > 1 else "single",
            "slot_policy": ("slru+lfu" if a.lfu else "slru")
                           + (f"+prefetch{a.prefetch}" if a.prefetch and world == 1 else ""),
            "local_experts": local_n,
            "offloaded": slots < local_n,
            "decoder": a.workload == "decoder",
            "cache_prefill": (f"{a.prompt_len}-token prompts" if a.workload == "decoder"
                              else f"{a.prefill_steps} steps"),
            "l2": "per-step expert weights >> 126 MB L2 (no flush needed)"}


def _workload_for(a, cfg, slots, tokens, layers, world=1):
    if a.workload != "decoder":
        return _workload(cfg, slots, tokens, layers, world)
    d = _decoder_cfg(a)
    local = cfg.num_experts // world
    where = (f"{slots} GPU slots, {local - slots} per layer in host RAM" if slots < local
             else "all resident")
    ep = f", expert-parallel over {world} GPUs ({local} experts per rank)" if world > 1 else ""
    return (f"{cfg.name} decoder: {d.num_layers} layers (dense FFN I={d.dense_intermediate} in "
            f"layer 0, {d.num_moe_layers} MoE layers of {cfg.num_experts} experts x "
            f"I={cfg.moe_intermediate} ({where}), top-{cfg.routing.topk}, {cfg.n_shared} "
            f"shared), MLA attention {d.num_heads} heads kv_lora {d.kv_lora_rank}, vocab "
            f"{d.vocab}, H={cfg.hidden}{ep}; {a.prompt_len}-token random prompts, greedy "
            f"decode, c={tokens} per GPU")


def _workload(cfg, slots, tokens, layers, world=1):
    local = cfg.num_experts // world
    where = (f"{slots} GPU slots, {local - slots} per layer in host RAM" if slots < local
             else "all resident")
    ep = f", expert-parallel over {world} GPUs ({local} experts per rank)" if world > 1 else ""
    return (f"{cfg.name} MoE decode stack: {layers} MoE layers, H={cfg.hidden}, "
            f"{cfg.num_experts} experts x I={cfg.moe_intermediate} ({where}){ep}, "
            f"top-{cfg.routing.topk}, {cfg.n_shared} shared, c={tokens} per GPU")


# ------------------------------------------------------------ clock sampling
_REASON_BITS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40,
                "sw_thermal_slowdown": 0x20, "sw_power_cap": 0x4}


class ClockSampler:
    """SM clock, power and throttle reasons of this process's GPU, sampled
    every 10 ms through NVML on a thread while the timed region runs (so even
    a region of tens of milliseconds gets samples); ``nvidia-smi -lms 200`` if
    NVML is unavailable. Read-only: no setting of the GPU is changed."""

    def __init__(self, index: int):
        self.index = index
        self.rows = []
        self._stop = None
        self._thread = None
        self._smi = None

    def _nvml_handle(self):
        import pynvml
        pynvml.nvmlInit()
        try:
            uuid = str(torch.cuda.get_device_properties(self.index).uuid)
            if not uuid.startswith("GPU-"):
                uuid = "GPU-" + uuid
            return pynvml.nvmlDeviceGetHandleByUUID(uuid)
        except Exception:
            return pynvml.nvmlDeviceGetHandleByIndex(self.index)

    def __enter__(self):
        import threading
        try:
            import pynvml
            h = self._nvml_handle()
            mx = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
            self._stop = threading.Event()

            def run():
                while not self._stop.is_set():
                    try:
                        sm = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                        pw = pynvml.nvmlDeviceGetPowerUsage(h) / 1000.0
                        rs = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                        self.rows.append((sm, mx, pw, rs))
                    except Exception:
                        pass
                    self._stop.wait(0.01)

            self._thread = threading.Thread(target=run, daemon=True)
            self._thread.start()
        except Exception:
            self._start_smi()
        return self

    def _start_smi(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self._smi = subprocess.Popen(["nvidia-smi", f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-i",
                                          str(self.index), "-lms", "200"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self._smi = None

    def __exit__(self, *a):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=5)
        if self._smi is not None:
            self._smi.terminate()
            try:
                self._smi.wait(timeout=5)
            except Exception:
                self._smi.kill()

    def summary(self):
        if self._thread is not None:
            if not self.rows:
                return None
            sm = [r[0] for r in self.rows]
            reasons = sorted({n for r in self.rows for n, bit in _REASON_BITS.items()
                              if r[3] & bit})
            return {"sm_mhz": statistics.median(sm), "sm_max_mhz": self.rows[0][1],
                    "power_w_max": max(r[2] for r in self.rows), "reasons": reasons,
                    "samples": len(self.rows), "source": "nvml, 10 ms"}
        try:
            self.f.flush()
            with open(self.f.name) as fh:
                rows = [r.split(", ") for r in fh.read().strip().splitlines() if r.strip()]
            os.unlink(self.f.name)
        except Exception:
            return None
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = max(float(r[2]) for r in rows)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4)
                          if len(r) > 5 + i and r[5 + i].strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": reasons, "samples": len(rows), "source": "nvidia-smi, 200 ms"}


# --------------------------------------------------------------- CPU port
def cpu_layer_runner(cfg, seed, n_weight_sets=1):
    """The reference's torch-native CPU path for one layer (oracle port):
    gate + routing, the gap's slot policy, the MoE with shared experts."""
    from oracle import moe as omoe
    from oracle import routing as orouting
    from oracle.slot_policy import SlotPolicyModel
    from sluice_b200 import synth

    dev = "cuda" if torch.cuda.is_available() else "cpu"
    sets = []
    for li in range(n_weight_sets):
        w13, w2 = synth.layer_weights(cfg, li, seed, device=dev)
        sh13, sh2 = synth.shared_weights(cfg, li, seed, device=dev)
        gw, lb, sb = synth.gate_params(cfg, li, seed, device="cpu")
        cpu = lambda t: None if t is None else t.cpu()
        sh = None
        if sh13 is not None:
            # one shared MLP of intermediate n*I, as the reference's shared_layer
            n, I = cfg.n_shared, cfg.moe_intermediate
            g13 = torch.cat([sh13[:, :I].reshape(n * I, -1), sh13[:, I:].reshape(n * I, -1)])
            g2 = sh2.permute(1, 0, 2).reshape(cfg.hidden, n * I)
            sh = (g13.cpu(), g2.cpu())
        sets.append((w13.cpu(), w2.cpu(), gw, lb, sb, sh))
        del w13, w2
    rc = cfg.routing
    policies = {}

    def run_layer(li, x, slots, decode=True):
        w13, w2, gw, lb, sb, sh = sets[li % n_weight_sets]
        logits = orouting.gate_logits(x, gw, lb)
        tw, ti = orouting.grouped_topk(logits, rc.topk, rc.renormalize, rc.num_expert_group,
                                       rc.topk_group, rc.scoring_func, 1.0, sb)
        pol = policies.setdefault(li, SlotPolicyModel(slots, list(range(cfg.num_experts)),
                                                      cfg.num_experts, 0.5, True))
        env = max(1, min(slots, cfg.num_experts) // rc.topk)
        if slots < cfg.num_experts and x.shape[0] > env:
            # beyond the envelope: the classic hook's expert waves (decode
            # steps decode-class, others by the working-set heuristic); the
            # waves' outputs add up to the MoE over every pair, computed once
            pol.run_moe(ti.flatten().tolist(), rc.topk, x.shape[0] if decode else 0)
        else:
            pol.gap(ti.flatten().tolist())
        routed = omoe.fused_experts(x, w13, w2, tw, ti)
        shared = omoe.shared_experts(x, *sh) if sh is not None else None
        return omoe.layer_output(routed, shared, cfg.routed_scaling_factor)

    run_layer.policies = policies
    return run_layer


def cpu_step_time(cfg, slots, tokens, layers, seed, steps, warmup, budget_s=None,
                  decode=True):
    """Seconds per full step of the CPU port (all layers): a decode step, or
    with ``decode=False`` a prefill-sized one (fresh random tokens)."""
    from sluice_b200 import synth

    run = cpu_layer_runner(cfg, seed, n_weight_sets=layers)
    stream = synth.TokenStream(cfg.hidden, tokens, seed=seed, reuse=0.6 if decode else 0.0)
    times = []
    t_start = time.perf_counter()
    for s in range(warmup + steps):
        x = stream.next()
        t0 = time.perf_counter()
        h = x
        for li in range(layers):
            h = h + run(li, h, slots, decode)
        dt = time.perf_counter() - t0
        if s >= warmup:
            times.append(dt)
        if budget_s is not None and s >= warmup and time.perf_counter() - t_start > budget_s:
            break
    return statistics.median(times), len(times)


def cpu_decoder_step_time(a, cfg, slots, T, layers, seed, steps, warmup, budget_s=None):
    """Seconds per decode step of the CPU port of the decoder workload: the
    same PyTorch decoder harness on the host, its MoE layers through the
    oracle's routing, slot policy and torch-native MoE (each layer its own
    weights); the prompts are fed first, untimed."""
    from sluice_b200.harness import DecoderHarness

    dcfg = _decoder_cfg(a)
    run = cpu_layer_runner(cfg, seed, n_weight_sets=layers)
    h = DecoderHarness(dcfg, lambda li, x: run(li, x, slots), T,
                       a.prompt_len + warmup + steps + 1, seed, device="cpu")
    g = torch.Generator().manual_seed(seed + 31)
    prompt = torch.randint(0, dcfg.vocab, (a.prompt_len, T), generator=g)
    ids = None
    for p in range(a.prompt_len):
        ids = h.step(prompt[p])
    times = []
    t_start = time.perf_counter()
    for s_ in range(warmup + steps):
        t0 = time.perf_counter()
        ids = h.step(ids)
        dt = time.perf_counter() - t0
        if s_ >= warmup:
            times.append(dt)
        if budget_s is not None and s_ >= warmup and time.perf_counter() - t_start > budget_s:
            break
    return statistics.median(times), len(times)


def _cpu_time(a, cfg, slots, T, layers, seed, steps, warmup, budget_s):
    if a.workload == "decoder":
        return cpu_decoder_step_time(a, cfg, slots, T, layers, seed, steps, warmup, budget_s)
    return cpu_step_time(cfg, slots, T, layers, seed, steps=steps, warmup=warmup,
                         budget_s=budget_s)


# ---------------------------------------------------------------- GPU arm
def h2d_ceiling_gbs(nbytes=1 << 30):
    src = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    dst = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    dst.copy_(src, non_blocking=True)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    best = 0.0
    for _ in range(3):
        a.record()
        dst.copy_(src, non_blocking=True)
        b.record()
        b.synchronize()
        best = max(best, nbytes / (a.elapsed_time(b) * 1e-3) / 1e9)
    del src, dst
    return best


def _graph_time_ms(fn, reps=10):
    """Device time per call of `fn` captured in a CUDA graph (no host gaps)."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        g.replay()
    b.record()
    b.synchronize()
    del g
    return a.elapsed_time(b) / reps


def profile_layers(stack, x):
    """Per-layer device time of route and fused_experts, each replayed as its
    own CUDA graph on the inputs of one real decode step; returns the lists
    of (ms, algorithmic bytes)."""
    from sluice_b200 import ops

    cfg = stack.layers[0].cfg   # the MoE layers' config (also under the decoder)
    bpe = cfg.bytes_per_expert
    route_ms, fused_ms, fused_bytes = [], [], []
    h = x
    for layer in stack.layers:
        tw, ti, _ = layer.router.route(h)
        layer.cache.gap(ti)
        out = torch.empty_like(h)
        hs = h.clone()
        fused = lambda: ops.fused_experts(hs, layer.cache.w13, layer.cache.w2, tw, ti,
                                          global_num_experts=cfg.num_experts,
                                          expert_map=layer.cache.expert_map,
                                          shared_w13=layer.shared_w13,
                                          shared_w2=layer.shared_w2,
                                          w1_scale=layer.cache.w13_scale,
                                          w2_scale=layer.cache.w2_scale,
                                          shared_w13_scale=layer.shared_w13_scale,
                                          shared_w2_scale=layer.shared_w2_scale,
                                          routed_scaling_factor=cfg.routed_scaling_factor,
                                          out=out)
        fused_ms.append(_graph_time_ms(fused))
        route_ms.append(_graph_time_ms(lambda: layer.router.route(hs)))
        # the experts this cache serves (all of them on one GPU; this rank's
        # under expert parallelism)
        emap = layer.cache.expert_map.cpu()
        ids = ti.flatten().cpu().long()
        valid = (ids >= 0) & (ids < emap.numel())
        u = len(set(ids[valid][emap[ids[valid]] >= 0].tolist()))
        fused_bytes.append((u + cfg.n_shared) * bpe)
        h = h + out
    torch.cuda.synchronize()
    return route_ms, fused_ms, fused_bytes


def stream_probe(stack, n_miss=12, ctas=(16, 32, 64, 128, 148)):
    """Streamer bandwidth: plan a gap that misses `n_miss` experts on layer 0,
    then re-run the streamer over that fill list (idempotent) per CTA count."""
    import ctypes
    from sluice_b200._lib import check, lib, ptr

    layer = stack.layers[0]
    cache = layer.cache
    if cache.state is None:
        return None
    resident = set(v for v in cache.snapshot()["expert_in_slot"] if v >= 0)
    cold = [e for e in range(cache.local_n) if e not in resident][:n_miss]
    if not cold:
        return None
    ids = torch.tensor(cold, dtype=torch.int32, device="cuda")
    cache.gap(ids)
    torch.cuda.synchronize()
    fills = cache.header()["fill_count"]
    n, src, dst, nb, hs = cache._stream_args
    out = {}
    for c in ctas:
        s = lambda: check(lib().sl_stream_experts_strided(
            ptr(cache.state), n, src, dst, nb, hs, c, torch.cuda.current_stream().cuda_stream),
            "stream")
        ms = _graph_time_ms(s, reps=5)
        out[c] = fills * cache.bytes_per_expert / (ms * 1e-3) / 1e9
    return {"fills": fills, "gbs_by_ctas": out}


def _traffic_per_launch(fbytes, cfg):
    """DRAM bytes per fused_experts launch: the ncu-measured bytes per expert
    (profiles/traffic.json, a smaller capture) times this run's mean experts
    per launch (DRAM traffic grows in proportion to the experts streamed)."""
    per = load_traffic().get("fused_experts_traffic_bytes_per_expert")
    if not per:
        return None
    return per * statistics.mean(fbytes) / cfg.bytes_per_expert


def load_traffic():
    p = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(p) as f:
            return json.load(f)
    except Exception:
        return {}


def _timed_c1(stack, cfg, K, W, seed, a=None):
    """Decode at concurrency 1 on the same MoE layers (its own CUDA graph;
    the decoder workload: a one-sequence decoder around them, after its own
    prompt)."""
    from sluice_b200 import synth

    if a is not None and a.workload == "decoder":
        from sluice_b200.harness import OffloadedDecoder
        eng = OffloadedDecoder(_decoder_cfg(a), stack.stack, 1, a.prompt_len + a.gen_len, seed)
        eng.capture()
        _precondition(a, eng, cfg, 1, 0)
        xs = [None] * (W + K)
    else:
        eng = stack
        eng.capture(tokens=1)
        st = synth.TokenStream(cfg.hidden, 1, seed=seed + 777)
        xs = torch.stack([st.next() for _ in range(W + K)]).cuda()
    for i in range(W):
        eng.replay(xs[i])
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(K):
        eng.replay(xs[W + i])
    e1.record()
    torch.cuda.synchronize()
    eng.check()
    ms = e0.elapsed_time(e1) / K
    return {"value": 1.0 / (ms * 1e-3), "unit": UNIT, "ms_per_step": ms}


def _step_bytes(stack, cfg):
    """Algorithmic HBM bytes of the last step's expert GEMMs on this rank:
    sum over layers of (distinct resident selected experts + shared) x bytes."""
    tot = 0
    for layer in stack.layers:
        ids = layer.last_ids
        if ids is None:
            continue
        emap = layer.cache.expert_map
        sel = ids.flatten().long()
        sel = sel[(sel >= 0) & (sel < emap.numel())]
        u = torch.unique(sel[emap[sel] >= 0]).numel()
        tot += (u + cfg.n_shared) * cfg.bytes_per_expert
    return tot


def layer_launches(cfg, tokens, world, slots, exchange="nvlink", no_overlap=False,
                   decode=True) -> int:
    """This build's kernel launches per MoE layer and step, following the
    launch rules of the host code: gate + select; a fused-experts call is its
    token grouping (one kernel for up to 1024 bf16 pairs, else grouping +
    gather; fp8: grouping + quantising gather), the gate/up and down GEMMs and
    the combine (an offloaded layer issues it in parts: grouping, the
    resident experts' GEMMs, the streamed experts' GEMMs on the stream's side
    stream, the combine: the GEMMs twice); an offloaded gap adds plan +
    stream; a
    step beyond the envelope runs max_waves waves (one plan, a stream per
    wave, wave 0 split in two phases, the rest whole calls; decode steps,
    every expert decode-class, take the tighter wave count); the NVLink
    exchange adds dispatch + combine."""
    from sluice_b200.offloader import max_waves_for, protected_cap_for

    local_n = cfg.num_experts // world
    k = cfg.routing.topk
    fp8 = cfg.weight_dtype == "fp8"
    align = 2 if fp8 or tokens * world * k > 1024 else 1
    ex = 2 if world > 1 and exchange == "nvlink" else 0
    if slots >= local_n:
        return 2 + align + 3 + ex
    S = min(slots, local_n)
    if tokens > max(1, S // k // world):
        mw = max_waves_for(S, min(local_n, tokens * world * k), protected_cap_for(S, 0.5), 0,
                           all_decode=decode)
        return 2 + 1 + mw + (align + 5) + (mw - 1) * (align + 3) + ex
    return 2 + 2 + (align + 3 if no_overlap else align + 5) + ex


def harness_launches(num_layers, tokens) -> int:
    """This build's kernels per decode step in the decoder harness around the
    MoE layers: the first RMSNorm, then per layer the MLA attention kernel
    and two residual add + RMSNorm kernels, and for one or two rows the q/kv
    and output projections (cuBLAS, not counted, above that)."""
    return 1 + num_layers * (3 + (2 if tokens <= 2 else 0))


def _stack_save(stack):
    """Device copies of every offloaded layer's planner state, map and slots,
    or None when they would not fit in 80% of free HBM."""
    need = sum(sum(t.numel() * t.element_size() for t in layer.cache.gpu_cache.values())
               for layer in stack.layers if not layer.cache.static_full)
    if need > 0.8 * torch.cuda.mem_get_info()[0]:
        return None
    snap = [None if layer.cache.static_full else layer.cache.save() for layer in stack.layers]
    own = stack.save() if hasattr(stack, "save") else None   # the decoder's sequences
    return snap, own


def _stack_restore(stack, snap) -> None:
    caches, own = snap
    for layer, sv in zip(stack.layers, caches):
        if sv is not None:
            layer.cache.restore(sv)
    if own is not None:
        stack.restore(own)
    torch.cuda.synchronize()


def _misses(s0, s1):
    """Experts missed (gap misses + misses of wave-planned steps) and streamed."""
    m = sum(s1.get(k, 0) - s0.get(k, 0) for k in ("misses", "scan_misses"))
    return m, s1.get("fills", 0) - s0.get("fills", 0)


def _max_over_ranks(v, dist):
    if not dist:
        return v
    t = torch.tensor([v], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _sum_over_ranks(vals, dist):
    if not dist:
        return vals
    t = torch.tensor(vals, device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return t.tolist()


def _timed_replays(stack, xs, W, K, dist, clocks=True):
    """ms for K graph replays on xs[W:W+K] (barrier + synchronize on both
    sides, CUDA events on the replaying stream, max over ranks), with the
    slot-cache counters before and after and the SM clocks sampled meanwhile."""
    s0 = stack.stats()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clk = ClockSampler(torch.cuda.current_device()) if clocks else None
    if clk:
        clk.__enter__()
        time.sleep(0.05)  # the sampling thread reaches its steady state first
    # an NVTX range marks the timed replays for profilers (--nvtx-include)
    torch.cuda.nvtx.range_push("sluice_timed")
    ev0.record()
    for i in range(K):
        stack.replay(xs[W + i])
    ev1.record()
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_pop()
    if clk:
        clk.__exit__()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    stack.check()
    ms = _max_over_ranks(ev0.elapsed_time(ev1), dist)
    return ms, s0, stack.stats(), (clk.summary() if clk else None)


def _stream_launch_window(stack, xs, W, K, bpe):
    """Every expert-stream launch of K steps replayed on xs[W:W+K], each step
    synchronised so that its launches' CUDA events (recorded on the stream
    the streamer runs on, inside the captured graph) and fill counts can be
    read: [(ms, bytes)] per launch."""
    rows = []
    for i in range(K):
        stack.replay(xs[W + i])
        torch.cuda.synchronize()
        for layer in stack.layers:
            if layer.stream_timer is None or layer.cache.static_full:
                continue
            la = layer.stream_timer.launches()
            waves = any(w >= 0 for _, w, _ in la)
            counts = layer.cache.last_fill_counts(wave_steps=waves)
            for ms, w, other in la:
                if other is not None:   # a prefetch into the next layer's cache
                    n = other.header()["prefetch_fills"]
                else:
                    n = counts[w] if w >= 0 else counts[0]
                rows.append((ms, n * bpe))
    return rows


def _step_roofline(hbm_step, host_step, t_ms, hbm_peak):
    t_roof = max(hbm_step / (hbm_peak * 1e9), host_step / PCIE_GEN5_X16_GBS / 1e9) * 1e3
    return {"t_roof_ms": t_roof, "t_ms": t_ms, "frac": t_roof / t_ms,
            "hbm_bytes_per_step": hbm_step, "host_bytes_per_step": host_step,
            "host_peak_gbs": PCIE_GEN5_X16_GBS, "hbm_peak_gbs": hbm_peak,
            "bound": "host link" if host_step / PCIE_GEN5_X16_GBS > hbm_step / hbm_peak
            else "hbm"}


def _build_stack(cfg, slots, layers, T, a, world, timers=False):
    """The measured engine, captured for T tokens per GPU: the MoE decode
    stack (``--workload moe-stack``) or the V2-Lite-shaped decoder around it
    (``--workload decoder``: attention, dense layer, head in PyTorch)."""
    from sluice_b200.layer import MoEDecodeStack, StreamTimer

    decoder = a.workload == "decoder"
    if world > 1:
        from sluice_b200.ep import EPDecodeStack
        stack = EPDecodeStack(cfg, slots=slots, seed=a.seed, num_layers=layers,
                              exchange=a.exchange, max_tokens=T, overlap=not a.no_overlap)
    else:
        stack = MoEDecodeStack(cfg, slots=slots, seed=a.seed, num_layers=layers,
                               overlap=not a.no_overlap, prefetch=a.prefetch)
    if timers:
        for layer in stack.layers:
            layer.stream_timer = StreamTimer()
    if decoder:
        from sluice_b200.harness import OffloadedDecoder
        eng = OffloadedDecoder(_decoder_cfg(a), stack, T, a.prompt_len + a.gen_len, a.seed)
        return eng, eng.capture()
    graphed = stack.capture(tokens=T)
    return stack, (True if graphed is None else bool(graphed))


def _decoder_cfg(a):
    """The V2-Lite-shaped decoder (--layers: its MoE layers, default 26)."""
    from dataclasses import replace

    from sluice_b200 import harness

    if a.config != "deepseek-v2-lite":
        raise ValueError("the decoder workload has the DeepSeek-V2-Lite shape")
    d = harness.V2_LITE_DECODER
    return replace(d, num_layers=d.first_dense + a.layers) if a.layers else d


def _precondition(a, eng, cfg, T, rank):
    """Fill the slot caches before warm-up: the moe-stack replays
    --prefill-steps synthetic decode steps; the decoder feeds each sequence's
    prompt of --prompt-len uniform random token ids, one position per step."""
    from sluice_b200 import synth

    if a.workload == "decoder":
        g = torch.Generator().manual_seed(a.seed + 31 + rank)
        prompt = torch.randint(0, _decoder_cfg(a).vocab, (a.prompt_len, T), generator=g).cuda()
        for p in range(a.prompt_len):
            eng.replay(prompt[p])
    else:
        stream = synth.TokenStream(cfg.hidden, T, seed=a.seed + 100 + rank)
        for _ in range(a.prefill_steps):
            eng.replay(stream.next().cuda())
    torch.cuda.synchronize()


def _step_inputs(a, cfg, T, n, rank, seed_off=0):
    """Inputs of n steps: synthetic hidden states (moe-stack), or None for
    the decoder (each step feeds back its own greedy ids)."""
    from sluice_b200 import synth

    if a.workload == "decoder":
        return [None] * n
    stream = synth.TokenStream(cfg.hidden, T, seed=a.seed + 100 + rank + seed_off)
    # continue the preconditioning stream (same seed) past its steps
    if seed_off == 0:
        for _ in range(a.prefill_steps):
            stream.next()
    return torch.stack([stream.next() for _ in range(n)]).cuda()


def _io_bytes(a, cfg, T):
    """Host bytes in and out per step and GPU for the e2e window."""
    return T * 8 if a.workload == "decoder" else T * cfg.hidden * 2


def _sweep_point(a, cfg, slots, layers, K, W, hbm_peak):
    """One point of decode tok/s against the slot count (one GPU): c=T and
    c=1 on fresh caches, with misses per step and the step roofline."""
    out = {"slots": slots, "slots_frac": slots / cfg.num_experts}
    for T in (a.tokens, 1):
        eng, _ = _build_stack(cfg, slots, layers, T, a, 1)
        _precondition(a, eng, cfg, T, 0)
        xs = _step_inputs(a, cfg, T, W + K, 0)
        for i in range(W):
            eng.replay(xs[i])
        torch.cuda.synchronize()
        ms, s0, s1, clk = _timed_replays(eng, xs, W, K, None)
        m, f = _misses(s0, s1)
        roof = _step_roofline(_step_bytes(eng, cfg), f / K * cfg.bytes_per_expert, ms / K,
                              hbm_peak)
        out[f"c{T}"] = {"value": T * K / (ms * 1e-3), "unit": UNIT, "ms_per_step": ms / K,
                        "misses_per_step": m / K, "step_roofline_frac": roof["frac"],
                        "clocks": clk}
        if hasattr(eng, "release"):
            eng.release()
        del eng, xs
        _free()
    return out


def _free():
    import gc

    gc.collect()
    torch.cuda.empty_cache()


def run_sluice(a):
    import datetime

    if a.lfu:
        os.environ["SLUICE_LFU"] = "1"

    from sluice_b200 import configs, synth

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    cfg = configs.CONFIGS[a.config]
    layers = a.layers or cfg.num_moe_layers
    T = a.tokens
    local_n = cfg.num_experts // world
    slots = _slots_for(a, cfg, world)
    offloaded = slots < local_n
    bpe = cfg.bytes_per_expert
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except Exception:
        pass
    hbm_peak = peaks.get("hbm_gbs", 6650.0)

    t_build = time.perf_counter()
    stack, graphed = _build_stack(cfg, slots, layers, T, a, world, timers=offloaded)
    build_s = time.perf_counter() - t_build
    # preconditioning (fill the slot caches; the decoder's prompts), then the
    # W warm-up steps
    _precondition(a, stack, cfg, T, rank)
    K, W = a.steps, a.warmup
    xs = _step_inputs(a, cfg, T, W + K, rank)
    for i in range(W):
        stack.replay(xs[i])
    torch.cuda.synchronize()
    # the e2e and stream-timing windows replay the timed window's inputs from
    # the same cache state (planner state, maps and slot contents restored)
    snap = _stack_save(stack)
    restored = _max_over_ranks(0.0 if snap is not None else 1.0, dist) == 0.0
    ms, s0, s1, clocks = _timed_replays(stack, xs, W, K, dist)
    value = world * T * K / (ms * 1e-3)
    misses, fills = _misses(s0, s1)
    misses, fills = _sum_over_ranks([misses, fills], dist)
    hbm_step = _step_bytes(stack, cfg)

    # end to end through the public call: pinned host in, host out
    if restored:
        _stack_restore(stack, snap)
    decoder = a.workload == "decoder"
    if decoder:
        # the serving loop: each step's ids go to the host and come back in
        oh = torch.empty(K + 1, T, dtype=torch.long).pin_memory()
        oh[0].copy_(stack._ids)
        xh = oh[:-1]
    else:
        xh = xs[W:W + K].cpu().pin_memory()
        oh = torch.empty(K, T, cfg.hidden, dtype=torch.bfloat16).pin_memory()
    se0 = stack.stats()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(K):
        stack.decode_step(xh[i], oh[i + 1] if decoder else oh[i])
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = _max_over_ranks(e0.elapsed_time(e1), dist)
    stack.check()
    e2e_misses, _ = _misses(se0, stack.stats())
    e2e_misses = _sum_over_ranks([e2e_misses], dist)[0]

    # the dominant kernel of an offloaded step: the expert streamer, each
    # launch timed by CUDA events on its own (side) stream inside the graph
    stream_rows = []
    if offloaded:
        if restored:
            _stack_restore(stack, snap)
        stream_rows = _stream_launch_window(stack, xs, W, K, bpe)
    del snap
    st_bytes, st_ms, st_n = _sum_over_ranks(
        [float(sum(b for _, b in stream_rows)), float(sum(t for t, _ in stream_rows)),
         float(len(stream_rows))], dist)
    h2d = h2d_ceiling_gbs()
    host_step = fills / K * bpe / world   # per rank: each streams over its own link
    step_roof = _step_roofline(hbm_step, host_step, ms / K, hbm_peak)
    traffic = load_traffic()

    roof_stream = None
    if st_n and st_ms > 0:
        gbs = st_bytes / (st_ms * 1e-3) / 1e9
        per_launch = st_bytes / st_n
        ratio = traffic.get("stream_kernel_dram_bytes_per_streamed_byte")
        pcie = traffic.get("stream_kernel_pcie_read_bytes_per_streamed_byte")
        roof_stream = {
            "bound": "host link", "kernel": "stream_kernel (expert streamer, side stream)",
            "achieved": gbs, "peak": PCIE_GEN5_X16_GBS, "unit": "GB/s",
            "frac": gbs / PCIE_GEN5_X16_GBS,
            "traffic": per_launch * ratio if ratio else None,
            "traffic_pcie_read": per_launch * pcie if pcie else None,
            "peak_source": "PCIe Gen5 x16, 32 GT/s x 16 x 128/130 / 8 (host link; "
                           "MEASURED_PEAKS.json has no host-link figure)",
            "copy_engine_ceiling_gbs": h2d, "frac_of_copy_engine_ceiling": gbs / h2d,
            "launches": int(st_n), "bytes_per_launch": per_launch,
            "avg_launch_ms": st_ms / st_n,
            "timing": "CUDA events recorded on the streamer's side stream around every "
                      "launch inside the captured step graph; the timed window's K steps "
                      "replayed on the same inputs from the same restored cache state"
                      + (", summed over ranks" if world > 1 else "")}

    sprobe = None
    # fused_experts: each layer's call replayed as its own CUDA graph (under
    # expert parallelism: this rank's experts on its own tokens; the slowest
    # rank's figures are reported)
    hx = synth.TokenStream(cfg.hidden, T, seed=a.seed + 555 + rank).next().cuda()
    route_ms, fused_ms, fbytes = profile_layers(stack, hx)
    t_fused = _max_over_ranks(statistics.mean(fused_ms), dist)
    t_route = _max_over_ranks(statistics.mean(route_ms), dist)
    f_bytes = statistics.mean(fbytes)
    fused_gbs = f_bytes / (t_fused * 1e-3) / 1e9
    roof_fused = {"bound": "hbm", "kernel": "fused_experts (align+gate/up+down+combine)",
                  "achieved": fused_gbs, "peak": hbm_peak, "unit": "GB/s",
                  "frac": fused_gbs / hbm_peak,
                  "traffic": _traffic_per_launch(fbytes, cfg),
                  "peak_source": "MEASURED_PEAKS.json hbm_gbs (measured)",
                  "per_launch_ms": {"route": t_route, "fused": t_fused},
                  "fused_bytes_per_launch": f_bytes,
                  "timing": "each layer's fused_experts replayed as its own CUDA graph, "
                            "CUDA events, mean over layers"
                            + ("; this rank's experts on its own tokens, slowest rank"
                               if world > 1 else "")}
    if world == 1 and offloaded:
        sprobe = stream_probe(stack)
    # the dominant kernel of the step: the expert streamer or the fused
    # experts, whichever takes more device time per step (per rank)
    roof = roof_fused
    fused_ms_step = t_fused * layers
    roof_fused["ms_per_step"] = fused_ms_step
    if roof_stream is not None:
        stream_ms_step = st_ms / K / (world if world > 1 else 1)
        roof_stream["ms_per_step"] = stream_ms_step
        if stream_ms_step >= fused_ms_step:
            roof = roof_stream
    roof_other = roof_stream if roof is roof_fused else roof_fused

    c1 = None
    if world == 1 and T != 1:
        c1 = _timed_c1(stack, cfg, K, W, a.seed, a)
    if hasattr(stack, "release"):
        stack.release()
    del stack, xs
    _free()

    # decode tok/s against the slot count (one GPU): the metric's second axis
    sweep = None
    if world == 1 and offloaded and not a.no_sweep:
        sweep = []
        for sv in [int(v) for v in a.sweep.split(",") if v]:
            if sv == slots or sv >= local_n:
                continue
            sweep.append(_sweep_point(a, cfg, sv, layers, K, W, hbm_peak))

    # resident comparison: same kernels, every local expert in HBM
    resident = None
    resident_bytes = layers * (local_n + cfg.n_shared) * bpe
    fits = resident_bytes < 0.8 * torch.cuda.mem_get_info()[1]
    if not a.no_resident and offloaded and not fits:
        resident = {"skipped": f"{resident_bytes / 1e9:.0f} GB of experts do not fit one GPU"}
    elif not a.no_resident and offloaded:
        rs, _ = _build_stack(cfg, local_n, layers, T, a, world)
        _precondition(a, rs, cfg, T, rank)
        rx = _step_inputs(a, cfg, T, W + K, rank)
        for i in range(W):
            rs.replay(rx[i])
        torch.cuda.synchronize()
        rms, _, _, rclk = _timed_replays(rs, rx, W, K, dist, clocks=False)
        resident = {"value": world * T * K / (rms * 1e-3), "unit": UNIT,
                    "slots": local_n, "ms_per_step": rms / K}
        if world == 1:
            resident["c1"] = _timed_c1(rs, cfg, K, W, a.seed, a)
        if hasattr(rs, "release"):
            rs.release()
        del rs, rx
        _free()

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        torch.set_num_threads(os.cpu_count() or 1)
        t_cpu, n = _cpu_time(a, cfg, slots, T, layers, a.seed, K, max(1, min(W, 2)), 150.0)
        cpu = {"value": T / t_cpu, "unit": UNIT, "cores": torch.get_num_threads(),
               "kind": "port",
               "sample": f"{n} full decode steps ({a.workload}, {layers} MoE layers, c={T}, "
                         f"each layer its own weights) of the torch-native CPU path (oracle "
                         f"routing + slot policy + MoE), median; the same sampling as the "
                         f"reference arm"}

    launches = K * layers * layer_launches(cfg, T, world, slots, a.exchange, a.no_overlap)
    if a.workload == "decoder":
        launches += K * harness_launches(_decoder_cfg(a).num_layers, T)
    if a.prefetch and offloaded and world == 1 and not a.no_overlap:
        # each layer but the last: the next router (gate + select), the
        # prefetch planner and its stream
        launches += K * (layers - 1) * 4
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": K,
        "warmup": W, "ms_per_step": ms / K, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16" if cfg.weight_dtype == "bf16" else "fp8e4m3 weights, bf16 activations",
        "data": "synthetic",
        "config": _config(a, cfg, slots, T, layers, world),
        "run": {"cuda_graph": graphed, "stream_overlap": offloaded and not a.no_overlap,
                "ep_exchange": a.exchange if world > 1 else None,
                "build_s": round(build_s, 1)},
        "e2e": {"value": world * T * K / (e2e_ms * 1e-3), "unit": UNIT,
                "h2d_bytes_per_step": world * _io_bytes(a, cfg, T),
                "d2h_bytes_per_step": world * _io_bytes(a, cfg, T),
                "misses_per_step": e2e_misses / K,
                "window": "the timed window's inputs"
                          + (" from its restored cache state (planner state, expert maps "
                             "and slot contents)" if restored else
                             ", continuing from the cache state the timed window left")},
        "roofline": roof,
        "roofline_other": roof_other,
        "step_roofline": step_roof,
        "stream": {"misses_per_step": misses / K, "fills_per_step": fills / K,
                   "bytes_per_step": fills / K * bpe, "probe": sprobe,
                   "h2d_ceiling_gbs": h2d, "pcie_gen5_x16_gbs": PCIE_GEN5_X16_GBS},
        "c1": c1,
        "slots_sweep": sweep,
        "resident": resident,
        "cpu_baseline": cpu,
        "gpu_launches": launches,
        "clocks": clocks,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()

# ------------------------------------------------- grouped-GEMM microbench
def fp8_peak_tflops(n=8192, reps=10):
    """Burst fp8 e4m3 GEMM throughput of this GPU (cuBLASLt through
    ``torch._scaled_mm``, n^3, best of ``reps``): the fp8 tensor denominator."""
    a = torch.randn(n, n, device="cuda").to(torch.float8_e4m3fn)
    b = torch.randn(n, n, device="cuda").to(torch.float8_e4m3fn).t()
    one = torch.ones((), device="cuda")
    for _ in range(3):
        torch._scaled_mm(a, b, one, one, out_dtype=torch.bfloat16)
    best = float("inf")
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
        e0.record()
        torch._scaled_mm(a, b, one, one, out_dtype=torch.bfloat16)
        e1.record()
        torch.cuda.synchronize()
        best = min(best, e0.elapsed_time(e1))
    return 2 * n ** 3 / (best * 1e-3) / 1e12


def run_grouped_gemm(a):
    """fp8 grouped expert GEMM at DeepSeek-V3 expert shapes (E=256, H=7168,
    I=2048, 128x128 block scales): experts 0..127 resident in slots, 128..255
    streamed from mapped pinned host RAM on every call; T tokens, top-8 ids
    Zipf(1.1) over a seeded expert permutation, renormalised fp32 weights.
    Per T: the all-resident GEMM alone, the stream alone, and the overlapped
    call (plan -> stream on a side stream || resident experts' GEMMs ->
    streamed experts' GEMMs), each against its roofline."""
    from sluice_b200 import configs, ops, synth
    from sluice_b200.offloader import ExpertStreamOffloader

    cfg = configs.DEEPSEEK_V3
    E, H, I, k = a.gemm_experts, cfg.hidden, cfg.moe_intermediate, 8
    half = E // 2
    dev = torch.device("cuda")
    with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
        peaks = json.load(f)
    hbm_peak, bf16_peak = peaks["hbm_gbs"], peaks["bf16_tflops"]
    fp8_peak = fp8_peak_tflops()
    # weights, generated and quantised 32 experts at a time
    w13 = torch.empty(E, 2 * I, H, dtype=torch.float8_e4m3fn, device=dev)
    w2 = torch.empty(E, H, I, dtype=torch.float8_e4m3fn, device=dev)
    s13 = torch.empty(E, 2 * I // 128, H // 128, dtype=torch.float32, device=dev)
    s2 = torch.empty(E, H // 128, I // 128, dtype=torch.float32, device=dev)
    for lo in range(0, E, 32):
        n = min(32, E - lo)
        prm = synth.layer_params(cfg, 0, a.seed, device=dev, num_experts=n, expert_lo=lo)
        w13[lo:lo + n].copy_(prm["w13"])
        w2[lo:lo + n].copy_(prm["w2"])
        s13[lo:lo + n].copy_(prm["w13_scale"])
        s2[lo:lo + n].copy_(prm["w2_scale"])
        del prm
    off = ExpertStreamOffloader(E, protect_frac=0.5, fast_hit=True, no_static_full=True)
    cache = off.install_layer(w13, w2, pins=list(range(half)), prefill_resident=False,
                              device=dev, w13_scale=s13, w2_scale=s2)
    del w13, w2, s13, s2
    torch.cuda.empty_cache()
    state0, map0 = cache.state.clone(), cache.expert_map.clone()
    bpe = cfg.bytes_per_expert
    side = torch.cuda.Stream()
    g = torch.Generator().manual_seed(a.seed + 7)
    perm = torch.randperm(E, generator=g)
    reps = max(3, min(a.steps, 10))

    def restore():
        cache.state.copy_(state0)
        cache.expert_map.copy_(map0)

    for T in [int(t) for t in a.gemm_tokens.split(",")]:
        ids = synth.zipf_ids(T, k, E, gen=g, perm=perm)
        tw = torch.rand(T, k, generator=g)
        tw = (tw / tw.sum(1, keepdim=True)).float()
        x = torch.randn(T, H, generator=g).to(torch.bfloat16)
        ti, tw, x = ids.to(dev), tw.to(dev), x.to(dev)
        uniq = torch.unique(ids)
        U, Us = int(uniq.numel()), int((uniq >= half).sum())
        ws = ops.fused_experts_workspace(T, k, H, I, E, 0, dev)
        out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
        kw = dict(w1_scale=cache.w13_scale, w2_scale=cache.w2_scale)

        def overlapped():
            main = torch.cuda.current_stream()
            cache.plan(ti)
            side.wait_stream(main)
            with torch.cuda.stream(side):
                cache.stream()
            args = (x, cache.w13, cache.w2, tw, ti, cache.expert_map, cache.state)
            ops.fused_experts_phase(*args, 0, ws, out, **kw)
            main.wait_stream(side)
            ops.fused_experts_phase(*args, 1, ws, out, **kw)

        def timed(fn, pre=None):
            ts = []
            for _ in range(reps + 2):
                if pre is not None:
                    pre()
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
                e0.record()
                fn()
                e1.record()
                torch.cuda.synchronize()
                ts.append(e0.elapsed_time(e1))
            return statistics.median(ts[2:])

        t_over = timed(overlapped, restore)
        cache.check()
        # every used expert is now resident: the GEMM alone over the same pairs
        t_gemm = timed(lambda: ops.fused_experts(x, cache.w13, cache.w2, tw, ti,
                                                 expert_map=cache.expert_map, out=out, **kw))

        def plan_only():
            restore()
            cache.plan(ti)

        t_stream = timed(lambda: cache.stream(), plan_only)
        flops = T * k * cfg.flops_per_pair
        hbm = U * bpe
        host = Us * bpe
        # fp8 e4m3 x e4m3 tensor-core work: the fp8 peak measured above
        t_roof_gemm = max(hbm / (hbm_peak * 1e9), flops / (fp8_peak * 1e12)) * 1e3
        t_roof = max(t_roof_gemm, host / 63.0e9 * 1e3)
        line = {
            "metric": "grouped GEMM microbench", "workload": "fp8 grouped expert GEMM, "
            f"E={E} H={H} I={I}, 128x128 block scales, experts 0..{half - 1} resident, "
            f"{half}..{E - 1} streamed from mapped pinned host per call, top-{k} Zipf(1.1)",
            "tokens": T, "pairs": T * k, "unique_experts": U, "streamed_experts": Us,
            "dtype": "fp8 e4m3 weights (128x128 block scales), activations quantised to e4m3 "
                     "per 128-column group, fp8 tensor cores (kind::f8f6f4), fp32 accumulate",
            "gemm": {"ms": t_gemm, "tflops": flops / (t_gemm * 1e-3) / 1e12,
                     "frac_bf16_peak": flops / (t_gemm * 1e-3) / 1e12 / bf16_peak,
                     "frac_fp8_peak": flops / (t_gemm * 1e-3) / 1e12 / fp8_peak,
                     "hbm_gbs": hbm / (t_gemm * 1e-3) / 1e9,
                     "frac_hbm_peak": hbm / (t_gemm * 1e-3) / 1e9 / hbm_peak,
                     "roofline_ms": t_roof_gemm, "frac_roofline": t_roof_gemm / t_gemm},
            "stream": {"ms": t_stream, "bytes": host,
                       "gbs": host / (t_stream * 1e-3) / 1e9 if Us else None,
                       "frac_pcie_gen5_x16": host / (t_stream * 1e-3) / 1e9 / 63.0 if Us else None},
            "overlapped": {"ms": t_over, "roofline_ms": t_roof, "frac_roofline": t_roof / t_over,
                           "serial_ms": t_gemm + t_stream},
            "peaks": {"hbm_gbs": hbm_peak, "bf16_tflops": bf16_peak, "fp8_tflops": fp8_peak,
                      "fp8_source": "measured here: torch._scaled_mm 8192^3, best of 10",
                      "host_link_gbs": 63.0},
        }
        print(json.dumps(line), flush=True)


def run_prefill(a):
    """Steps beyond the envelope (prefill-sized batches of --prefill-tokens
    tokens) through the same MoE stack twice: in expert waves (the
    reference's classic-hook route for such steps) and in envelope-sized
    token chunks through the gap. One JSON line per mode: tok/s, the experts
    streamed per step and the roofline max(HBM bytes / copy peak, host bytes /
    PCIe Gen5 x16, FLOPs / bf16 peak). Fresh random tokens every step."""
    import gc

    from sluice_b200 import configs
    from sluice_b200.layer import MoEDecodeStack

    cfg = configs.CONFIGS[a.config]
    layers = a.layers or 4
    slots = _slots_for(a, cfg)
    T, K, W = a.prefill_tokens, a.steps, a.warmup
    with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
        peaks = json.load(f)
    hbm_peak, bf16_peak, host_peak = peaks["hbm_gbs"], peaks["bf16_tflops"], 63.0
    bpe, k = cfg.bytes_per_expert, cfg.routing.topk
    cpu = None
    if not a.no_cpu_baseline:
        # the CPU port (oracle routing, the classic hook's wave plan, MoE in
        # torch) on one layer of the same step size, scaled to the stack
        t_layer, n = cpu_step_time(cfg, slots, T, 1, a.seed, steps=1, warmup=1,
                                   decode=False)
        cpu = {"value": T / (t_layer * layers), "unit": "tok/s",
               "cores": torch.get_num_threads(), "kind": "port",
               "sample": f"{n} {T}-token step of 1 of the {layers} layers (after 1 warm-up), "
                         f"scaled by {layers}: torch-native routing + wave plan + MoE"}
    for mode in a.prefill_modes.split(","):
        if mode not in ("waves", "chunks"):
            raise ValueError(f"unknown prefill mode {mode!r}")
        stack = MoEDecodeStack(cfg, slots=slots, seed=a.seed, num_layers=layers)
        for layer in stack.layers:
            layer.beyond_envelope = mode
        g = torch.Generator().manual_seed(a.seed + 11)
        xs = [torch.randn(T, cfg.hidden, generator=g).to(torch.bfloat16).cuda()
              for _ in range(W + K)]
        # prefill steps: no decode rows (the working-set heuristic classifies)
        for i in range(W):
            stack.step(xs[i], decode_rows=0)
        torch.cuda.synchronize()
        s0 = stack.stats()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(torch.cuda.current_device()) as clk:
            ev0.record()
            for i in range(K):
                stack.step(xs[W + i], decode_rows=0)
            ev1.record()
            torch.cuda.synchronize()
        ms = ev0.elapsed_time(ev1) / K
        stack.check()
        s1 = stack.stats()
        # experts the last step selected, per layer (every one is read once)
        uniq = sum(int(torch.unique(layer.last_ids).numel()) for layer in stack.layers)
        # end to end: the step's tokens from pinned host memory, its output
        # read back, inside the timed region
        xh = [x.cpu().pin_memory() for x in xs[W:]]
        oh = torch.empty(T, cfg.hidden, dtype=torch.bfloat16).pin_memory()
        torch.cuda.synchronize()
        ev0.record()
        for i in range(K):
            oh.copy_(stack.step(xh[i].to("cuda", non_blocking=True), decode_rows=0),
                     non_blocking=True)
        ev1.record()
        torch.cuda.synchronize()
        e2e_ms = ev0.elapsed_time(ev1) / K
        fills = (s1["fills"] - s0["fills"]) / K
        host = fills * bpe
        hbm = uniq * bpe + layers * cfg.n_shared * bpe
        flops = layers * T * (k + cfg.n_shared) * cfg.flops_per_pair
        t_roof = max(hbm / (hbm_peak * 1e9), host / (host_peak * 1e9),
                     flops / (bf16_peak * 1e12)) * 1e3
        line = {
            "metric": "prefill MoE tok/s", "value": T / (ms * 1e-3), "unit": "tok/s",
            "mode": mode, "n_gpus": 1, "steps": K, "warmup": W, "ms_per_step": ms,
            "higher_is_better": True, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"{cfg.name} MoE stack, {layers} layers, {slots} slots "
                       f"of {cfg.num_experts} experts, {T}-token steps beyond the envelope "
                       f"({slots // k} tokens), fresh random tokens per step"},
            "experts_streamed_per_step": fills,
            "waves_per_step": (s1["waves"] - s0["waves"]) / K,
            "host_gbs": host / (ms * 1e-3) / 1e9,
            "roofline": {"ms": t_roof, "frac": t_roof / ms, "host_bytes": host,
                         "hbm_bytes": hbm, "flops": flops,
                         "peaks": {"hbm_gbs": hbm_peak, "bf16_tflops": bf16_peak,
                                   "host_link_gbs": host_peak}},
            "e2e": {"value": T / (e2e_ms * 1e-3), "unit": "tok/s",
                    "h2d_bytes_per_step": T * cfg.hidden * 2,
                    "d2h_bytes_per_step": T * cfg.hidden * 2},
            "gpu_launches": K * layers * layer_launches(cfg, T, 1, slots, decode=False)
            if mode == "waves" else None,
            "clocks": clk.summary(),
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
        del stack, xs
        gc.collect()
        torch.cuda.empty_cache()


def run_reference(a):
    """The reference's CPU path (oracle port) on the host cores, rank 0 only."""
    from sluice_b200 import configs

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    cfg = configs.CONFIGS[a.config]
    layers = a.layers or cfg.num_moe_layers
    slots = _slots_for(a, cfg)
    # the same global batch as the GPU arm: c tokens per GPU on N GPUs; the
    # port runs every expert of the model with --slots-frac of them in slots
    T = a.tokens * world
    torch.set_num_threads(os.cpu_count() or 1)
    t_step, n = _cpu_time(a, cfg, slots, T, layers, a.seed, a.steps,
                          max(1, min(a.warmup, 2)), 150.0)
    v = T / t_step
    line = {
        "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": world, "steps": n,
        "warmup": a.warmup, "ms_per_step": t_step * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "impl": "reference",
        "config": _config(a, cfg, _slots_for(a, cfg, world), a.tokens, layers, world),
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": torch.get_num_threads(),
                         "kind": "port",
                         "sample": f"{n} full decode steps ({a.workload}, {layers} MoE "
                                   f"layers, each its own weights, c={T}, {slots} of "
                                   f"{cfg.num_experts} experts in slots), median"},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main(argv=None):
    a = _args(argv)
    if a.impl == "reference":
        run_reference(a)
    elif a.workload == "grouped-gemm":
        run_grouped_gemm(a)
    elif a.workload == "prefill":
        run_prefill(a)
    else:
        run_sluice(a)   # decoder or moe-stack


if __name__ == "__main__":
    main()
