"""One MoE layer on the router-split path, and a decode stack of such layers.

``SluiceMoELayer.forward`` is the router-split entry of the reference
(``offloader.py:2578-2603``) plus vLLM's runner tail
(``runner/moe_runner.py:663-680``), with every box on sm_100a kernels:

    gate + select_experts      -> sl_route        (router kernels)
    sluice_stream_gap          -> SlotCache.gap   (planner + streamer, no sync)
    fused_experts + shared MLP -> sl_fused_experts (tcgen05 GEMMs + combine)
      + routed scaling + add

Steps beyond the envelope (``slots // topk`` tokens: prefills, mixed
batches) take the route the reference gives them under router-split, its
classic hook (``run_moe`` 1452-1764 and ``_run_waves`` 1846-1933): the
device plans expert waves, and each wave's fills stream on a side stream
while the previous wave computes; the waves' fp32 outputs add up to the step.

``MoEDecodeStack`` chains layers with a residual (``h = h + moe(h)``) to run
the decode step of a MoE decoder's expert layers over the slot caches; the
step is capturable in one CUDA graph because no kernel waits on the host.
"""

from __future__ import annotations

import torch

from . import ops, synth
from .configs import MoEConfig
from .offloader import ExpertStreamOffloader, SlotCache


def decode_rows_from_query_start_loc(query_start_loc, num_tokens: int, max_query_len: int,
                                     num_actual_tokens: int | None = None):
    """The decode rows of a batch from a non-MLA attention backend's metadata
    (the reference's opt-in ``_non_mla_decode_rows``, offloader.py:1802-1844):
    a request whose query is one token is a decode, and its row is its query
    start. Returns the row indices (every row when ``max_query_len`` is 1, an
    empty tensor for a pure prefill), or None when the metadata does not
    describe this batch (the caller then passes 0: the working-set heuristic).
    Pass the result as ``decode_rows``."""
    if query_start_loc is None or max_query_len is None:
        return None
    if num_actual_tokens is not None and int(num_actual_tokens) != num_tokens:
        return None
    if int(max_query_len) == 1:
        return torch.arange(num_tokens)
    qsl = torch.as_tensor(query_start_loc).cpu()
    if qsl.ndim != 1 or qsl.numel() < 2 or int(qsl[-1]) != num_tokens:
        return None
    starts = qsl[:-1]
    return starts[(qsl[1:] - starts) == 1].long()


class StreamTimer:
    """Optional CUDA-event timing of a layer's expert-stream launches.

    Each launch is bracketed by two timing events recorded on the stream the
    streamer runs on; the events are external, so inside a CUDA-graph capture
    they become event-record nodes that every replay rewrites. ``launches()``
    (after the step has completed) gives each launch's device time with its
    wave (-1 for a gap's single stream) and, for a prefetch launch, the cache
    it filled."""

    def __init__(self):
        self.pairs: list = []

    def reset(self) -> None:
        self.pairs = []

    def around(self, stream: torch.cuda.Stream, fn, wave: int = -1, other=None) -> None:
        a = torch.cuda.Event(enable_timing=True, external=True)
        b = torch.cuda.Event(enable_timing=True, external=True)
        a.record(stream)
        fn()
        b.record(stream)
        self.pairs.append((a, b, wave, other))

    def launches(self) -> list[tuple[float, int, object]]:
        """(ms, wave, other cache) per launch; ``other`` is the cache a
        prefetch launch filled (the next layer's), else None."""
        return [(a.elapsed_time(b), w, o) for a, b, w, o in self.pairs]


def _timed(timer: "StreamTimer | None", stream: torch.cuda.Stream, fn, wave: int = -1,
           other=None) -> None:
    if timer is None:
        fn()
    else:
        timer.around(stream, fn, wave, other)


def expert_waves(c: SlotCache, side: torch.cuda.Stream, hs: torch.Tensor, tw: torch.Tensor,
                 ti: torch.Tensor, decode_rows, shared_w13, shared_w2, shared_t0: int,
                 shared_nt: int, scale: float, shared_w13_scale=None, shared_w2_scale=None,
                 stream_ctas: int = 16, timer: StreamTimer | None = None) -> torch.Tensor:
    """One step of ``hs`` [T, H] (routed as ``tw`` / ``ti``) in expert waves
    over the cache ``c``; returns the fp32 output [T, H]: the routed experts
    scaled by ``scale`` plus the shared experts on rows [shared_t0, shared_t0
    + shared_nt).

    plan waves -> wave 0 (resident experts || its fills, then the filled
    ones and the shared experts) -> waves 1.. (each after its fills, which
    stream on ``side`` while the previous wave computes). A fixed number of
    waves is issued for the step's size (``c.waves_for``; waves past the
    plan's count do no work), so the step captures in a CUDA graph.
    """
    main = torch.cuda.current_stream()
    T, H = hs.shape
    c.plan_waves(ti, decode_rows)
    n_sh = 0 if shared_w13 is None else shared_w13.shape[0]
    ws = ops.fused_experts_workspace(T, ti.shape[1], H, c.w13.shape[1] // 2, c.num_slots,
                                     n_sh, hs.device)
    acc = torch.empty(T, H, dtype=torch.float32, device=hs.device)
    # every row a decode: every expert decode-class (a tighter wave count);
    # the planner reads a count above T as no per-token signal
    all_decode = isinstance(decode_rows, int) and decode_rows == T
    MW = c.waves_for(ti.numel(), all_decode)
    filled = [torch.cuda.Event() for _ in range(MW)]
    computed = [torch.cuda.Event() for _ in range(MW)]

    def stream(k: int) -> None:
        with torch.cuda.stream(side):
            _timed(timer, side, lambda: c.stream_wave(k, stream_ctas), k)
            filled[k].record(side)

    side.wait_stream(main)
    stream(0)
    args = (hs, c.w13, c.w2, tw, ti, c.wave_map(0))
    kw = dict(shared_w13=shared_w13, shared_w2=shared_w2, shared_t0=shared_t0,
              shared_nt=shared_nt, routed_scaling_factor=scale, out=acc, w1_scale=c.w13_scale,
              w2_scale=c.w2_scale, shared_w13_scale=shared_w13_scale,
              shared_w2_scale=shared_w2_scale, slot_state=c.state, workspace=ws)
    ops.fused_experts_partial(*args, phase=0, **kw)
    main.wait_event(filled[0])
    ops.fused_experts_partial(*args, phase=1, **kw)
    computed[0].record(main)
    # wave k refills the slots wave k - 2 read (ping-pong) or, with a single
    # rotation group, wave k - 1's; waves 1 and 2 follow wave 0
    lag = 2 if c.waves_pingpong else 1
    for k in range(1, min(1 + lag, MW)):
        side.wait_event(computed[0])
        stream(k)
    for k in range(1, MW):
        main.wait_event(filled[k])
        ops.fused_experts_accumulate(hs, c.w13, c.w2, tw, ti, c.wave_map(k), acc, ws,
                                     routed_scaling_factor=scale, w1_scale=c.w13_scale,
                                     w2_scale=c.w2_scale)
        computed[k].record(main)
        if k + lag < MW:
            side.wait_event(computed[k])
            stream(k + lag)
    main.wait_stream(side)
    return acc


class SluiceMoELayer:
    def __init__(self, cfg: MoEConfig, router: ops.Router, cache: SlotCache,
                 shared_w13: torch.Tensor | None, shared_w2: torch.Tensor | None,
                 layer_idx: int = 0, overlap: bool = True, stream_ctas: int = 16,
                 shared_w13_scale: torch.Tensor | None = None,
                 shared_w2_scale: torch.Tensor | None = None,
                 beyond_envelope: str = "waves"):
        if beyond_envelope not in ("waves", "chunks"):
            raise ValueError("beyond_envelope is 'waves' or 'chunks'")
        self.cfg = cfg
        # steps larger than the envelope: expert waves (the reference's
        # classic hook), or envelope-sized token chunks through the gap
        self.beyond_envelope = beyond_envelope
        self.shared_w13_scale = shared_w13_scale
        self.shared_w2_scale = shared_w2_scale
        # overlap the gap's expert stream with the resident experts' GEMMs
        self.overlap = overlap and not cache.static_full
        self.stream_ctas = stream_ctas
        self._side = torch.cuda.Stream(device=cache.device) \
            if not cache.static_full else None
        self.router = router
        self.cache = cache
        self.shared_w13 = shared_w13
        self.shared_w2 = shared_w2
        self.layer_idx = layer_idx
        self.last_ids = None
        self.last_logits = None
        # set to a StreamTimer to time every expert-stream launch
        self.stream_timer: StreamTimer | None = None
        # opt-in cross-layer prefetch: the next layer (whose experts this
        # layer predicts and streams after its own stream) and the event the
        # next layer's planner waits for
        self.prefetch_next: "SluiceMoELayer | None" = None
        self.prefetch_max_fills = 0
        self._prefetched: torch.cuda.Event | None = None
        self._prefetch_input: torch.Tensor | None = None

    @property
    def envelope(self) -> int:
        """Tokens per single-wave step: ``slots // topk`` (the reference's
        router-split batch envelope, ``offloader.py:816-842``); a fully
        resident layer has none."""
        if self.cache.static_full:
            return 1 << 30
        return max(1, self.cache.num_slots // self.cfg.routing.topk)

    def forward(self, hs: torch.Tensor, decode_rows=0) -> torch.Tensor:
        """One step of ``hs`` [T, H]. ``decode_rows`` only matters beyond the
        envelope: rows [0, decode_rows) are single-token decodes (the
        reference's ``num_decode_tokens``, decode rows first), 0 leaves the
        step's class to the working-set heuristic, < 0 makes it a scan; or
        the indices of the decode rows wherever they sit (the opt-in non-MLA
        classifier's signal, ``decode_rows_from_query_start_loc``)."""
        thr = self.envelope
        if self.stream_timer is not None:
            self.stream_timer.reset()
        if hs.shape[0] > thr:
            if self.beyond_envelope == "waves":
                return self._forward_waves(hs, decode_rows)
            # consecutive envelope-sized chunks, as the reference's piecewise
            # mode requires of the batch (max_num_batched_tokens = slots //
            # topk): every chunk is a single-wave gap plus fused experts
            outs, ids, logits = [], [], []
            for c in hs.split(thr):
                outs.append(self._forward_step(c))
                ids.append(self.last_ids)
                logits.append(self.last_logits)
            self.last_ids, self.last_logits = torch.cat(ids), torch.cat(logits)
            return torch.cat(outs)
        return self._forward_step(hs)

    def _await_prefetch(self) -> None:
        """Order this layer's planner (and everything after it) after the
        previous layer's prefetch into this cache, which wrote its state,
        fill list and slots; the router runs before, unordered."""
        if self._prefetched is not None:
            torch.cuda.current_stream().wait_event(self._prefetched)
            self._prefetched = None
            self._prefetch_input = None

    def _forward_waves(self, hs: torch.Tensor, decode_rows) -> torch.Tensor:
        hs = hs.contiguous()
        tw, ti, logits = self.router.route(hs)
        self.last_ids, self.last_logits = ti, logits
        self._await_prefetch()
        acc = expert_waves(self.cache, self._side, hs, tw, ti, decode_rows,
                           self.shared_w13, self.shared_w2, 0, hs.shape[0],
                           self.cfg.routed_scaling_factor, self.shared_w13_scale,
                           self.shared_w2_scale, self.stream_ctas, self.stream_timer)
        return acc.to(torch.bfloat16)

    def _forward_step(self, hs: torch.Tensor) -> torch.Tensor:
        tw, ti, logits = self.router.route(hs)
        self.last_ids, self.last_logits = ti, logits
        self._await_prefetch()
        if self.overlap:
            return self._forward_overlapped(hs, tw, ti)
        self.cache.gap(ti)
        c = self.cache
        return ops.fused_experts(hs, c.w13, c.w2, tw, ti,
                                 global_num_experts=self.cfg.num_experts,
                                 expert_map=c.expert_map, w1_scale=c.w13_scale,
                                 w2_scale=c.w2_scale, shared_w13=self.shared_w13,
                                 shared_w2=self.shared_w2,
                                 shared_w13_scale=self.shared_w13_scale,
                                 shared_w2_scale=self.shared_w2_scale,
                                 routed_scaling_factor=self.cfg.routed_scaling_factor)

    def _forward_overlapped(self, hs, tw, ti):
        """plan -> grouping -> [stream, then the streamed experts' GEMMs, on a
        side stream || resident experts' GEMMs] -> combine. A layer without
        misses thus puts no launch between its resident GEMMs and its
        combine. With prefetch on, the side stream then plans and streams the
        next layer's predicted experts (its router on this layer's input)
        while this layer finishes."""
        from ._lib import (PHASE_COMBINE, PHASE_GROUP, PHASE_RESIDENT_GEMMS,
                           PHASE_STREAMED_GEMMS)
        c, cfg = self.cache, self.cfg
        main = torch.cuda.current_stream()
        hs = hs.contiguous()
        c.plan(ti)
        self._side.wait_stream(main)
        T, H = hs.shape
        ws = ops.fused_experts_workspace(T, ti.shape[1], H, c.w13.shape[1] // 2,
                                         c.num_slots, 0 if self.shared_w13 is None
                                         else self.shared_w13.shape[0], hs.device)
        out = torch.empty_like(hs)
        args = (hs, c.w13, c.w2, tw, ti, c.expert_map, c.state)
        kw = dict(w1_scale=c.w13_scale, w2_scale=c.w2_scale, shared_w13=self.shared_w13,
                  shared_w2=self.shared_w2, shared_w13_scale=self.shared_w13_scale,
                  shared_w2_scale=self.shared_w2_scale,
                  routed_scaling_factor=cfg.routed_scaling_factor)
        with torch.cuda.stream(self._side):
            _timed(self.stream_timer, self._side, lambda: c.stream(self.stream_ctas))
        ops.fused_experts_phase(*args, PHASE_GROUP, ws, out, **kw)
        grouped = torch.cuda.Event()
        grouped.record(main)
        streamed = torch.cuda.Event()
        nxt = self.prefetch_next
        prefetch = (nxt is not None and not nxt.cache.static_full and
                    self.prefetch_max_fills > 0)
        with torch.cuda.stream(self._side):
            self._side.wait_event(grouped)
            ops.fused_experts_phase(*args, PHASE_STREAMED_GEMMS, ws, out, **kw)
            streamed.record(self._side)
            if prefetch:
                # on the copy stream, after this layer's own stream and its
                # streamed experts' GEMMs: predict the next layer's experts (its
                # router on this layer's input), plan and stream them; the next
                # layer plans after this
                _, ti_next, _ = nxt.router.route(hs)
                nc = nxt.cache
                nc.prefetch(ti_next, self.prefetch_max_fills)
                _timed(self.stream_timer, self._side, lambda: nc.stream(self.stream_ctas),
                       other=nc)
                done = torch.cuda.Event()
                done.record(self._side)
                nxt._prefetched = done
                # the copy stream reads hs: keep it alive until the next layer
                # has ordered its stream after that read
                nxt._prefetch_input = hs
        ops.fused_experts_phase(*args, PHASE_RESIDENT_GEMMS, ws, out, **kw)
        main.wait_event(streamed)
        return ops.fused_experts_phase(*args, PHASE_COMBINE, ws, out, **kw)

    __call__ = forward


class MoEDecodeStack:
    """The MoE layers of a decoder, each behind its own slot cache."""

    def __init__(self, cfg: MoEConfig, slots: int, seed: int = 0, device="cuda",
                 protect_frac: float | None = None, fast_hit: bool = True,
                 num_layers: int | None = None, overlap: bool = True, prefetch: int = 0):
        """``prefetch`` > 0 turns on the opt-in cross-layer prefetch: each
        offloaded layer predicts the next layer's experts (the next router on
        its own input) and streams up to ``prefetch`` of them into free or
        probation slots after its own stream (``SlotCache.prefetch``). Off by
        default: the slot maps then follow the reference's policy exactly."""
        self.cfg = cfg
        self.device = torch.device(device)
        self.offloader = ExpertStreamOffloader(slots, protect_frac=protect_frac,
                                               fast_hit=fast_hit)
        self.layers: list[SluiceMoELayer] = []
        n = cfg.num_moe_layers if num_layers is None else num_layers
        for li in range(n):
            prm = synth.layer_params(cfg, li, seed, device=self.device)
            cache = self.offloader.install_layer(prm["w13"], prm["w2"], device=self.device,
                                                 w13_scale=prm.get("w13_scale"),
                                                 w2_scale=prm.get("w2_scale"))
            del prm
            gw, lb, sb = synth.gate_params(cfg, li, seed, device=self.device)
            router = ops.Router(cfg.routing, gw, lb, sb)
            sh = synth.shared_params(cfg, li, seed, device=self.device)
            self.layers.append(SluiceMoELayer(
                cfg, router, cache, sh.get("shared_w13"), sh.get("shared_w2"), li,
                overlap=overlap, shared_w13_scale=sh.get("shared_w13_scale"),
                shared_w2_scale=sh.get("shared_w2_scale")))
        if prefetch > 0 and overlap:
            for cur, nxt in zip(self.layers, self.layers[1:]):
                cur.prefetch_next = nxt
                cur.prefetch_max_fills = int(prefetch)
        torch.cuda.synchronize(self.device)
        self.graphs: dict = {}  # tokens -> (graph, static input, static output)

    def step(self, x: torch.Tensor, decode_rows=None) -> torch.Tensor:
        """One step through every layer. By default a decode step: every row
        is a decode (decode-class experts when the step exceeds the envelope
        and runs in waves); ``decode_rows`` as ``SluiceMoELayer.forward``
        otherwise (0 for a prefill: the working-set heuristic)."""
        d = x.shape[0] if decode_rows is None else decode_rows
        h = x
        for layer in self.layers:
            h = h + layer(h, decode_rows=d)
        return h

    # -- CUDA graphs of one decode step (one per token count) -----------------
    def capture(self, tokens: int) -> None:
        static_in = torch.zeros(tokens, self.cfg.hidden, dtype=torch.bfloat16,
                                device=self.device)
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            self.step(static_in)  # allocator warm-up outside capture
        torch.cuda.current_stream(self.device).wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            static_out = self.step(static_in)
        self.graphs[tokens] = (g, static_in, static_out)

    @property
    def graph(self):
        return next(iter(self.graphs.values()))[0] if self.graphs else None

    def replay(self, x: torch.Tensor) -> torch.Tensor:
        g, static_in, static_out = self.graphs[x.shape[0]]
        static_in.copy_(x, non_blocking=True)
        g.replay()
        return static_out

    def decode_step(self, x_host: torch.Tensor, out_host: torch.Tensor) -> torch.Tensor:
        """Public end-to-end call: host tokens in, host hidden states out."""
        out_host.copy_(self.replay(x_host), non_blocking=True)
        return out_host

    def check(self) -> None:
        for layer in self.layers:
            layer.cache.check()

    def stats(self) -> dict:
        tot = {}
        for layer in self.layers:
            for k, v in layer.cache.stats().items():
                if isinstance(v, bool):
                    continue
                tot[k] = tot.get(k, 0) + v
        return tot
