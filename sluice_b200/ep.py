"""Expert parallelism for the offloaded MoE layer (one process per GPU).

Experts are sharded in contiguous ranges, as vLLM's ``expert_map`` does for
the reference (global id -> local id, -1 on other ranks; the reference honours
it at ``offloader.py:974-986`` and skips non-owned ids in the gap,
``2432-2435``). Every rank keeps its own host shard, slot cache and device
planner. One decode step of a layer:

1. route the rank's own tokens (gate + select_experts, replicated gate);
2. dispatch: each token travels only to the ranks owning one of its top-k
   experts (``NvlinkExchange``: one routed push kernel over NVLink peer
   memory); every rank ends up with its own tokens first, then the tokens its
   peers sent it;
3. gap on the **post-dispatch** ids (the lesson of ``offloader.py:1192-1201``):
   the planner sees every received id and plans only the ones this rank owns;
4. ``fused_experts_partial`` over the received rows: this rank's experts
   (fp32, scaled), plus the shared experts on this rank's own token rows;
5. combine: each received row's fp32 partial goes back to its home rank,
   which sums its own and its peers' partials per token and rounds once to
   bf16.

``exchange="nccl"`` keeps the collective form for comparison: an NCCL
all-gather of every rank's rows (every rank receives every token) and a
reduce-scatter of the partials.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import ops
from .layer import StreamTimer, _timed, expert_waves
from .configs import MoEConfig


def expert_shard(num_experts: int, world: int, rank: int):
    """(first global id, local count, local_of[global]) of a contiguous shard."""
    if num_experts % world:
        raise ValueError(f"{num_experts} experts do not split over {world} ranks")
    per = num_experts // world
    lo = rank * per
    local_of = [g - lo if lo <= g < lo + per else -1 for g in range(num_experts)]
    return lo, per, local_of


def pack_routing(x: torch.Tensor, tw: torch.Tensor, ti: torch.Tensor) -> torch.Tensor:
    """One byte row per token: [hidden bf16 | topk weights f32 | topk ids i32]."""
    T = x.shape[0]
    return torch.cat([x.contiguous().view(torch.uint8).view(T, -1),
                      tw.contiguous().view(torch.uint8).view(T, -1),
                      ti.contiguous().view(torch.uint8).view(T, -1)], dim=1)


def unpack_routing(buf: torch.Tensor, H: int, k: int):
    n = buf.shape[0]
    xb = 2 * H
    x = buf[:, :xb].contiguous().view(torch.bfloat16).view(n, H)
    tw = buf[:, xb:xb + 4 * k].contiguous().view(torch.float32).view(n, k)
    ti = buf[:, xb + 4 * k:].contiguous().view(torch.int32).view(n, k)
    return x, tw, ti


def dispatch(x, tw, ti, group=None):
    """All-gather of every rank's tokens and routing: ([N*T,H], [N*T,k], [N*T,k])."""
    world = dist.get_world_size(group)
    packed = pack_routing(x, tw, ti)
    out = torch.empty((world * packed.shape[0], packed.shape[1]), dtype=torch.uint8,
                      device=packed.device)
    dist.all_gather_into_tensor(out, packed, group=group)
    return unpack_routing(out, x.shape[1], tw.shape[1])


def combine(partial: torch.Tensor, group=None) -> torch.Tensor:
    """Sum of every rank's fp32 partial rows for this rank's tokens."""
    world = dist.get_world_size(group)
    out = torch.empty((partial.shape[0] // world, partial.shape[1]), dtype=partial.dtype,
                      device=partial.device)
    dist.reduce_scatter_tensor(out, partial, group=group)
    return out


class NvlinkExchange:
    """Dispatch / combine kernels over NVLink peer memory (``sl_ep_dispatch``,
    ``sl_ep_combine``). One symmetric allocation per rank
    (``torch.distributed._symmetric_memory``), mapped into every peer:
    [dispatch receive halves | combine receive halves | 16 signal words],
    sized for ``max_tokens`` tokens per rank per call."""

    SIGNAL_BYTES = 256

    def __init__(self, max_tokens: int, hidden: int, topk: int, group=None, device="cuda"):
        import ctypes

        import torch.distributed._symmetric_memory as symm_mem

        from . import _lib

        self.group = group
        self.max_tokens = max_tokens
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        L = _lib.lib()
        nd = L.sl_ep_dispatch_recv_bytes(self.world, max_tokens, hidden, topk)
        nc = L.sl_ep_combine_recv_bytes(self.world, max_tokens, hidden)
        nd = (nd + 255) // 256 * 256
        nc = (nc + 255) // 256 * 256
        self.buf = symm_mem.empty(nd + nc + self.SIGNAL_BYTES, dtype=torch.uint8, device=device)
        self.buf[nd + nc:].zero_()
        grp = group if group is not None else dist.group.WORLD
        self.handle = symm_mem.rendezvous(self.buf, grp)
        ptrs = list(self.handle.buffer_ptrs)
        vp = ctypes.c_void_p * self.world
        self._recv_d = vp(*ptrs)
        self._recv_c = vp(*[p + nd for p in ptrs])
        self._sig = vp(*[p + nd + nc for p in ptrs])
        self.book = torch.zeros(4, dtype=torch.int32, device=device)
        self.status = torch.zeros(1, dtype=torch.int32, device=device)
        torch.cuda.synchronize(device)
        dist.barrier(group)  # every rank's signal words are zero before any peer signals

    def dispatch(self, x, tw, ti, global_n: int):
        """Routed dispatch of this rank's tokens: returns ``(xg, twg, tig,
        src)`` over ``world * T`` rows — this rank's tokens first, then the
        rows peers sent (rank order), then empty rows (id -1, weight 0);
        ``src`` [world * T] int32 is ``(home rank << 16) | token`` (-1 empty)."""
        from ._lib import check, lib, ptr

        T, H = x.shape
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens exceed the exchange's {self.max_tokens}")
        k = tw.shape[1]
        x = x.contiguous()
        tw = tw.contiguous().float()
        ti = ti.contiguous().to(torch.int32)
        n = self.world * T
        xg = torch.empty(n, H, dtype=torch.bfloat16, device=x.device)
        twg = torch.empty(n, k, dtype=torch.float32, device=x.device)
        tig = torch.empty(n, k, dtype=torch.int32, device=x.device)
        src = torch.empty(n, dtype=torch.int32, device=x.device)
        # the kernel packs (hidden | weights | ids | token) rows while pushing
        check(lib().sl_ep_dispatch(ptr(x), ptr(tw), ptr(ti), T, H, k, int(global_n), self.rank,
                                   self.world, self._recv_d, self._sig, ptr(self.book),
                                   ptr(xg), ptr(twg), ptr(tig), ptr(src), ptr(self.status),
                                   torch.cuda.current_stream().cuda_stream), "sl_ep_dispatch")
        return xg, twg, tig, src

    def combine(self, partial: torch.Tensor, src: torch.Tensor, ti: torch.Tensor,
                global_n: int, residual: torch.Tensor | None = None) -> torch.Tensor:
        """This rank's tokens' summed partials in bf16 (``partial`` and
        ``src`` as the dispatch produced them, ``ti`` this rank's own top-k
        ids); with ``residual`` (bf16 [T, H]) the result is ``residual +
        that``, as a bf16 add."""
        from ._lib import check, lib, ptr

        n, H = partial.shape
        T = n // self.world
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens exceed the exchange's {self.max_tokens}")
        out = torch.empty(T, H, dtype=torch.bfloat16, device=partial.device)
        if residual is not None:
            residual = residual.contiguous()
        ti = ti.contiguous().to(torch.int32)
        check(lib().sl_ep_combine(ptr(partial), ptr(src), ptr(ti), T, H, ti.shape[1],
                                  int(global_n), self.rank, self.world, self._recv_c, self._sig,
                                  ptr(self.book), ptr(residual), ptr(out), ptr(self.status),
                                  torch.cuda.current_stream().cuda_stream), "sl_ep_combine")
        return out

    def check(self) -> None:
        from . import _lib

        st = int(self.status.item())
        if st != _lib.SL_OK:
            raise _lib.SluiceError("expert-parallel exchange", st)


class EPMoELayer:
    """One MoE layer's expert-parallel step on this rank."""

    def __init__(self, cfg: MoEConfig, router: ops.Router, cache, shared_w13, shared_w2,
                 group=None, shared_w13_scale=None, shared_w2_scale=None,
                 exchange: "NvlinkExchange | None" = None, overlap: bool = True,
                 stream_ctas: int = 16, beyond_envelope: str = "waves"):
        if beyond_envelope not in ("waves", "chunks"):
            raise ValueError("beyond_envelope is 'waves' or 'chunks'")
        self.cfg = cfg
        # steps whose gathered rows exceed the envelope: expert waves over
        # the gathered rows, or envelope-sized token chunks through the gap
        self.beyond_envelope = beyond_envelope
        self.exchange = exchange  # None: NCCL all-gather / reduce-scatter
        self.shared_w13_scale = shared_w13_scale
        self.shared_w2_scale = shared_w2_scale
        self.router = router
        self.cache = cache
        self.shared_w13 = shared_w13
        self.shared_w2 = shared_w2
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.last_ids = None
        # overlap the gap's expert stream with the resident experts' GEMMs
        self.overlap = overlap and not cache.static_full
        self.stream_ctas = stream_ctas
        self._side = torch.cuda.Stream(device=cache.device) \
            if not cache.static_full else None
        # set to a StreamTimer to time every expert-stream launch
        self.stream_timer: StreamTimer | None = None

    @property
    def envelope(self) -> int:
        """This rank's tokens per single-wave step: the gap plans over every
        rank's gathered tokens, so the reference's ``slots // topk`` envelope
        (``offloader.py:816-842``) is split across the world; a fully
        resident shard has none."""
        if self.cache.static_full:
            return 1 << 30
        return max(1, self.cache.num_slots // self.cfg.routing.topk // self.world)

    def forward(self, x: torch.Tensor, add_residual: bool = False,
                decode: bool = True) -> torch.Tensor:
        """This rank's MoE output for its tokens ``x``; ``add_residual``
        returns ``x + output`` (the decoder's residual add; folded into the
        combine kernel under the NVLink exchange). Every rank steps the same
        token count. A step whose rows exceed the envelope runs in expert
        waves over the gathered rows (decode steps decode-class; ``decode=False``
        plans a scan, as the reference's data-parallel mode classifies every
        step it plans in its hook); it is split only where it exceeds the
        exchange's capacity. With ``beyond_envelope="chunks"`` such steps run
        as envelope-sized chunks through the gap instead."""
        thr = self.envelope
        if self.stream_timer is not None:
            self.stream_timer.reset()
        if self.beyond_envelope == "chunks" or self.cache.static_full:
            if x.shape[0] > thr:
                return torch.cat([self._forward_step(c, add_residual, decode)
                                  for c in x.split(thr)])
            return self._forward_step(x, add_residual, decode)
        cap = self.exchange.max_tokens if self.exchange is not None else x.shape[0]
        if x.shape[0] > cap:
            return torch.cat([self._forward_step(c, add_residual, decode)
                              for c in x.split(cap)])
        return self._forward_step(x, add_residual, decode)

    def _forward_step(self, x: torch.Tensor, add_residual: bool,
                      decode: bool = True) -> torch.Tensor:
        T = x.shape[0]
        G = self.cfg.num_experts
        tw, ti, _ = self.router.route(x)
        if self.exchange is not None:
            # routed: this rank's own tokens are rows [0, T)
            xg, twg, tig, src = self.exchange.dispatch(x, tw, ti, G)
            own0 = 0
        else:
            # all-gather: rank r's tokens are rows [r*T, (r+1)*T)
            xg, twg, tig = dispatch(x, tw, ti, self.group)
            own0 = self.rank * T
        self.last_ids = tig
        c = self.cache
        kw = dict(shared_t0=own0, shared_nt=T,
                  routed_scaling_factor=self.cfg.routed_scaling_factor, w1_scale=c.w13_scale,
                  w2_scale=c.w2_scale, shared_w13_scale=self.shared_w13_scale,
                  shared_w2_scale=self.shared_w2_scale)
        args = (xg, c.w13, c.w2, twg, tig, c.expert_map, self.shared_w13, self.shared_w2)
        if T > self.envelope:
            # the gathered rows' working set can exceed the slots: waves
            part = expert_waves(c, self._side, xg, twg, tig, tig.shape[0] if decode else -1,
                                self.shared_w13, self.shared_w2, own0, T,
                                self.cfg.routed_scaling_factor, self.shared_w13_scale,
                                self.shared_w2_scale, self.stream_ctas, self.stream_timer)
        elif self.overlap:
            # plan -> grouping -> [stream, then the streamed experts, on a side
            # stream || resident experts] -> combine
            from ._lib import (PHASE_COMBINE, PHASE_GROUP, PHASE_RESIDENT_GEMMS,
                               PHASE_STREAMED_GEMMS)
            main = torch.cuda.current_stream()
            c.plan(tig)
            self._side.wait_stream(main)
            with torch.cuda.stream(self._side):
                _timed(self.stream_timer, self._side, lambda: c.stream(self.stream_ctas))
            n_sh = 0 if self.shared_w13 is None else self.shared_w13.shape[0]
            ws = ops.fused_experts_workspace(xg.shape[0], tig.shape[1], xg.shape[1],
                                             c.w13.shape[1] // 2, c.num_slots, n_sh, xg.device)
            part = torch.empty(xg.shape, dtype=torch.float32, device=xg.device)

            def run(phase):
                ops.fused_experts_partial(*args, out=part, slot_state=c.state, phase=phase,
                                          workspace=ws, **kw)
            run(PHASE_GROUP)
            grouped = torch.cuda.Event()
            grouped.record(main)
            with torch.cuda.stream(self._side):
                self._side.wait_event(grouped)
                run(PHASE_STREAMED_GEMMS)
            run(PHASE_RESIDENT_GEMMS)
            main.wait_stream(self._side)
            run(PHASE_COMBINE)
        else:
            c.gap(tig)
            part = ops.fused_experts_partial(*args, **kw)
        if self.exchange is not None:
            return self.exchange.combine(part, src, ti, G, x if add_residual else None)
        out = combine(part, self.group).to(torch.bfloat16)
        return x + out if add_residual else out

    __call__ = forward


class EPDecodeStack:
    """The MoE layers of a decoder under expert parallelism on this rank."""

    def __init__(self, cfg: MoEConfig, slots: int, seed: int = 0, device="cuda",
                 num_layers: int | None = None, group=None, protect_frac=None,
                 exchange: str = "nvlink", max_tokens: int = 16, overlap: bool = True):
        from . import synth
        from .offloader import ExpertStreamOffloader

        self.cfg = cfg
        self.device = torch.device(device)
        self.group = group
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        lo, per, local_of = expert_shard(cfg.num_experts, world, rank)
        self.offloader = ExpertStreamOffloader(slots, protect_frac=protect_frac, fast_hit=True)
        self.exchange = (NvlinkExchange(max_tokens, cfg.hidden, cfg.routing.topk, group,
                                        self.device) if exchange == "nvlink" else None)
        self.layers: list[EPMoELayer] = []
        n = cfg.num_moe_layers if num_layers is None else num_layers
        for li in range(n):
            prm = synth.layer_params(cfg, li, seed, device=self.device, num_experts=per,
                                     expert_lo=lo)
            cache = self.offloader.install_layer(prm["w13"], prm["w2"], global_n=cfg.num_experts,
                                                 local_of=local_of, device=self.device,
                                                 w13_scale=prm.get("w13_scale"),
                                                 w2_scale=prm.get("w2_scale"))
            del prm
            gw, lb, sb = synth.gate_params(cfg, li, seed, device=self.device)
            sh = synth.shared_params(cfg, li, seed, device=self.device)
            self.layers.append(EPMoELayer(cfg, ops.Router(cfg.routing, gw, lb, sb), cache,
                                          sh.get("shared_w13"), sh.get("shared_w2"), group,
                                          sh.get("shared_w13_scale"),
                                          sh.get("shared_w2_scale"), self.exchange,
                                          overlap=overlap))
        torch.cuda.synchronize(self.device)
        dist.barrier(group)  # ranks enter the first exchange together (peer waits are bounded)
        self.graph = None
        self._static_in = None
        self._static_out = None

    def step(self, x: torch.Tensor) -> torch.Tensor:
        h = x
        for layer in self.layers:
            h = layer(h, add_residual=True)  # h + moe(h)
        return h

    def capture(self, tokens: int) -> bool:
        """Capture one step (NCCL collectives included) in a CUDA graph;
        returns False (eager replay) if this stack cannot be captured."""
        self._static_in = torch.zeros(tokens, self.cfg.hidden, dtype=torch.bfloat16,
                                      device=self.device)
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            self.step(self._static_in)
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)
        try:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self._static_out = self.step(self._static_in)
            self.graph = g
            return True
        except Exception:
            self.graph = None
            torch.cuda.synchronize(self.device)
            return False

    def replay(self, x: torch.Tensor | None = None) -> torch.Tensor:
        if x is not None:
            self._static_in.copy_(x, non_blocking=True)
        if self.graph is None:
            self._static_out = self.step(self._static_in)
        else:
            self.graph.replay()
        return self._static_out

    def decode_step(self, x_host: torch.Tensor, out_host: torch.Tensor) -> torch.Tensor:
        self.replay(x_host.to(self.device, non_blocking=True))
        out_host.copy_(self._static_out, non_blocking=True)
        return out_host

    def release(self) -> None:
        """Drop the captured graph (it holds NCCL work) before process-group teardown."""
        self.graph = None

    def check(self) -> None:
        for layer in self.layers:
            layer.cache.check()
        if self.exchange is not None:
            self.exchange.check()

    def stats(self) -> dict:
        tot = {}
        for layer in self.layers:
            for k, v in layer.cache.stats().items():
                if isinstance(v, bool):
                    continue
                tot[k] = tot.get(k, 0) + v
        return tot
