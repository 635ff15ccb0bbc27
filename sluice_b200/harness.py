"""A DeepSeek-V2-Lite-shaped decoder around the offloaded MoE layers.

The reference's headline numbers are whole-model decode tok/s inside vLLM;
this harness gives the MoE hot path the same surroundings at the shapes the
workload names (random-init bf16, no checkpoint): token embedding, 27
decoder layers of [RMSNorm -> multi-head latent attention -> residual ->
RMSNorm -> FFN -> residual] with a dense SwiGLU FFN in layer 0 and an MoE
layer elsewhere, final RMSNorm, the vocabulary head and greedy sampling.

The MoE layers are this package's hot path (``SluiceMoELayer``: router,
device slot planner, expert streamer, tcgen05 fused experts). Around them,
on a CUDA device, the attention core, each residual add + RMSNorm and (for
one or two sequences) the projections are also this package's kernels
(``sl_mla_decode``, ``sl_add_rmsnorm``, ``sl_linear_small``); the rest is
PyTorch (cuBLAS GEMMs): it is the harness around the hot path, not part of
it. The same module runs on the host for the CPU baseline, with PyTorch ops
throughout and the MoE layers replaced by the oracle's torch-native MoE and
slot policy.

Attention is decode-only MLA in its absorbed form over a compressed cache
(kv_lora_rank 512 latent + 64 rotary dims per token and layer): per token
``q`` (16 heads x (128 nope + 64 rope)), the latent ``c_kv`` (RMSNormed) and
``k_pe`` (rotary) are written at the sequence's position; scores are
``q_nope W_uk . c_kv + q_pe . k_pe`` over every cached position (fixed
shapes, masked beyond the sequence's length, so a step captures in one CUDA
graph); the output is ``softmax . c_kv`` projected through ``W_uv`` and the
output projection. Prompt tokens are fed through the same decode step, one
position per step. Rotary embedding: RoPE (theta 10000) on adjacent dim
pairs. In the PyTorch form the causal mask is an additive bias folded into
the score GEMM; the fused kernel reads each sequence's positions 0..P.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from .configs import V2_LITE, MoEConfig


@dataclass(frozen=True)
class DecoderConfig:
    moe: MoEConfig
    num_layers: int
    first_dense: int          # leading layers with a dense FFN
    dense_intermediate: int
    num_heads: int
    kv_lora_rank: int
    qk_nope: int
    qk_rope: int
    v_head: int
    vocab: int
    rms_eps: float = 1e-6
    rope_theta: float = 10000.0

    @property
    def hidden(self) -> int:
        return self.moe.hidden

    @property
    def num_moe_layers(self) -> int:
        return self.num_layers - self.first_dense


V2_LITE_DECODER = DecoderConfig(
    moe=V2_LITE, num_layers=27, first_dense=1, dense_intermediate=10944, num_heads=16,
    kv_lora_rank=512, qk_nope=128, qk_rope=64, v_head=128, vocab=102400)


def _rms(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    return F.rms_norm(x, (x.shape[-1],), w, eps)


def _rope(x: torch.Tensor, freqs: torch.Tensor) -> torch.Tensor:
    """RoPE on the last dim of x [B, ..., R] (pairs of adjacent dims rotated
    as complex numbers) by freqs [B, R/2] (complex64)."""
    shape = [freqs.shape[0]] + [1] * (x.dim() - 2) + [freqs.shape[1]]
    xc = torch.view_as_complex(x.float().reshape(*x.shape[:-1], -1, 2))
    return torch.view_as_real(xc * freqs.view(shape)).flatten(-2).to(x.dtype)


class DecoderHarness:
    """Greedy decode of ``batch`` sequences through the decoder; ``moe(li,
    x)`` computes MoE layer ``li`` (0-based over the MoE layers) of normed
    hidden states ``x`` [batch, H]."""

    def __init__(self, cfg: DecoderConfig, moe, batch: int, max_len: int, seed: int = 0,
                 device="cuda", std: float = 0.02, fused_attention: bool | None = None):
        """``fused_attention`` (default: on a CUDA device) runs each layer's
        attention core as the library's one-launch MLA decode kernel
        (``sl_mla_decode``) and each residual add with the RMSNorm after it
        as one launch (``sl_add_rmsnorm``); otherwise, and on the host, as
        PyTorch ops."""
        self.cfg = cfg
        self.moe = moe
        self.batch = batch
        self.max_len = max_len
        self.device = torch.device(device)
        dev, bf = self.device, torch.bfloat16
        # seeded on the device that holds the weights (the host port draws
        # its own values: it is timed, not compared)
        g = torch.Generator(device=dev)
        g.manual_seed(seed * 7919 + 17)
        H, nh = cfg.hidden, cfg.num_heads
        dq = cfg.qk_nope + cfg.qk_rope

        def w(*shape):
            return (torch.randn(*shape, generator=g, device=dev) * std).to(bf)

        self.embed = w(cfg.vocab, H)
        self.head = w(cfg.vocab, H)
        self.final_norm = torch.ones(H, dtype=bf, device=dev)
        self.layers = []
        for li in range(cfg.num_layers):
            lw = {
                "in_norm": torch.ones(H, dtype=bf, device=dev),
                "post_norm": torch.ones(H, dtype=bf, device=dev),
                "kv_norm": torch.ones(cfg.kv_lora_rank, dtype=bf, device=dev),
                # q_proj [nh * dq, H] and kv_a_proj [rank + rope, H] as one GEMM
                "wqkv": w(nh * dq + cfg.kv_lora_rank + cfg.qk_rope, H),
                # kv_b_proj [nh * (nope + v), rank] split per head into the
                # absorbed key (W_uk) and value (W_uv) maps
                "w_uk": w(nh, cfg.qk_nope, cfg.kv_lora_rank),
                "w_uv": w(nh, cfg.v_head, cfg.kv_lora_rank),
                "wo": w(H, nh * cfg.v_head),
            }
            if li < cfg.first_dense:
                lw["w13"] = w(2 * cfg.dense_intermediate, H)
                lw["w2"] = w(H, cfg.dense_intermediate)
            self.layers.append(lw)
        L = cfg.num_layers
        # compressed cache per layer and position: [c_kv (rank) | k_pe (rope)]
        self.cache = torch.zeros(L, batch, max_len, cfg.kv_lora_rank + cfg.qk_rope, dtype=bf,
                                 device=dev)
        inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, cfg.qk_rope, 2).float() / cfg.qk_rope))
        ang = torch.arange(max_len).float()[:, None] * inv[None, :]
        self.freqs = torch.polar(torch.ones_like(ang), ang).to(dev)   # complex64
        self.rope_cs = torch.view_as_real(self.freqs).contiguous()    # [max_len, r/2, 2]
        self.fused_attention = (self.device.type == "cuda") if fused_attention is None \
            else bool(fused_attention)
        self.pos = torch.zeros(batch, dtype=torch.long, device=dev)
        self.scale = 1.0 / math.sqrt(dq)
        self._ar = torch.arange(max_len, device=dev)
        self._rows = torch.arange(batch, device=dev)
        # w_uk / w_uv per head, laid out for batched GEMMs over heads
        for lw in self.layers:
            lw["w_uk_t"] = lw["w_uk"].contiguous()                  # [nh, nope, rank]
            lw["w_uv_t"] = lw["w_uv"].transpose(1, 2).contiguous()  # [nh, rank, v]

    def reset(self) -> None:
        self.pos.zero_()

    def _attention(self, li: int, x: torch.Tensor, mask_bias: torch.Tensor,
                   freqs: torch.Tensor) -> torch.Tensor:
        cfg, lw = self.cfg, self.layers[li]
        B, nh, R = x.shape[0], cfg.num_heads, cfg.kv_lora_rank
        dq = cfg.qk_nope + cfg.qk_rope
        qkv = self._linear(x, lw["wqkv"])
        if self.fused_attention:
            from ._lib import check, lib, ptr
            o = torch.empty(B, nh * cfg.v_head, dtype=x.dtype, device=x.device)
            check(lib().sl_mla_decode(ptr(qkv), qkv.shape[1], ptr(lw["kv_norm"]), cfg.rms_eps,
                                      ptr(lw["w_uk_t"]), ptr(lw["w_uv"]), ptr(self.rope_cs),
                                      ptr(self.pos), ptr(self.cache[li]), B, nh, cfg.qk_nope,
                                      cfg.qk_rope, R, cfg.v_head, self.max_len, self.scale,
                                      ptr(o), torch.cuda.current_stream().cuda_stream),
                  "sl_mla_decode")
            return self._linear(o, lw["wo"])
        q = qkv[:, :nh * dq].view(B, nh, dq)
        kv = qkv[:, nh * dq:]
        c = _rms(kv[:, :R], lw["kv_norm"], cfg.rms_eps)
        k_pe = _rope(kv[:, R:], freqs)
        self.cache[li, self._rows, self.pos] = torch.cat([c, k_pe], dim=-1)
        # absorbed query: [q_nope W_uk | rope(q_pe)] against [c_kv | k_pe]
        q_lat = torch.bmm(q[..., :cfg.qk_nope].transpose(0, 1), lw["w_uk_t"])  # [nh, B, R]
        qf = torch.cat([q_lat.transpose(0, 1), _rope(q[..., cfg.qk_nope:], freqs)], dim=-1)
        cl = self.cache[li]                                                   # [B, Lmax, R+r]
        s = torch.baddbmm(mask_bias, qf, cl.transpose(1, 2), alpha=self.scale)
        p = torch.softmax(s, dim=-1)
        o_lat = torch.bmm(p, cl[..., :R])                                     # [B, nh, R]
        o = torch.bmm(o_lat.transpose(0, 1), lw["w_uv_t"])                   # [nh, B, v]
        return F.linear(o.transpose(0, 1).reshape(B, nh * cfg.v_head), lw["wo"])

    def _linear(self, x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """x @ w.T: the library's skinny linear (``sl_linear_small``) for
        one or two rows on the device (faster than cuBLAS there), else
        PyTorch's (cuBLAS)."""
        if self.fused_attention and x.shape[0] <= 2 and x.shape[1] * x.shape[0] * 2 <= 200 * 1024:
            from ._lib import check, lib, ptr
            x = x.contiguous()
            y = torch.empty(x.shape[0], w.shape[0], dtype=x.dtype, device=x.device)
            check(lib().sl_linear_small(ptr(x), x.shape[0], x.shape[1], ptr(w), w.shape[0],
                                        ptr(y), torch.cuda.current_stream().cuda_stream),
                  "sl_linear_small")
            return y
        return F.linear(x, w)

    def _add_norm(self, h: torch.Tensor, delta: torch.Tensor | None,
                  w: torch.Tensor) -> torch.Tensor:
        """h += delta (in place; None: no add), then RMSNorm(h) * w."""
        eps = self.cfg.rms_eps
        if self.fused_attention:
            from ._lib import check, lib, ptr
            out = torch.empty_like(h)
            check(lib().sl_add_rmsnorm(ptr(h), ptr(delta) if delta is not None else None,
                                       ptr(w), eps, ptr(out), h.shape[0], h.shape[1],
                                       torch.cuda.current_stream().cuda_stream),
                  "sl_add_rmsnorm")
            return out
        if delta is not None:
            h.add_(delta)
        return _rms(h, w, eps)

    def _dense_ffn(self, li: int, x: torch.Tensor) -> torch.Tensor:
        lw = self.layers[li]
        g, u = F.linear(x, lw["w13"]).chunk(2, dim=-1)
        return F.linear(F.silu(g) * u, lw["w2"])

    def step(self, ids: torch.Tensor) -> torch.Tensor:
        """One decode step: token ids [batch] at the sequences' positions ->
        the greedy next ids [batch]; the positions advance by one."""
        cfg = self.cfg
        h = self.embed[ids]
        # per step: the positions' rotations and the causal mask as an additive
        # bias over the cache (0 up to each sequence's position, -inf after)
        freqs = self.freqs[self.pos]
        mask_bias = torch.zeros(h.shape[0], 1, self.max_len, dtype=h.dtype, device=h.device)
        mask_bias.masked_fill_((self._ar[None, :] > self.pos[:, None])[:, None, :],
                               float("-inf"))
        x = self._add_norm(h, None, self.layers[0]["in_norm"])
        for li in range(cfg.num_layers):
            lw = self.layers[li]
            x = self._add_norm(h, self._attention(li, x, mask_bias, freqs), lw["post_norm"])
            f = self._dense_ffn(li, x) if li < cfg.first_dense else \
                self.moe(li - cfg.first_dense, x)
            nxt = self.layers[li + 1]["in_norm"] if li + 1 < cfg.num_layers else self.final_norm
            x = self._add_norm(h, f, nxt)
        logits = F.linear(x, self.head)
        self.pos.add_(1)
        return logits.argmax(dim=-1)


class OffloadedDecoder:
    """The decoder on this GPU with its MoE layers behind slot caches: the
    layers of a ``MoEDecodeStack`` (one GPU) or an ``EPDecodeStack``
    (expert parallelism: every rank decodes its own sequences, the MoE
    layers exchange tokens with the other ranks). A decode step replays as
    one CUDA graph that also feeds its greedy ids back as the next input."""

    def __init__(self, cfg: DecoderConfig, stack, batch: int, max_len: int, seed: int = 0):
        self.cfg = cfg
        self.stack = stack
        self.device = stack.device
        layers = stack.layers
        if len(layers) != cfg.num_moe_layers:
            raise ValueError(f"{len(layers)} MoE layers for a decoder with {cfg.num_moe_layers}")
        self.layers = layers          # the MoE layers (slot caches, stream timers)
        self.model = DecoderHarness(cfg, lambda li, x: layers[li](x), batch, max_len, seed,
                                    self.device)
        self.graph = None
        self._ids = torch.zeros(batch, dtype=torch.long, device=self.device)
        self._out = None

    def _step(self) -> torch.Tensor:
        out = self.model.step(self._ids)
        self._ids.copy_(out)
        return out

    def capture(self, tokens: int | None = None) -> bool:
        """Capture one decode step (after one eager warm-up step, whose
        position is then rewound)."""
        ids0 = self._ids.clone()
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            self._step()
        torch.cuda.current_stream(self.device).wait_stream(s)
        self.model.pos.sub_(1)
        self._ids.copy_(ids0)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._out = self._step()
        self.graph = g
        return True

    def replay(self, ids: torch.Tensor | None = None) -> torch.Tensor:
        """One decode step; ``ids`` [batch] (device) are the input tokens, or
        None to continue from the last step's greedy ids. Returns the next
        ids [batch] (a static buffer)."""
        if ids is not None:
            self._ids.copy_(ids, non_blocking=True)
        self.graph.replay()
        return self._out

    def decode_step(self, ids_host: torch.Tensor, out_host: torch.Tensor) -> torch.Tensor:
        """Public end-to-end call: host token ids in, host next ids out."""
        out_host.copy_(self.replay(ids_host.to(self.device, non_blocking=True)),
                       non_blocking=True)
        return out_host

    def save(self) -> dict:
        """The sequences' state (KV caches, positions, next input ids)."""
        m = self.model
        return {"cache": m.cache.clone(), "pos": m.pos.clone(), "ids": self._ids.clone()}

    def restore(self, saved: dict) -> None:
        m = self.model
        m.cache.copy_(saved["cache"])
        m.pos.copy_(saved["pos"])
        self._ids.copy_(saved["ids"])

    def check(self) -> None:
        self.stack.check()

    def stats(self) -> dict:
        return self.stack.stats()

    def release(self) -> None:
        self.graph = None
        if hasattr(self.stack, "release"):
            self.stack.release()
