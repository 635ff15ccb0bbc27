"""Seeded synthetic layers and token streams (no checkpoints are available).

Follows the workload definitions: expert weights ~ N(0, 0.02) in bf16; gate
W [E, H] ~ N(0, 0.02) plus a per-expert logit bias ``b_e = 1.5 * log(1 /
rank_e)`` over a seeded permutation (Zipf-like popularity); decode tokens
~ N(0, 1) with 60% of each step's tokens repeating the previous step's vector
plus N(0, 0.1) noise (temporal locality).
"""

from __future__ import annotations

import math

import torch

from .configs import MoEConfig


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def layer_weights(cfg: MoEConfig, layer: int, seed: int = 0, device="cuda",
                  std: float = 0.02, num_experts: int | None = None, expert_lo: int = 0):
    """(w13 [E,2I,H], w2 [E,H,I]) bf16 for experts [expert_lo, expert_lo+num_experts).

    Each expert's weights come from its own seeded stream, so any subset
    (an expert-parallel shard) reproduces the same values.
    """
    E = cfg.num_experts if num_experts is None else num_experts
    H, I = cfg.hidden, cfg.moe_intermediate
    w13 = torch.empty(E, 2 * I, H, dtype=torch.bfloat16, device=device)
    w2 = torch.empty(E, H, I, dtype=torch.bfloat16, device=device)
    for i in range(E):
        e = expert_lo + i
        g = _gen(seed * 1_000_003 + layer * 4099 + e, device)
        w13[i].copy_(torch.randn(2 * I, H, generator=g, device=device) * std)
        w2[i].copy_(torch.randn(H, I, generator=g, device=device) * std)
    return w13, w2


def quantize_block_fp8(w: torch.Tensor, block: int = 128):
    """e4m3 weights and fp32 block scales (dequantised value = q * scale) for
    [..., N, K] weights, one scale per 128x128 block (max-abs / 448)."""
    *lead, N, K = w.shape
    wb = w.float().reshape(*lead, N // block, block, K // block, block)
    amax = wb.abs().amax(dim=(-3, -1), keepdim=True).clamp(min=1e-12)
    scale = amax / 448.0
    q = (wb / scale).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)
    return (q.reshape(*lead, N, K),
            scale.reshape(*lead, N // block, K // block).contiguous())


def shared_weights(cfg: MoEConfig, layer: int, seed: int = 0, device="cuda", std=0.02):
    """Shared experts as n_shared experts of the routed I: ([n,2I,H], [n,H,I])."""
    if cfg.n_shared == 0:
        return None, None
    H, I, n = cfg.hidden, cfg.moe_intermediate, cfg.n_shared
    g = _gen(seed * 1_000_003 + layer * 4099 + 777_777, device)
    w13 = (torch.randn(n, 2 * I, H, generator=g, device=device) * std).to(torch.bfloat16)
    w2 = (torch.randn(n, H, I, generator=g, device=device) * std).to(torch.bfloat16)
    return w13, w2


def layer_params(cfg: MoEConfig, layer: int, seed: int = 0, device="cuda",
                 num_experts: int | None = None, expert_lo: int = 0) -> dict:
    """Routed expert parameters in the config's weight dtype: ``w13``, ``w2``
    and, for fp8 configs, ``w13_scale`` / ``w2_scale`` (128x128 blocks)."""
    w13, w2 = layer_weights(cfg, layer, seed, device=device, num_experts=num_experts,
                            expert_lo=expert_lo)
    if cfg.weight_dtype != "fp8":
        return {"w13": w13, "w2": w2}
    q13, s13 = quantize_block_fp8(w13)
    del w13
    q2, s2 = quantize_block_fp8(w2)
    return {"w13": q13, "w2": q2, "w13_scale": s13, "w2_scale": s2}


def shared_params(cfg: MoEConfig, layer: int, seed: int = 0, device="cuda") -> dict:
    """Shared experts in the config's weight dtype (empty dict if none)."""
    sh13, sh2 = shared_weights(cfg, layer, seed, device=device)
    if sh13 is None:
        return {}
    if cfg.weight_dtype != "fp8":
        return {"shared_w13": sh13, "shared_w2": sh2}
    q13, s13 = quantize_block_fp8(sh13)
    q2, s2 = quantize_block_fp8(sh2)
    return {"shared_w13": q13, "shared_w2": q2, "shared_w13_scale": s13,
            "shared_w2_scale": s2}


def gate_params(cfg: MoEConfig, layer: int, seed: int = 0, device="cuda", std=0.02,
                zipf_bias: float = 1.5):
    """(gate W [E,H] bf16, logit bias [E] f32, score bias [E] f32 or None)."""
    E, H = cfg.num_experts, cfg.hidden
    g = _gen(seed * 1_000_003 + layer * 4099 + 555_555, "cpu")
    w = (torch.randn(E, H, generator=g) * std).to(torch.bfloat16)
    rank = torch.randperm(E, generator=g).double() + 1.0
    lb = (zipf_bias * torch.log(1.0 / rank)).float()
    sb = (torch.rand(E, generator=g) * 0.1).float() if cfg.routing.has_score_bias else None
    to = lambda t: None if t is None else t.to(device)
    return to(w), to(lb), to(sb)


class TokenStream:
    """Decode-step inputs with temporal locality (seeded, CPU generation)."""

    def __init__(self, hidden: int, tokens: int, seed: int = 0, reuse: float = 0.6,
                 noise: float = 0.1):
        self.hidden, self.tokens = hidden, tokens
        self.reuse, self.noise = reuse, noise
        self.g = torch.Generator().manual_seed(seed + 31337)
        self.prev = None

    def next(self) -> torch.Tensor:
        x = torch.randn(self.tokens, self.hidden, generator=self.g)
        if self.prev is not None:
            keep = torch.rand(self.tokens, generator=self.g) < self.reuse
            noisy = self.prev + self.noise * torch.randn(self.tokens, self.hidden, generator=self.g)
            x = torch.where(keep.unsqueeze(1), noisy, x)
        self.prev = x
        return x.to(torch.bfloat16)


def zipf_ids(tokens: int, topk: int, num_experts: int, s: float = 1.1,
             gen: torch.Generator | None = None, perm: torch.Tensor | None = None):
    """Top-k ids per token without replacement, Zipf(s) over a permutation."""
    p = 1.0 / torch.arange(1, num_experts + 1, dtype=torch.float64) ** s
    idx = torch.multinomial(p.expand(tokens, -1), topk, replacement=False, generator=gen)
    if perm is not None:
        idx = perm[idx]
    return idx.to(torch.int32)


def expected_unique(topk: int, tokens: int, num_experts: int) -> float:
    """Uniform-routing expectation of distinct experts (for reporting only)."""
    n = topk * tokens
    return num_experts * (1 - (1 - 1 / num_experts) ** n)


__all__ = ["layer_weights", "shared_weights", "quantize_block_fp8", "layer_params",
           "shared_params", "gate_params", "TokenStream", "zipf_ids",
           "expected_unique", "math"]
