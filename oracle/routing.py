"""CPU restatement of the router arithmetic (TEST INFRASTRUCTURE).

The reference calls vLLM for routing (``offloader.py:2582-2585``:
``runner.gate(hs)`` then ``router.select_experts``). vLLM is third-party
code: the reference pins v0.23 (``README.md:13``, ``pyproject.toml:19-22``);
0.22.0 is installed here. This module restates, with torch on the CPU:

* gate: ``logits = bf16(x @ W^T [+ b])`` — vLLM's bf16 ``ReplicatedLinear``
  gate; the optional per-expert logit bias is the synthetic workload's
  popularity skew (added in fp32 before the bf16 rounding);
* ``grouped_topk``: vLLM ``model_executor/layers/fused_moe/cpu_fused_moe.py``
  59-115 (same arithmetic as ``router/grouped_topk_router.py`` 81-166):
  fp32 softmax or sigmoid, optional ``e_score_correction_bias`` (group score =
  sum of the top-2 biased scores, selection on biased scores, weights from
  unbiased scores), group mask over the ``topk_group`` best groups, top-k,
  optional renormalisation, ``routed_scaling_factor``;
* ``softmax_topk``: the contract of vLLM's CUDA ``topk_softmax`` used by
  ``FusedTopKRouter`` (``router/fused_topk_router.py`` 69-118): fp32 softmax
  over all experts, top-k, optional division by the sum of the selected
  weights.

Every top-k here uses the canonical tie rule: score descending, id ascending
(``torch.sort(..., stable=True)``), and returns ids in that order.
"""

from __future__ import annotations

import torch


def gate_logits(x: torch.Tensor, w: torch.Tensor,
                bias: torch.Tensor | None = None) -> torch.Tensor:
    """bf16 router logits [T, E] from bf16 x [T, H] and bf16 W [E, H]."""
    acc = x.float() @ w.float().t()
    if bias is not None:
        acc = acc + bias.float().unsqueeze(0)
    return acc.to(torch.bfloat16)


def canonical_topk(scores: torch.Tensor, k: int):
    """Top-k along the last dim: values descending, ties to the lower id."""
    vals, idx = torch.sort(scores, dim=-1, descending=True, stable=True)
    return vals[..., :k], idx[..., :k]


def grouped_topk(logits: torch.Tensor, topk: int, renormalize: bool,
                 num_expert_group: int = 1, topk_group: int = 1,
                 scoring_func: str = "softmax",
                 routed_scaling_factor: float = 1.0,
                 e_score_correction_bias: torch.Tensor | None = None):
    """Restates cpu_fused_moe.py:59-115. Returns (weights f32, ids i32)."""
    g = logits.float()
    if scoring_func == "softmax":
        scores = torch.softmax(g, dim=-1)
    elif scoring_func == "sigmoid":
        scores = g.sigmoid()
    else:
        raise ValueError(scoring_func)
    T, E = scores.shape
    if e_score_correction_bias is not None:
        original = scores
        scores = scores + e_score_correction_bias.float().unsqueeze(0)
        top2, _ = canonical_topk(scores.view(T, num_expert_group, -1), 2)
        group_scores = top2.sum(dim=-1)
    else:
        group_scores = scores.view(T, num_expert_group, -1).max(dim=-1).values
    _, group_idx = canonical_topk(group_scores, topk_group)
    group_mask = torch.zeros_like(group_scores)
    group_mask.scatter_(1, group_idx, 1)
    score_mask = (group_mask.unsqueeze(-1)
                  .expand(T, num_expert_group, E // num_expert_group)
                  .reshape(T, -1))
    masked = scores.masked_fill(~score_mask.bool(), float("-inf"))
    if e_score_correction_bias is not None:
        _, ids = canonical_topk(masked, topk)
        weights = original.gather(1, ids)
    else:
        weights, ids = canonical_topk(masked, topk)
    if renormalize:
        weights = weights / weights.sum(dim=-1, keepdim=True)
    if routed_scaling_factor != 1.0:
        weights = weights * routed_scaling_factor
    return weights.to(torch.float32), ids.to(torch.int32)


def softmax_topk(logits: torch.Tensor, topk: int, renormalize: bool):
    """topk_softmax contract (fused_topk_router.py:69-118)."""
    scores = torch.softmax(logits.float(), dim=-1)
    weights, ids = canonical_topk(scores, topk)
    if renormalize:
        weights = weights / weights.sum(dim=-1, keepdim=True)
    return weights.to(torch.float32), ids.to(torch.int32)


def route(logits: torch.Tensor, cfg) -> tuple[torch.Tensor, torch.Tensor]:
    """Dispatch on a routing config (``sluice_b200.configs.RoutingConfig``
    fields: topk, renormalize, num_expert_group, topk_group, scoring_func,
    routed_scaling_factor, use_grouped_topk) with an optional score bias."""
    if cfg.use_grouped_topk:
        return grouped_topk(logits, cfg.topk, cfg.renormalize,
                            cfg.num_expert_group, cfg.topk_group,
                            cfg.scoring_func, cfg.routed_scaling_factor,
                            getattr(cfg, "score_bias", None))
    return softmax_topk(logits, cfg.topk, cfg.renormalize)


def kth_margin(logits: torch.Tensor, cfg) -> torch.Tensor:
    """Per token, the gap between the k-th and (k+1)-th selection score.

    Used by tests to skip tokens whose selection sits on an exact (or
    sub-rounding) tie, where the reference's choice is implementation-defined.
    """
    g = logits.float()
    s = torch.softmax(g, -1) if cfg.scoring_func == "softmax" else g.sigmoid()
    b = getattr(cfg, "score_bias", None)
    if b is not None:
        s = s + b.float().unsqueeze(0)
    vals, _ = torch.sort(s, dim=-1, descending=True)
    k = cfg.topk
    if vals.shape[-1] <= k:
        return torch.full((s.shape[0],), float("inf"))
    return vals[:, k - 1] - vals[:, k]
