"""Layer shapes and routing modes of the workloads the reference is measured on.

The reference publishes decode numbers for DeepSeek-V2-Lite and
Qwen3-30B-A3B (``README.md:49-67`` of kfirtoledo/sluice) and the workload set
adds a grouped-GEMM microbench and a DeepSeek-V3-shaped expert-parallel stack.
Routing modes follow the vLLM model definitions the reference runs under:
V2-Lite — softmax, one group, top-6, no renormalisation; Qwen3 — softmax
top-8 with renormalisation (``topk_softmax``); V3 — sigmoid with
``e_score_correction_bias``, 8 groups / top-4 groups, top-8, renormalised,
``routed_scaling_factor`` 2.5 applied to the routed output by the runner tail.
"""

from __future__ import annotations

from dataclasses import dataclass, field


@dataclass(frozen=True)
class RoutingConfig:
    topk: int
    renormalize: bool
    scoring_func: str = "softmax"        # "softmax" | "sigmoid"
    num_expert_group: int = 1
    topk_group: int = 1
    use_grouped_topk: bool = False
    has_score_bias: bool = False         # e_score_correction_bias

    @property
    def scoring(self) -> int:
        return 0 if self.scoring_func == "softmax" else 1


@dataclass(frozen=True)
class MoEConfig:
    name: str
    hidden: int
    num_experts: int
    moe_intermediate: int
    n_shared: int
    routing: RoutingConfig
    num_moe_layers: int
    routed_scaling_factor: float = 1.0
    weight_dtype: str = "bf16"

    @property
    def bytes_per_expert(self) -> int:
        """w13 [2I, H] + w2 [H, I] in the weight dtype (+ fp32 128x128 block
        scales for fp8)."""
        H, I = self.hidden, self.moe_intermediate
        if self.weight_dtype == "bf16":
            return 6 * H * I
        return 3 * H * I + 4 * (2 * I // 128 * (H // 128) + (H // 128) * (I // 128))

    @property
    def flops_per_pair(self) -> int:
        return 6 * self.hidden * self.moe_intermediate


V2_LITE = MoEConfig(
    name="deepseek-v2-lite", hidden=2048, num_experts=64, moe_intermediate=1408,
    n_shared=2, num_moe_layers=26,
    routing=RoutingConfig(topk=6, renormalize=False, use_grouped_topk=True))

QWEN3_30B_A3B = MoEConfig(
    name="qwen3-30b-a3b", hidden=2048, num_experts=128, moe_intermediate=768,
    n_shared=0, num_moe_layers=48,
    routing=RoutingConfig(topk=8, renormalize=True))

DEEPSEEK_V3 = MoEConfig(
    name="deepseek-v3", hidden=7168, num_experts=256, moe_intermediate=2048,
    n_shared=1, num_moe_layers=58, routed_scaling_factor=2.5, weight_dtype="fp8",
    routing=RoutingConfig(topk=8, renormalize=True, scoring_func="sigmoid",
                          num_expert_group=8, topk_group=4, use_grouped_topk=True,
                          has_score_bias=True))

CONFIGS = {c.name: c for c in (V2_LITE, QWEN3_30B_A3B, DEEPSEEK_V3)}


def with_layers(cfg: MoEConfig, n: int) -> MoEConfig:
    from dataclasses import replace
    return replace(cfg, num_moe_layers=n)
