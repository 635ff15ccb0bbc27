"""CPU restatement of the MoE layer arithmetic (TEST INFRASTRUCTURE).

The reference's routed computation is ``torch.ops.vllm.fused_experts(h, w13,
w2, tw, ti, activation="silu", global_num_experts, expert_map)``
(``offloader.py:2590-2599``), third-party vLLM code. Its semantics restated
here follow vLLM 0.22:

* per (token t, choice j): ``e = expert_map[ids[t, j]]``; a ``-1`` entry (not
  resident / owned by another rank) contributes nothing
  (``fused_moe.py:1798``, ``1837-1838``);
* expert MLP: ``gate_up = x @ w13[e]^T`` (``w13[e]`` is ``[2I, H]``, gate rows
  first), ``a = silu(gate_up[:I]) * gate_up[I:]``
  (``layers/activation.py:137-141``), ``z = a @ w2[e]^T`` (``w2[e]`` is
  ``[H, I]``);
* the bf16 rounding chain and the weighted top-k sum of vLLM's torch-native
  ``cpu_fused_moe_torch`` (``cpu_fused_moe.py:428-482``): each linear rounds to
  bf16, the activation rounds to bf16, then ``sum_j w[t,j] * z`` in fp32 and
  one final bf16 rounding;
* the shared experts (``offloader.py:2602``) are a dense SwiGLU MLP on every
  token, and vLLM's tail (``runner/moe_runner.py:350-366``, ``663-680``)
  scales the routed output by ``routed_scaling_factor`` in bf16 and adds the
  shared output in bf16;
* fp8 (vLLM's ``use_fp8_w8a8`` with ``block_shape=[128, 128]``,
  ``fused_moe.py:1587-1632``): e4m3 weights times fp32 128x128 block scales;
  the activations entering each GEMM (the token rows, then the SwiGLU
  output) are quantised per token and 128-column group the way
  ``per_token_group_quant_fp8`` does ([vLLM] ``quantization/utils/fp8_utils.py``
  ``_per_token_group_quant_fp8``, 95-150: scale = max(amax, 1e-10) * (1/448),
  ``q = clamp(x / scale, -448, 448)`` to e4m3; vLLM's compiled CUDA op and
  its torch-native ``QuantFP8._quantize_group_native`` compute the same
  scale as ``amax / 448``, which can differ from this one in the last bit);
  products of the dequantised
  operands accumulate in fp32, each GEMM output rounds to bf16.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


def silu_and_mul(x: torch.Tensor) -> torch.Tensor:
    d = x.shape[-1] // 2
    return F.silu(x[..., :d]) * x[..., d:]


FP8_MAX = 448.0


def quant_group_fp8(x: torch.Tensor, group: int = 128):
    """vLLM's per-token-group e4m3 quantisation: (q e4m3 [..., K], scale fp32
    [..., K/group])."""
    *lead, K = x.shape
    g = x.float().reshape(*lead, K // group, group)
    amax = g.abs().amax(dim=-1, keepdim=True).clamp(min=1e-10)
    scale = amax * (1.0 / FP8_MAX)
    q = (g / scale).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)
    return q.reshape(*lead, K), scale.reshape(*lead, K // group)


def quant_dequant_group_fp8(x: torch.Tensor, group: int = 128) -> torch.Tensor:
    """Activations through vLLM's per-token-group e4m3 quantisation, returned
    dequantised in fp32 (q * scale)."""
    *lead, K = x.shape
    q, scale = quant_group_fp8(x, group)
    g = q.float().reshape(*lead, K // group, group) * scale.unsqueeze(-1)
    return g.reshape(*lead, K)


def expert_mlp(x: torch.Tensor, w13: torch.Tensor, w2: torch.Tensor,
               act_quant: bool = False) -> torch.Tensor:
    """One expert's SwiGLU MLP in the dtype of its operands. ``act_quant``:
    quantise each GEMM's activations per 128-column group (fp8 w8a8)."""
    if w13.dtype != x.dtype:
        # dequantised fp32 weights: compute in fp32, round like a bf16 kernel
        xa = quant_dequant_group_fp8(x) if act_quant else x.float()
        gu = F.linear(xa, w13.float()).to(x.dtype)
        a = silu_and_mul(gu)
        aa = quant_dequant_group_fp8(a) if act_quant else a.float()
        return F.linear(aa, w2.float()).to(x.dtype)
    gu = F.linear(x, w13)
    return F.linear(silu_and_mul(gu), w2)


def dequant_block_fp8(w: torch.Tensor, scale: torch.Tensor,
                      block: tuple[int, int] = (128, 128)) -> torch.Tensor:
    """e4m3 [..., N, K] times scale [..., ceil(N/bn), ceil(K/bk)] -> fp32."""
    bn, bk = block
    s = scale.float().repeat_interleave(bn, dim=-2).repeat_interleave(bk, dim=-1)
    s = s[..., : w.shape[-2], : w.shape[-1]]
    return w.float() * s


def fused_experts(hs: torch.Tensor, w13: torch.Tensor, w2: torch.Tensor,
                  topk_weights: torch.Tensor, topk_ids: torch.Tensor,
                  expert_map: torch.Tensor | None = None,
                  w13_scale: torch.Tensor | None = None,
                  w2_scale: torch.Tensor | None = None,
                  block_shape=(128, 128)) -> torch.Tensor:
    """Routed output [T, H] (bf16) of the experts held in ``w13``/``w2``.

    ``w13``/``w2`` are indexed by slot (``expert_map[global] -> slot``) or, with
    no map, by global id.
    """
    T, H = hs.shape
    ids = topk_ids.long()
    if expert_map is not None:
        m = expert_map.long()
        valid = (ids >= 0) & (ids < m.numel())
        slots = torch.where(valid, m[ids.clamp(0, m.numel() - 1)],
                            torch.full_like(ids, -1))
    else:
        slots = ids
    z = torch.zeros(T, ids.shape[1], H, dtype=hs.dtype)
    for s in sorted(set(slots.flatten().tolist())):
        if s < 0:
            continue
        sel = (slots == s).nonzero(as_tuple=False)
        tok = sel[:, 0]
        a = w13[s]
        b = w2[s]
        if w13_scale is not None:
            a = dequant_block_fp8(a, w13_scale[s], block_shape)
            b = dequant_block_fp8(b, w2_scale[s], block_shape)
        z[sel[:, 0], sel[:, 1]] = expert_mlp(hs[tok], a, b, act_quant=w13_scale is not None)
    return (z.float() * topk_weights.float().unsqueeze(-1)).sum(dim=1).to(hs.dtype)


def shared_experts(hs: torch.Tensor, w13_sh: torch.Tensor, w2_sh: torch.Tensor,
                   w13_scale=None, w2_scale=None, block_shape=(128, 128)):
    """Dense shared-expert MLP (one MLP of intermediate n_shared*I)."""
    a, b = w13_sh, w2_sh
    if w13_scale is not None:
        a = dequant_block_fp8(a, w13_scale, block_shape)
        b = dequant_block_fp8(b, w2_scale, block_shape)
    return expert_mlp(hs, a, b, act_quant=w13_scale is not None)


def layer_output(routed: torch.Tensor, shared: torch.Tensor | None,
                 routed_scaling_factor: float = 1.0) -> torch.Tensor:
    """vLLM runner tail: bf16 scale of the routed output, bf16 add."""
    out = routed.clone()
    if routed_scaling_factor != 1.0:
        out *= routed_scaling_factor
    if shared is not None:
        out = shared + out
    return out


def split_shared(w13_sh: torch.Tensor, w2_sh: torch.Tensor, n_shared: int):
    """Split one shared MLP of intermediate n*I into n experts of I each.

    ``w13_sh`` is [2*n*I, H] (all gate rows, then all up rows); ``w2_sh`` is
    [H, n*I]. Returns ([n, 2I, H], [n, H, I]) with sum over the n experts
    equal to the single MLP in exact arithmetic.
    """
    two_ni, H = w13_sh.shape
    I = two_ni // (2 * n_shared)
    gate = w13_sh[: n_shared * I].view(n_shared, I, H)
    up = w13_sh[n_shared * I:].view(n_shared, I, H)
    w13 = torch.cat([gate, up], dim=1).contiguous()
    w2 = w2_sh.view(H, n_shared, I).permute(1, 0, 2).contiguous()
    return w13, w2
