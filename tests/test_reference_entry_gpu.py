"""The reference's router-split entry, run on this build's ops under the
reference's own op names.

The reference patches vLLM's ``MoERunner._forward_entry`` with a closure
(``offloader.py:2578-2603``) that calls ``gate``, ``select_experts``,
``torch.ops.vllm.sluice_stream_gap`` and ``torch.ops.vllm.fused_experts``,
then runs the shared-expert MLP and returns ``(shared, routed)`` for vLLM's
runner tail to add. ``make_forward_entry`` below follows that closure call for
call, with the same argument names and keyword arguments; it binds this
build's ``Router`` and the ops that ``ops.register_reference_names()``
defines. Checked per step against the oracle (slot map: the reference's SLRU
restated; output: vLLM's torch-native MoE restated, 2e-2 relative), eagerly
and replayed from a CUDA graph captured around the whole entry.
"""

import pytest
import torch
import torch.nn.functional as F

from oracle import moe as omoe
from oracle.slot_policy import SlotPolicyModel
from sluice_b200 import configs, ops, synth
from sluice_b200.offloader import ExpertStreamOffloader
from test_moe_gpu import assert_moe_close

pytestmark = pytest.mark.gpu


def make_forward_entry(idx, w13, w2, gne, emap, shared_layer, sel, orig, gate, thr):
    """The reference's per-layer entry factory (offloader.py:2569-2603), the
    staged-ids branch left out (a kept negative result there, off by
    default)."""

    def _forward_entry(hs, rl, sei, iid, lname, unpad):
        if hs.shape[0] > thr:
            return orig(hs, rl, sei, iid, lname, unpad)
        if gate is not None:
            rl, _ = gate(hs)
        tw, ti = sel(hidden_states=hs, router_logits=rl, input_ids=iid)
        h = torch.ops.vllm.sluice_stream_gap(hs, ti, idx)
        routed = torch.ops.vllm.fused_experts(h, w13, w2, tw, ti, activation="silu",
                                              global_num_experts=gne, expert_map=emap)
        if shared_layer is None:
            return routed
        sh = shared_layer(sei if sei is not None else hs)
        return (sh, routed)

    return _forward_entry


class SharedMLP:
    """The caller's shared-expert MLP (vLLM's dense SwiGLU: gate_up_proj with
    every gate row then every up row, down_proj), in bf16 on the GPU."""

    def __init__(self, sh13, sh2):
        n, two_i, H = sh13.shape
        I = two_i // 2
        self.w13 = torch.cat([sh13[:, :I].reshape(n * I, H), sh13[:, I:].reshape(n * I, H)])
        self.w2 = sh2.permute(1, 0, 2).reshape(H, n * I).contiguous()

    def __call__(self, x):
        gu = F.linear(x, self.w13)
        g, u = gu.chunk(2, dim=-1)
        return F.linear(F.silu(g) * u, self.w2)


def test_reference_entry_runs_unedited_on_the_registered_ops():
    ops.register_reference_names()
    cfg = configs.V2_LITE
    T, slots = 8, 48
    w13, w2 = synth.layer_weights(cfg, 0, seed=5, device="cuda")
    gw, lb, sb = synth.gate_params(cfg, 0, seed=5, device="cuda")
    sh13, sh2 = synth.shared_weights(cfg, 0, seed=5, device="cuda")
    off = ExpertStreamOffloader(slots, protect_frac=0.5, fast_hit=True)
    cache = off.install_layer(w13, w2, device="cuda")
    idx = ops.register_gap_layer(cache)
    router = ops.Router(cfg.routing, gw, lb, sb)

    def orig(*a):
        raise AssertionError("decode-sized steps stay on the router-split entry")

    model = SlotPolicyModel(cache.num_slots, list(range(cfg.num_experts)), cfg.num_experts,
                            0.5, True)
    w13c, w2c = w13.cpu(), w2.cpu()
    sh_w13 = SharedMLP(sh13, sh2)
    g13c, g2c = sh_w13.w13.cpu(), sh_w13.w2.cpu()
    stream = synth.TokenStream(cfg.hidden, T, seed=6, reuse=0.3)

    def check_step(x, sh, routed, step):
        torch.cuda.synchronize()
        cache.check()
        ti = last["ti"].cpu()
        tw = last["tw"].cpu()
        model.gap(ti.flatten().tolist())
        assert cache.expert_map.cpu().tolist() == model.expert_map, step
        ref_routed = omoe.fused_experts(x, w13c, w2c, tw, ti)
        ref = omoe.layer_output(ref_routed, omoe.shared_experts(x, g13c, g2c), 1.0)
        assert_moe_close(routed, ref_routed)
        # vLLM's runner tail: shared + routed (routed scaling 1.0 here)
        assert_moe_close(sh + routed, ref)

    last = {}

    def sel(**kw):
        tw, ti = router.select_experts(**kw)
        last["tw"], last["ti"] = tw, ti
        return tw, ti

    entry = make_forward_entry(idx, cache.w13, cache.w2, cfg.num_experts, cache.expert_map,
                               SharedMLP(sh13, sh2), sel, orig, router.gate,
                               slots // cfg.routing.topk)
    misses0 = cache.stats()["misses"]
    for step in range(4):
        x = stream.next()
        sh, routed = entry(x.cuda(), None, None, None, "model.layers.1.mlp.experts", cfg.hidden)
        check_step(x, sh, routed, step)

    # the whole entry captured in one CUDA graph, replayed on new tokens; one
    # more real step on a side stream first (library handles and workspaces
    # are created outside capture)
    static_x = torch.zeros(T, cfg.hidden, dtype=torch.bfloat16, device="cuda")
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    x = stream.next()
    with torch.cuda.stream(side):
        static_x.copy_(x.cuda())
        sh, routed = entry(static_x, None, None, None, "model.layers.1.mlp.experts", cfg.hidden)
    torch.cuda.current_stream().wait_stream(side)
    check_step(x, sh, routed, 4)
    g = torch.cuda.CUDAGraph()
    # the gap must not run twice for one step: capture records, it does not
    # execute, so the planner state only advances on replay
    with torch.cuda.graph(g):
        static_sh, static_routed = entry(static_x, None, None, None,
                                         "model.layers.1.mlp.experts", cfg.hidden)
    for step in range(5, 9):
        x = stream.next()
        static_x.copy_(x.cuda())
        g.replay()
        check_step(x, static_sh, static_routed, step)
    assert cache.stats()["misses"] > misses0, "the steps must stream misses"
    del g
