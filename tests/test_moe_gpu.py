"""GPU parity: fused_experts (tcgen05 grouped GEMMs + combine) vs the oracle.

Tolerance (bf16): |out - ref| <= 2e-2 * max|ref| + 2e-2 * |ref| elementwise,
the north star's 2e-2 relative, scaled by the output's magnitude so that
near-zero entries are not held to their own relative error.
"""

import os

import numpy as np
import pytest
import torch

from oracle import moe as omoe
from sluice_b200 import ops

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
RTOL = 2e-2


def assert_moe_close(out, ref, rtol=RTOL):
    out, ref = out.float().cpu(), ref.float().cpu()
    assert torch.isfinite(out).all()
    scale = ref.abs().max().item()
    err = (out - ref).abs()
    bound = rtol * scale + rtol * ref.abs()
    bad = (err > bound).sum().item()
    assert bad == 0, f"{bad} elements off; max err {err.max().item():.3e} vs scale {scale:.3e}"
    rel = (err.norm() / ref.norm()).item()
    assert rel < rtol / 2, rel


def test_golden_case_through_expert_map():
    z = np.load(os.path.join(GOLDEN, "moe.npz"))
    bf = lambda a: torch.from_numpy(a).view(torch.bfloat16)
    hs, w13, w2 = bf(z["hs"]), bf(z["w13"]), bf(z["w2"])
    tw, ti = torch.from_numpy(z["topk_weights"]), torch.from_numpy(z["topk_ids"])
    emap = torch.from_numpy(z["expert_map"])
    ref = bf(z["out"])
    out = ops.fused_experts(hs.cuda(), w13.cuda(), w2.cuda(), tw.cuda(), ti.cuda(),
                            global_num_experts=emap.numel(), expert_map=emap.cuda())
    torch.cuda.synchronize()
    assert ops.workspace_status(ops.fused_experts.last_workspace) == 0
    assert_moe_close(out, ref)


def _random_case(T, H, I, S, E, k, n_sh, seed, map_frac=0.8, std=0.02):
    g = torch.Generator().manual_seed(seed)
    hs = torch.randn(T, H, generator=g).to(torch.bfloat16)
    w13 = (torch.randn(S, 2 * I, H, generator=g) * std).to(torch.bfloat16)
    w2 = (torch.randn(S, H, I, generator=g) * std).to(torch.bfloat16)
    perm = torch.randperm(E, generator=g)
    emap = torch.full((E,), -1, dtype=torch.int32)
    nres = min(S, int(E * map_frac))
    emap[perm[:nres]] = torch.randperm(S, generator=g)[:nres].to(torch.int32)
    ti = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).to(torch.int32)
    tw = torch.rand(T, k, generator=g).float()
    sh13 = sh2 = None
    if n_sh:
        sh13 = (torch.randn(n_sh, 2 * I, H, generator=g) * std).to(torch.bfloat16)
        sh2 = (torch.randn(n_sh, H, I, generator=g) * std).to(torch.bfloat16)
    return hs, w13, w2, emap, ti, tw, sh13, sh2


def _reference(hs, w13, w2, emap, ti, tw, sh13, sh2, scale):
    routed = omoe.fused_experts(hs, w13, w2, tw, ti, emap)
    shared = None
    if sh13 is not None:
        shared = sum(omoe.expert_mlp(hs, sh13[i], sh2[i]).float()
                     for i in range(sh13.shape[0])).to(torch.bfloat16)
    return omoe.layer_output(routed, shared, scale)


@pytest.mark.parametrize("T,H,I,S,E,k,n_sh,scale", [
    (8, 2048, 1408, 48, 64, 6, 2, 1.0),     # V2-Lite decode, c=8
    (1, 2048, 1408, 48, 64, 6, 2, 1.0),     # c=1
    (12, 2048, 768, 96, 128, 8, 0, 1.0),    # Qwen3 decode, c=12
    (16, 2048, 768, 128, 128, 8, 0, 1.0),   # Qwen3 resident
    (5, 256, 128, 6, 8, 3, 1, 2.5),         # tiny, shared + routed scaling
    (40, 512, 256, 16, 32, 4, 0, 1.0),      # experts with > 16 tokens (several items)
])
def test_random_cases(T, H, I, S, E, k, n_sh, scale):
    hs, w13, w2, emap, ti, tw, sh13, sh2 = _random_case(T, H, I, S, E, k, n_sh, seed=T * 7 + H)
    c = lambda t: None if t is None else t.cuda()
    out = ops.fused_experts(c(hs), c(w13), c(w2), c(tw), c(ti), global_num_experts=E,
                            expert_map=c(emap), shared_w13=c(sh13), shared_w2=c(sh2),
                            routed_scaling_factor=scale)
    torch.cuda.synchronize()
    assert ops.workspace_status(ops.fused_experts.last_workspace) == 0
    assert_moe_close(out, _reference(hs, w13, w2, emap, ti, tw, sh13, sh2, scale))


def test_unmapped_and_out_of_range_ids_contribute_nothing():
    T, H, I, S, E, k = 4, 256, 128, 4, 8, 2
    hs, w13, w2, emap, ti, tw, _, _ = _random_case(T, H, I, S, E, k, 0, seed=11)
    emap[:] = -1
    out = ops.fused_experts(hs.cuda(), w13.cuda(), w2.cuda(), tw.cuda(), ti.cuda(),
                            global_num_experts=E, expert_map=emap.cuda())
    assert torch.count_nonzero(out).item() == 0
    ti2 = ti.clone()
    ti2[:, 0] = -1
    ti2[:, 1] = 1000
    emap2 = torch.arange(E, dtype=torch.int32) % S
    out2 = ops.fused_experts(hs.cuda(), w13.cuda(), w2.cuda(), tw.cuda(), ti2.cuda(),
                             global_num_experts=E, expert_map=emap2.cuda())
    assert torch.count_nonzero(out2).item() == 0


def test_no_map_indexes_slots_directly_and_repeats_are_stable():
    T, H, I, S, k = 8, 512, 256, 8, 2
    hs, w13, w2, _, _, tw, _, _ = _random_case(T, H, I, S, S, k, 0, seed=3)
    g = torch.Generator().manual_seed(4)
    ti = torch.stack([torch.randperm(S, generator=g)[:k] for _ in range(T)]).to(torch.int32)
    a = ops.fused_experts(hs.cuda(), w13.cuda(), w2.cuda(), tw.cuda(), ti.cuda())
    b = ops.fused_experts(hs.cuda(), w13.cuda(), w2.cuda(), tw.cuda(), ti.cuda())
    assert torch.equal(a, b)
    assert_moe_close(a, omoe.fused_experts(hs, w13, w2, tw, ti))


def test_torch_op_registration():
    T, H, I, S, E, k = 3, 256, 128, 4, 8, 2
    hs, w13, w2, emap, ti, tw, _, _ = _random_case(T, H, I, S, E, k, 0, seed=21)
    out = torch.ops.sluice.fused_experts(hs.cuda(), w13.cuda(), w2.cuda(), tw.cuda(),
                                         ti.cuda(), "silu", E, emap.cuda())
    assert_moe_close(out, omoe.fused_experts(hs, w13, w2, tw, ti, emap))


@pytest.mark.parametrize("T,H,I,S,E,k,n_sh,scale", [
    (8, 512, 256, 8, 16, 4, 1, 1.0),
    (8, 7168, 2048, 16, 256, 8, 1, 2.5),    # DeepSeek-V3 expert shape, decode
    (33, 1024, 512, 6, 12, 3, 0, 1.0),      # several items per expert
    (400, 1024, 512, 8, 8, 2, 1, 2.5),      # ~100 tokens per expert: wide token tiles
    (1000, 512, 256, 6, 6, 2, 0, 1.0),      # 333 per expert: two wide items each
])
def test_fp8_block_scaled_cases(T, H, I, S, E, k, n_sh, scale):
    """fp8 e4m3 weights with 128x128 block scales: within 5e-2 of the oracle's
    fp32 dequantised math."""
    from sluice_b200 import synth
    hs, w13, w2, emap, ti, tw, sh13, sh2 = _random_case(T, H, I, S, E, k, n_sh, seed=T + H)
    q13, s13 = synth.quantize_block_fp8(w13)
    q2, s2 = synth.quantize_block_fp8(w2)
    qs13 = qs2 = ss13 = ss2 = None
    if n_sh:
        qs13, ss13 = synth.quantize_block_fp8(sh13)
        qs2, ss2 = synth.quantize_block_fp8(sh2)
    c = lambda t: None if t is None else t.cuda()
    out = ops.fused_experts(c(hs), c(q13), c(q2), c(tw), c(ti), global_num_experts=E,
                            expert_map=c(emap), w1_scale=c(s13), w2_scale=c(s2),
                            block_shape=[128, 128], shared_w13=c(qs13), shared_w2=c(qs2),
                            shared_w13_scale=c(ss13), shared_w2_scale=c(ss2),
                            routed_scaling_factor=scale)
    torch.cuda.synchronize()
    assert ops.workspace_status(ops.fused_experts.last_workspace) == 0
    routed = omoe.fused_experts(hs, q13, q2, tw, ti, emap, s13, s2)
    shared = None
    if n_sh:
        shared = sum(omoe.shared_experts(hs, qs13[i], qs2[i], ss13[i], ss2[i]).float()
                     for i in range(n_sh)).to(torch.bfloat16)
    assert_moe_close(out, omoe.layer_output(routed, shared, scale), rtol=5e-2)


@pytest.mark.parametrize("fp8", [False, True], ids=["bf16", "fp8"])
@pytest.mark.parametrize("T,H,I,S,E,k", [
    (64, 1024, 512, 16, 16, 8),      # 32 tokens per expert: 64-token tiles
    (256, 1024, 512, 16, 16, 8),     # 128 per expert: 128-token tiles
    (1024, 1024, 512, 16, 20, 8),    # grid-wide token gather, a few unmapped experts
])
def test_prefill_sized_steps(T, H, I, S, E, k, fp8):
    """Token tiles of 64 / 128 and the grid-wide gather, bf16 and fp8."""
    from sluice_b200 import synth
    hs, w13, w2, emap, ti, tw, _, _ = _random_case(T, H, I, S, E, k, 0, seed=T + k,
                                                   map_frac=1.0 if E == S else 0.8)
    c = lambda t: None if t is None else t.cuda()
    kw, ref_kw, rtol = {}, {}, RTOL
    if fp8:
        w13, s13 = synth.quantize_block_fp8(w13)
        w2, s2 = synth.quantize_block_fp8(w2)
        kw = dict(w1_scale=c(s13), w2_scale=c(s2))
        ref_kw = dict(w13_scale=s13, w2_scale=s2)
        rtol = 5e-2
    out = ops.fused_experts(c(hs), c(w13), c(w2), c(tw), c(ti), global_num_experts=E,
                            expert_map=c(emap), **kw)
    torch.cuda.synchronize()
    assert ops.workspace_status(ops.fused_experts.last_workspace) == 0
    assert_moe_close(out, omoe.fused_experts(hs, w13, w2, tw, ti, emap, **ref_kw), rtol=rtol)


def test_empty_step_and_oversized_slot_count():
    """T = 0 returns an empty output without launching work; more slots plus
    shared experts than the grouping step handles (1056) is refused with an
    error instead of running."""
    from sluice_b200 import _lib
    H, I = 256, 128
    w13 = torch.zeros(4, 2 * I, H, dtype=torch.bfloat16, device="cuda")
    w2 = torch.zeros(4, H, I, dtype=torch.bfloat16, device="cuda")
    hs = torch.empty(0, H, dtype=torch.bfloat16, device="cuda")
    tw = torch.empty(0, 2, dtype=torch.float32, device="cuda")
    ti = torch.empty(0, 2, dtype=torch.int32, device="cuda")
    out = ops.fused_experts(hs, w13, w2, tw, ti, global_num_experts=4)
    assert out.shape == (0, H)
    S = 1100
    w13b = torch.zeros(S, 2 * I, H, dtype=torch.bfloat16, device="cuda")
    w2b = torch.zeros(S, H, I, dtype=torch.bfloat16, device="cuda")
    hs = torch.randn(2, H, device="cuda").to(torch.bfloat16)
    tw = torch.ones(2, 2, device="cuda")
    ti = torch.zeros(2, 2, dtype=torch.int32, device="cuda")
    with pytest.raises(_lib.SluiceError) as ei:
        ops.fused_experts(hs, w13b, w2b, tw, ti, global_num_experts=S)
    assert ei.value.status == _lib.SL_ERR_UNSUPPORTED


def test_fp8_wide_tiles_split_around_the_stream():
    """The wide-tile fp8 GEMMs (a prefill-sized step: ~100 tokens per expert)
    split around the gap's expert stream: phase 0 over the resident experts
    while the misses stream, phase 1 over the streamed ones and the combine,
    against the oracle; then the whole call again on the now-resident experts,
    bit-equal to the split one."""
    from sluice_b200 import synth
    from sluice_b200.offloader import ExpertStreamOffloader
    T, H, I, E, S, k = 320, 1024, 512, 16, 8, 2
    g = torch.Generator().manual_seed(5)
    w13 = (torch.randn(E, 2 * I, H, generator=g) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn(E, H, I, generator=g) * 0.02).to(torch.bfloat16)
    q13, s13 = synth.quantize_block_fp8(w13)
    q2, s2 = synth.quantize_block_fp8(w2)
    hs = torch.randn(T, H, generator=g).to(torch.bfloat16)
    # every token picks 2 distinct experts among 6: 3 pinned (resident), 3 streamed
    choice = torch.stack([torch.randperm(6, generator=g)[:k] for _ in range(T)])
    pool = torch.tensor([0, 1, 2, 9, 11, 14])
    ti = pool[choice].to(torch.int32)
    tw = torch.rand(T, k, generator=g)
    tw = (tw / tw.sum(1, keepdim=True)).float()
    off = ExpertStreamOffloader(S, protect_frac=0.5, fast_hit=True)
    cache = off.install_layer(q13, q2, pins=[0, 1, 2], prefill_resident=False, device="cuda",
                              w13_scale=s13, w2_scale=s2)
    x, tic, twc = hs.cuda(), ti.cuda(), tw.cuda()
    ws = ops.fused_experts_workspace(T, k, H, I, S, 0, torch.device("cuda"))
    out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    kw = dict(w1_scale=cache.w13_scale, w2_scale=cache.w2_scale)
    main, side = torch.cuda.current_stream(), torch.cuda.Stream()
    cache.plan(tic)
    side.wait_stream(main)
    with torch.cuda.stream(side):
        cache.stream()
    args = (x, cache.w13, cache.w2, twc, tic, cache.expert_map, cache.state)
    ops.fused_experts_phase(*args, 0, ws, out, **kw)
    main.wait_stream(side)
    ops.fused_experts_phase(*args, 1, ws, out, **kw)
    torch.cuda.synchronize()
    cache.check()
    assert ops.workspace_status(ws) == 0
    assert int((cache.expert_map >= 0).sum()) == 6
    ref = omoe.fused_experts(hs, q13, q2, tw, ti, None, s13, s2)
    assert_moe_close(out, ref, rtol=5e-2)
    whole = ops.fused_experts(x, cache.w13, cache.w2, twc, tic, expert_map=cache.expert_map,
                              **kw)
    torch.cuda.synchronize()
    assert torch.equal(whole, out)


@pytest.mark.parametrize("fp8,T", [(False, 8), (True, 8), (False, 320), (True, 320)])
def test_four_part_split_on_two_streams(fp8, T):
    """The phased call in its four parts as the offloaded layer issues them:
    grouping and the resident experts' GEMMs on the main stream; the stream,
    then (after the grouping) the streamed experts' GEMMs on a side stream;
    the combine on the main stream after both. Against the oracle, and bit-
    equal to the whole call on the now-resident experts (decode- and
    prefill-sized steps, bf16 and fp8)."""
    from sluice_b200 import _lib, synth
    from sluice_b200.offloader import ExpertStreamOffloader
    H, I, E, S, k = 1024, 512, 16, 8, 2
    g = torch.Generator().manual_seed(11 + T)
    w13 = (torch.randn(E, 2 * I, H, generator=g) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn(E, H, I, generator=g) * 0.02).to(torch.bfloat16)
    hs = torch.randn(T, H, generator=g).to(torch.bfloat16)
    # every token picks 2 distinct experts among 6: 3 pinned (resident), 3 streamed
    choice = torch.stack([torch.randperm(6, generator=g)[:k] for _ in range(T)])
    ti = torch.tensor([0, 1, 2, 9, 11, 14])[choice].to(torch.int32)
    tw = torch.rand(T, k, generator=g)
    tw = (tw / tw.sum(1, keepdim=True)).float()
    off = ExpertStreamOffloader(S, protect_frac=0.5, fast_hit=True)
    if fp8:
        q13, s13 = synth.quantize_block_fp8(w13)
        q2, s2 = synth.quantize_block_fp8(w2)
        cache = off.install_layer(q13, q2, pins=[0, 1, 2], prefill_resident=False,
                                  device="cuda", w13_scale=s13, w2_scale=s2)
        ref = omoe.fused_experts(hs, q13, q2, tw, ti, None, s13, s2)
        rtol = 5e-2
    else:
        cache = off.install_layer(w13, w2, pins=[0, 1, 2], prefill_resident=False,
                                  device="cuda")
        ref = omoe.fused_experts(hs, w13, w2, tw, ti)
        rtol = RTOL
    x, tic, twc = hs.cuda(), ti.cuda(), tw.cuda()
    ws = ops.fused_experts_workspace(T, k, H, I, S, 0, torch.device("cuda"))
    out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    kw = dict(w1_scale=cache.w13_scale, w2_scale=cache.w2_scale)
    args = (x, cache.w13, cache.w2, twc, tic, cache.expert_map, cache.state)
    main, side = torch.cuda.current_stream(), torch.cuda.Stream()
    cache.plan(tic)
    side.wait_stream(main)
    with torch.cuda.stream(side):
        cache.stream()
    ops.fused_experts_phase(*args, _lib.PHASE_GROUP, ws, out, **kw)
    grouped = torch.cuda.Event()
    grouped.record(main)
    with torch.cuda.stream(side):
        side.wait_event(grouped)
        ops.fused_experts_phase(*args, _lib.PHASE_STREAMED_GEMMS, ws, out, **kw)
    ops.fused_experts_phase(*args, _lib.PHASE_RESIDENT_GEMMS, ws, out, **kw)
    main.wait_stream(side)
    ops.fused_experts_phase(*args, _lib.PHASE_COMBINE, ws, out, **kw)
    torch.cuda.synchronize()
    cache.check()
    assert ops.workspace_status(ws) == 0
    assert int((cache.expert_map >= 0).sum()) == 6
    assert_moe_close(out, ref, rtol=rtol)
    whole = ops.fused_experts(x, cache.w13, cache.w2, twc, tic, expert_map=cache.expert_map,
                              **kw)
    torch.cuda.synchronize()
    assert torch.equal(whole, out)
