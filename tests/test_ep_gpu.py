"""Expert parallelism on 2 GPUs: each rank's layer output (its own tokens,
experts sharded across ranks, fp32 partials summed on the home rank) must
match the single-process oracle within the bf16 tolerance, with the exchange
done by the NVLink peer-memory kernels and by NCCL collectives; the two
exchanges must agree bit for bit (two ranks: one fp32 addition either way),
eager and under CUDA-graph replay. Skipped on a box with fewer than 2 GPUs."""

import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, out_dir, exchange, slots=48):
    import torch.distributed as dist

    from oracle import moe as omoe
    from oracle import routing as orouting
    from sluice_b200 import configs, ep, synth

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port),
                      NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        cfg = configs.V2_LITE
        stack = ep.EPDecodeStack(cfg, slots=slots, seed=3, num_layers=1, exchange=exchange)
        layer = stack.layers[0]
        w13, w2 = synth.layer_weights(cfg, 0, 3, device="cuda")
        w13, w2 = w13.cpu(), w2.cpu()
        sh13, sh2 = (t.cpu() for t in synth.shared_weights(cfg, 0, 3, device="cuda"))
        tokens = synth.TokenStream(cfg.hidden, 8, seed=50 + rank)
        errs = []
        for _ in range(3):
            x = tokens.next().cuda()
            out = layer(x)
            tw, ti, logits = layer.router.route(x)
            torch.cuda.synchronize()
            xc = x.cpu()
            rc = cfg.routing
            otw, oti = orouting.grouped_topk(logits.cpu(), rc.topk, rc.renormalize)
            routed = omoe.fused_experts(xc, w13, w2, otw, oti)
            shared = sum(omoe.expert_mlp(xc, sh13[i], sh2[i]).float()
                         for i in range(cfg.n_shared)).to(torch.bfloat16)
            ref = omoe.layer_output(routed, shared).float()
            got = out.float().cpu()
            errs.append(((got - ref).abs().max() / ref.abs().max()).item())
        stack.check()
        torch.save(torch.tensor(errs), os.path.join(out_dir, f"err{rank}.pt"))
    finally:
        dist.destroy_process_group()


def _v3_mini():
    """A DeepSeek-V3-style layer at test size: fp8 e4m3 experts with 128x128
    block scales, sigmoid scoring with score bias, 8 groups / top-4 groups,
    top-8 with renormalisation, routed scaling 2.5, one shared expert."""
    from sluice_b200 import configs
    return configs.MoEConfig(
        name="v3-mini", hidden=1024, num_experts=64, moe_intermediate=256, n_shared=1,
        num_moe_layers=1, routed_scaling_factor=2.5, weight_dtype="fp8",
        routing=configs.RoutingConfig(topk=8, renormalize=True, scoring_func="sigmoid",
                                      num_expert_group=8, topk_group=4,
                                      use_grouped_topk=True, has_score_bias=True))


def _rank_main_fp8(rank, world, port, out_dir, slots=48):
    import torch.distributed as dist

    from oracle import moe as omoe
    from oracle import routing as orouting
    from sluice_b200 import ep, synth

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port),
                      NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    stack = None
    try:
        cfg = _v3_mini()
        stack = ep.EPDecodeStack(cfg, slots=slots, seed=4, num_layers=1)
        layer = stack.layers[0]
        prm = {k: v.cpu() for k, v in synth.layer_params(cfg, 0, 4, device="cuda").items()}
        sh = {k: v.cpu() for k, v in synth.shared_params(cfg, 0, 4, device="cuda").items()}
        _, _, sb = synth.gate_params(cfg, 0, 4, device="cpu")
        tokens = synth.TokenStream(cfg.hidden, 8, seed=60 + rank)
        rc = cfg.routing
        errs = []
        for _ in range(3):
            x = tokens.next().cuda()
            out = layer(x)
            tw, ti, logits = layer.router.route(x)
            torch.cuda.synchronize()
            xc = x.cpu()
            otw, oti = orouting.grouped_topk(logits.cpu(), rc.topk, rc.renormalize,
                                             rc.num_expert_group, rc.topk_group,
                                             rc.scoring_func, 1.0, sb)
            routed = omoe.fused_experts(xc, prm["w13"], prm["w2"], otw, oti, None,
                                        prm["w13_scale"], prm["w2_scale"])
            shared = omoe.shared_experts(xc, sh["shared_w13"][0], sh["shared_w2"][0],
                                         sh["shared_w13_scale"][0], sh["shared_w2_scale"][0])
            ref = omoe.layer_output(routed, shared, cfg.routed_scaling_factor).float()
            got = out.float().cpu()
            errs.append(((got - ref).abs().max() / ref.abs().max()).item())
        stack.check()
        torch.save(torch.tensor(errs), os.path.join(out_dir, f"errf{rank}.pt"))
    finally:
        if stack is not None:
            stack.release()
        dist.destroy_process_group()


@pytest.mark.parametrize("slots", [48, 16], ids=["resident", "offloaded-waves"])
def test_ep2_fp8_v3_style_layer_matches_oracle(tmp_path, slots):
    """fp8 block-scaled experts, sigmoid grouped routing and routed scaling
    under expert parallelism (NVLink exchange): within the fp8 tolerance.
    16 slots of 32 local experts: 8 tokens per rank exceed the envelope, so
    the gathered rows run in expert waves (weights and scales streamed)."""
    mp.start_processes(_rank_main_fp8, args=(2, _free_port(), str(tmp_path), slots),
                       nprocs=2, start_method="spawn")
    for r in range(2):
        errs = torch.load(os.path.join(tmp_path, f"errf{r}.pt"))
        assert (errs < 5e-2).all(), errs


def _agree_main(rank, world, port, out_dir, slots=48):
    import torch.distributed as dist

    from sluice_b200 import configs, ep, synth

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port),
                      NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    stacks = []
    try:
        cfg = configs.V2_LITE
        outs = {}
        for exchange in ("nvlink", "nccl"):
            stack = ep.EPDecodeStack(cfg, slots=slots, seed=5, num_layers=2, exchange=exchange)
            stacks.append(stack)
            tokens = synth.TokenStream(cfg.hidden, 4, seed=70 + rank)
            xs = [tokens.next().cuda() for _ in range(4)]
            eager = [stack.step(x).clone() for x in xs[:2]]
            graphed = stack.capture(4)
            replay = [stack.replay(x).clone() for x in xs[2:]]
            torch.cuda.synchronize()
            stack.check()
            outs[exchange] = (torch.stack(eager + replay).cpu(), graphed)
        same = bool(torch.equal(outs["nvlink"][0], outs["nccl"][0]))
        torch.save({"same": same, "graphed": outs["nvlink"][1]},
                   os.path.join(out_dir, f"agree{rank}.pt"))
    finally:
        for s in stacks:
            s.release()
        dist.destroy_process_group()


@pytest.mark.parametrize("exchange,slots", [("nvlink", 48), ("nccl", 48), ("nvlink", 24)],
                         ids=["nvlink-resident", "nccl-resident", "nvlink-offloaded"])
def test_ep2_layer_matches_oracle(tmp_path, exchange, slots):
    """slots 48 >= 32 local experts: every expert resident; slots 24: the
    gap streams misses on a side stream while the resident experts run."""
    mp.start_processes(_rank_main, args=(2, _free_port(), str(tmp_path), exchange, slots),
                       nprocs=2, start_method="spawn")
    for r in range(2):
        errs = torch.load(os.path.join(tmp_path, f"err{r}.pt"))
        assert (errs < 2e-2).all(), errs


@pytest.mark.parametrize("slots", [48, 16], ids=["resident", "offloaded-waves"])
def test_ep2_nvlink_exchange_equals_nccl(tmp_path, slots):
    """Both exchanges, eager and graph-replayed; 16 slots: steps of 4 tokens
    per rank exceed the envelope (16 // 6 // 2 = 1) and run in waves."""
    mp.start_processes(_agree_main, args=(2, _free_port(), str(tmp_path), slots), nprocs=2,
                       start_method="spawn")
    for r in range(2):
        res = torch.load(os.path.join(tmp_path, f"agree{r}.pt"))
        assert res["graphed"], "the NVLink exchange must capture in a CUDA graph"
        assert res["same"]
