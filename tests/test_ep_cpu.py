"""Expert-parallel dispatch / combine on CPU with gloo ranks (world size 2
and 4): the product's shard map, packed all-gather dispatch and
reduce-scatter combine (the NCCL exchange), and the routed exchange's row
layout and sum rule (the NVLink kernels' semantics, with gloo collectives
standing in for the peer pushes), with the per-rank expert math done by the
oracle, must reproduce the single-process oracle layer output."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import moe as omoe
from oracle import routing as orouting

H, I, E, K, T, NSH = 256, 128, 16, 4, 3, 1


def _model(seed=0):
    g = torch.Generator().manual_seed(seed)
    w13 = (torch.randn(E, 2 * I, H, generator=g) * 0.05).to(torch.bfloat16)
    w2 = (torch.randn(E, H, I, generator=g) * 0.05).to(torch.bfloat16)
    sh13 = (torch.randn(NSH, 2 * I, H, generator=g) * 0.05).to(torch.bfloat16)
    sh2 = (torch.randn(NSH, H, I, generator=g) * 0.05).to(torch.bfloat16)
    gw = (torch.randn(E, H, generator=g) * 0.05).to(torch.bfloat16)
    return w13, w2, sh13, sh2, gw


def _tokens(rank):
    g = torch.Generator().manual_seed(100 + rank)
    return torch.randn(T, H, generator=g).to(torch.bfloat16)


def _route(x, gw):
    return orouting.grouped_topk(orouting.gate_logits(x, gw), K, True)


def _reference(world):
    w13, w2, sh13, sh2, gw = _model()
    outs = []
    for r in range(world):
        x = _tokens(r)
        tw, ti = _route(x, gw)
        routed = omoe.fused_experts(x, w13, w2, tw, ti)
        shared = sum(omoe.expert_mlp(x, sh13[i], sh2[i]).float() for i in range(NSH))
        outs.append((routed.float() * 2.0 + shared).to(torch.bfloat16))
    return outs


def _rank_main(rank, world, port, result_dir):
    from sluice_b200 import ep
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w13, w2, sh13, sh2, gw = _model()
        lo, per, local_of = ep.expert_shard(E, world, rank)
        x = _tokens(rank)
        tw, ti = _route(x, gw)
        xg, twg, tig = ep.dispatch(x, tw, ti)
        assert xg.shape == (world * T, H) and tig.shape == (world * T, K)
        assert torch.equal(xg[rank * T:(rank + 1) * T], x)
        # the per-rank expert computation (oracle here; sl_fused_experts_partial on GPU)
        emap = torch.tensor(local_of, dtype=torch.int32)
        routed = omoe.fused_experts(xg, w13[lo:lo + per], w2[lo:lo + per], twg, tig, emap)
        part = routed.float() * 2.0
        own = slice(rank * T, (rank + 1) * T)
        part[own] += sum(omoe.expert_mlp(x, sh13[i], sh2[i]).float() for i in range(NSH))
        out = ep.combine(part).to(torch.bfloat16)
        torch.save(out, os.path.join(result_dir, f"out{rank}.pt"))
    finally:
        dist.destroy_process_group()


def _routed_rows(xs, tws, tis, rank, world):
    """The routed dispatch's output on `rank` (sl_ep_dispatch): its own T
    tokens, then each peer's tokens that select one of `rank`'s experts
    (peers in rank order, tokens in order), then empty rows (id -1, weight
    0); src = (home rank << 16) | token, -1 for an empty row."""
    per = E // world
    rows_x, rows_w, rows_i, src = [xs[rank]], [tws[rank]], [tis[rank]], \
        [(rank << 16) | t for t in range(T)]
    for p in range(world):
        if p == rank:
            continue
        for t in range(T):
            if bool(((tis[p][t].long() // per) == rank).any()):
                rows_x.append(xs[p][t:t + 1])
                rows_w.append(tws[p][t:t + 1])
                rows_i.append(tis[p][t:t + 1])
                src.append((p << 16) | t)
    xg, twg, tig = torch.cat(rows_x), torch.cat(rows_w), torch.cat(rows_i)
    pad = world * T - xg.shape[0]
    xg = torch.cat([xg, torch.zeros(pad, H, dtype=xg.dtype)])
    twg = torch.cat([twg, torch.zeros(pad, K)])
    tig = torch.cat([tig, torch.full((pad, K), -1, dtype=torch.int32)])
    return xg, twg, tig, src + [-1] * pad


def _routed_rank_main(rank, world, port, result_dir):
    """The routed exchange's data flow with gloo collectives standing in for
    the peer pushes: every rank's partials over the rows it received travel
    back to their home rank, which sums its own partial and those of the
    ranks its token went to, in rank order."""
    from sluice_b200 import ep
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w13, w2, sh13, sh2, gw = _model()
        lo, per, local_of = ep.expert_shard(E, world, rank)
        x = _tokens(rank)
        tw, ti = _route(x, gw)
        gather = lambda t: [torch.empty_like(t) for _ in range(world)]
        xs, tws, tis = gather(x), gather(tw), gather(ti)
        for out, t in ((xs, x), (tws, tw), (tis, ti)):
            dist.all_gather(out, t)
        xg, twg, tig, src = _routed_rows(xs, tws, tis, rank, world)
        emap = torch.tensor(local_of, dtype=torch.int32)
        part = omoe.fused_experts(xg, w13[lo:lo + per], w2[lo:lo + per], twg, tig,
                                  emap).float() * 2.0
        part[:T] += sum(omoe.expert_mlp(x, sh13[i], sh2[i]).float() for i in range(NSH))
        # combine: rows received from peer p go back to p at their token
        back = torch.zeros(world, T, H)
        for r, s_ in enumerate(src):
            if s_ >= 0 and (s_ >> 16) != rank:
                back[s_ >> 16, s_ & 0xffff] = part[r]
        recv = [torch.empty(world, T, H) for _ in range(world)]
        dist.all_gather(recv, back)
        went = [(ti[t].long() // per) for t in range(T)]
        out = torch.zeros(T, H)
        for q in range(world):
            for t in range(T):
                if q == rank:
                    out[t] += part[t]
                elif bool((went[t] == q).any()):
                    out[t] += recv[q][rank, t]
        torch.save(out.to(torch.bfloat16), os.path.join(result_dir, f"out{rank}.pt"))
        torch.save(int(sum(1 for s_ in src if s_ >= 0)), os.path.join(result_dir, f"n{rank}.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_routed_exchange_matches_single_process(world, tmp_path):
    mp.start_processes(_routed_rank_main, args=(world, _free_port(), str(tmp_path)),
                       nprocs=world, start_method="spawn")
    ref = _reference(world)
    rows = 0
    for r in range(world):
        out = torch.load(os.path.join(tmp_path, f"out{r}.pt")).float()
        want = ref[r].float()
        assert (out - want).abs().max() <= 2e-2 * want.abs().max()
        rows += torch.load(os.path.join(tmp_path, f"n{r}.pt"))
    # routed: fewer rows than an all-gather (world * world * T) whenever some
    # token's experts miss some rank
    assert rows <= world * world * T


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("world", [2, 4])
def test_ep_dispatch_combine_matches_single_process(world, tmp_path):
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       start_method="spawn")
    ref = _reference(world)
    for r in range(world):
        out = torch.load(os.path.join(tmp_path, f"out{r}.pt")).float()
        want = ref[r].float()
        # partial sums are combined in fp32 across ranks: bf16-level agreement
        assert (out - want).abs().max() <= 2e-2 * want.abs().max()


def test_expert_shard_covers_every_expert_once():
    from sluice_b200 import ep
    for world in (1, 2, 4, 8):
        seen = []
        for r in range(world):
            lo, per, local_of = ep.expert_shard(256, world, r)
            owned = [g for g, l in enumerate(local_of) if l >= 0]
            assert owned == list(range(lo, lo + per))
            assert [local_of[g] for g in owned] == list(range(per))
            seen += owned
        assert sorted(seen) == list(range(256))
    with pytest.raises(ValueError):
        ep.expert_shard(64, 3, 0)


def test_pack_unpack_round_trip():
    from sluice_b200 import ep
    x = torch.randn(5, 64).to(torch.bfloat16)
    tw = torch.rand(5, 3)
    ti = torch.randint(0, 100, (5, 3), dtype=torch.int32)
    x2, tw2, ti2 = ep.unpack_routing(ep.pack_routing(x, tw, ti), 64, 3)
    assert torch.equal(x2, x) and torch.equal(tw2, tw) and torch.equal(ti2, ti)
