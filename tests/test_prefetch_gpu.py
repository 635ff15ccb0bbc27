"""Opt-in cross-layer prefetch (sl_prefetch_slots) on the GPU.

* The device prefetch planner follows the oracle's restatement bit for bit
  (expert map, slot owners, SLRU order, the fill list and the streamed slot
  contents) over a random run that interleaves gaps with prefetches, and a
  gap after a correct prediction streams nothing.
* A decode stack with prefetch on gives the same outputs as the oracle
  (every selected expert is resident when the GEMMs read it), eagerly and
  replayed from a CUDA graph, and actually prefetches; with prefetch off the
  stack's slot maps are the reference policy's (the default path issues no
  prefetch call).
"""

import random

import pytest
import torch

from oracle import moe as omoe
from oracle import routing as orouting
from oracle.slot_policy import PROBATION, PROTECTED, SlotPolicyModel
from sluice_b200 import configs, synth
from sluice_b200.layer import MoEDecodeStack
from sluice_b200.offloader import ExpertStreamOffloader
from test_moe_gpu import assert_moe_close
from test_slots_gpu import _payload_params

pytestmark = pytest.mark.gpu


def _compare(cache, model, step):
    snap = cache.snapshot()
    assert snap["expert_map"] == model.expert_map, step
    assert snap["expert_in_slot"] == model.expert_in_slot, step
    assert snap["probation"] == model.segment_order(PROBATION), step
    assert snap["protected"] == model.segment_order(PROTECTED), step


def test_prefetch_planner_matches_oracle_and_streams():
    G = L = 64
    S = 24
    off = ExpertStreamOffloader(S, protect_frac=0.5, fast_hit=True)
    w13, w2 = _payload_params(L)
    cache = off.install_layer(w13, w2, device="cuda")
    model = SlotPolicyModel(S, list(range(G)), L, 0.5, True)
    rng = random.Random(7)
    hot = list(range(12))
    prefetched = 0
    for step in range(80):
        ids = [rng.choice(hot) if rng.random() < 0.5 else rng.randrange(G) for _ in range(12)]
        ids_t = torch.tensor(ids, dtype=torch.int32, device="cuda")
        if step % 3 == 1:
            n = rng.choice([1, 2, 4, 8])
            fills = model.prefetch(ids, n)
            cache.prefetch(ids_t, n)
        else:
            fills = model.gap(ids)
            cache.plan(ids_t)
        cache.stream()
        torch.cuda.synchronize()
        cache.check()
        _compare(cache, model, step)
        snap = cache.snapshot()
        assert snap["fills"] == fills, step
        prefetched += len(fills) if step % 3 == 1 else 0
        # slot contents: every resident slot holds its expert's rows
        eis = torch.tensor(model.expert_in_slot)
        res = (eis >= 0).nonzero().flatten()
        assert torch.equal(cache.w13[res.cuda()].cpu(), w13[eis[res]]), step
        assert torch.equal(cache.w2[res.cuda()].cpu(), w2[eis[res]]), step
    assert prefetched > 0
    assert cache.counters()["prefetches"] == model.prefetches
    # a correct prediction: the next gap on those ids streams nothing new
    ids = list(range(40, 46))
    ids_t = torch.tensor(ids, dtype=torch.int32, device="cuda")
    assert model.prefetch(ids, 8)
    cache.prefetch(ids_t, 8)
    cache.stream()
    assert model.gap(ids) == []
    cache.plan(ids_t)
    torch.cuda.synchronize()
    assert cache.header()["fill_count"] == 0
    _compare(cache, model, "after")


def test_stack_with_prefetch_matches_oracle_eager_and_replayed():
    cfg = configs.V2_LITE
    layers, T, seed = 3, 8, 11
    stack = MoEDecodeStack(cfg, slots=48, seed=seed, num_layers=layers, prefetch=4)
    assert all(l.prefetch_next is not None for l in stack.layers[:-1])
    w = [synth.layer_weights(cfg, li, seed, device="cuda") for li in range(layers)]
    w = [(a.cpu(), b.cpu()) for a, b in w]
    sh = [tuple(t.cpu() for t in synth.shared_weights(cfg, li, seed, device="cuda"))
          for li in range(layers)]
    rc = cfg.routing
    tokens = synth.TokenStream(cfg.hidden, T, seed=12, reuse=0.3)

    def check(x, out):
        torch.cuda.synchronize()
        stack.check()
        h = x
        for li, layer in enumerate(stack.layers):
            logits = layer.last_logits.cpu()
            tw, ti = orouting.grouped_topk(logits, rc.topk, rc.renormalize)
            assert torch.equal(ti, layer.last_ids.cpu())
            routed = omoe.fused_experts(h, w[li][0], w[li][1], tw, ti)
            shared = sum(omoe.expert_mlp(h, sh[li][0][i], sh[li][1][i]).float()
                         for i in range(cfg.n_shared)).to(torch.bfloat16)
            h = h + omoe.layer_output(routed, shared)
            # every selected expert is resident after the step
            emap = layer.cache.expert_map.cpu()
            assert (emap[ti.flatten().long()] >= 0).all()
        assert_moe_close(out, h)

    for _ in range(3):
        x = tokens.next()
        check(x, stack.step(x.cuda()))
    stack.capture(tokens=T)
    for _ in range(3):
        x = tokens.next()
        check(x, stack.replay(x.cuda()))
    assert stack.stats()["prefetches"] > 0


def test_stack_without_prefetch_follows_the_reference_policy():
    cfg = configs.V2_LITE
    stack = MoEDecodeStack(cfg, slots=48, seed=13, num_layers=2)
    assert all(l.prefetch_next is None for l in stack.layers)
    models = [SlotPolicyModel(48, list(range(cfg.num_experts)), cfg.num_experts, 0.5, True)
              for _ in stack.layers]
    tokens = synth.TokenStream(cfg.hidden, 8, seed=14)
    for step in range(4):
        stack.step(tokens.next().cuda())
        torch.cuda.synchronize()
        for layer, m in zip(stack.layers, models):
            m.gap(layer.last_ids.cpu().flatten().tolist())
            assert layer.cache.expert_map.cpu().tolist() == m.expert_map, step
    assert stack.stats()["prefetches"] == 0
