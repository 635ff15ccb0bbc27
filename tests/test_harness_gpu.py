"""The decoder harness around the offloaded MoE layers (the bench's default
workload): a captured decode step replays the eager step exactly (same
greedy ids, same slot-cache statistics) and its MoE layers stream experts."""

import pytest
import torch
from dataclasses import replace

from sluice_b200 import configs
from sluice_b200.harness import V2_LITE_DECODER, OffloadedDecoder
from sluice_b200.layer import MoEDecodeStack

pytestmark = pytest.mark.gpu


def _decoder(layers=3, slots=40, batch=4, seed=3):
    dcfg = replace(V2_LITE_DECODER, num_layers=1 + layers, vocab=4096)
    stack = MoEDecodeStack(configs.V2_LITE, slots=slots, seed=seed, num_layers=layers)
    return OffloadedDecoder(dcfg, stack, batch, 64, seed)


def test_captured_decode_step_replays_the_eager_step():
    a, b = _decoder(), _decoder()
    b.capture()
    # the same warm-up step capture runs first (then rewinds the position)
    a._step()
    a.model.pos.sub_(1)
    a._ids.zero_()
    g = torch.Generator().manual_seed(9)
    prompt = torch.randint(0, 4096, (12, 4), generator=g).cuda()
    for p in range(prompt.shape[0]):
        a._ids.copy_(prompt[p])
        ids_a = a._step()
        ids_b = b.replay(prompt[p])
        torch.cuda.synchronize()
        assert torch.equal(ids_a, ids_b), p
    for t in range(8):
        ids_a = a._step()
        ids_b = b.replay()
        torch.cuda.synchronize()
        assert torch.equal(ids_a, ids_b), t
    a.check()
    b.check()
    assert a.stats() == b.stats()
    assert b.stats()["fills"] > 0
    assert int(b.model.pos[0]) == 20
