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


def test_fused_mla_decode_matches_the_pytorch_attention():
    """sl_mla_decode (the harness's one-launch attention) against the same
    attention in PyTorch ops, on caches filled by earlier steps: the layer's
    output within bf16 tolerance and the written cache row equal."""
    from sluice_b200.harness import DecoderHarness

    dcfg = replace(V2_LITE_DECODER, num_layers=2, vocab=2048)
    h = DecoderHarness(dcfg, lambda li, x: torch.zeros_like(x), batch=3, max_len=40, seed=4,
                       fused_attention=False)
    g = torch.Generator(device="cuda").manual_seed(5)
    ids = torch.randint(0, 2048, (3,), device="cuda", generator=g)
    for _ in range(9):                      # fill positions 0..8 with the PyTorch path
        ids = h.step(ids)
    h.pos[1] = 3                            # ragged: sequences at different positions
    h.pos[2] = 0                            # a sequence at its first position
    x = torch.randn(3, dcfg.hidden, device="cuda", generator=g).to(torch.bfloat16)
    freqs = h.freqs[h.pos]
    mask = torch.zeros(3, 1, h.max_len, dtype=torch.bfloat16, device="cuda")
    mask.masked_fill_((h._ar[None, :] > h.pos[:, None])[:, None, :], float("-inf"))
    for li in range(dcfg.num_layers):
        before = h.cache[li].clone()
        h.fused_attention = False
        ref = h._attention(li, x, mask, freqs)
        ref_cache = h.cache[li].clone()
        h.cache[li].copy_(before)
        h.fused_attention = True
        got = h._attention(li, x, mask, freqs)
        torch.cuda.synchronize()
        err = (got.float() - ref.float()).abs().max().item()
        assert err <= 2e-2 * ref.float().abs().max().item() + 1e-3, (li, err)
        rows = torch.arange(3, device="cuda")
        new, old = h.cache[li][rows, h.pos].float(), ref_cache[rows, h.pos].float()
        assert (new - old).abs().max().item() <= 1e-2 * old.abs().max().item(), li


def test_fused_add_rmsnorm_matches_pytorch():
    """sl_add_rmsnorm (the harness's residual add + RMSNorm) against the same
    two PyTorch ops: the updated residual bit-equal, the normed rows within
    one bf16 rounding; without a delta, the residual untouched."""
    from sluice_b200._lib import check, lib, ptr

    g = torch.Generator(device="cuda").manual_seed(11)
    for rows, H in ((8, 2048), (3, 7168), (1, 512)):
        h = torch.randn(rows, H, device="cuda", generator=g).to(torch.bfloat16)
        d = torch.randn(rows, H, device="cuda", generator=g).to(torch.bfloat16)
        w = (1 + 0.1 * torch.randn(H, device="cuda", generator=g)).to(torch.bfloat16)
        ref_h = h + d
        ref = torch.nn.functional.rms_norm(ref_h, (H,), w, 1e-6)
        got_h, out = h.clone(), torch.empty_like(h)
        stream = torch.cuda.current_stream().cuda_stream
        check(lib().sl_add_rmsnorm(ptr(got_h), ptr(d), ptr(w), 1e-6, ptr(out), rows, H, stream),
              "sl_add_rmsnorm")
        torch.cuda.synchronize()
        assert torch.equal(got_h, ref_h)
        err = (out.float() - ref.float()).abs()
        assert (err <= 1e-2 * ref.float().abs() + 1e-2).all(), err.max().item()
        plain = torch.empty_like(h)
        check(lib().sl_add_rmsnorm(ptr(h), None, ptr(w), 1e-6, ptr(plain), rows, H, stream),
              "sl_add_rmsnorm")
        torch.cuda.synchronize()
        ref2 = torch.nn.functional.rms_norm(h, (H,), w, 1e-6)
        assert ((plain.float() - ref2.float()).abs() <= 1e-2 * ref2.float().abs() + 1e-2).all()


def test_skinny_linear_matches_pytorch():
    """sl_linear_small (the harness's decode-batch projections) against an
    fp32 product of the same bf16 operands, within one bf16 rounding."""
    from sluice_b200._lib import check, lib, ptr

    g = torch.Generator(device="cuda").manual_seed(13)
    for T, K, N in ((1, 2048, 3648), (2, 2048, 2048), (1, 2048, 100), (4, 4096, 301),
                    (3, 10944, 64), (4, 520, 7)):
        x = torch.randn(T, K, device="cuda", generator=g).to(torch.bfloat16)
        w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
        y = torch.empty(T, N, dtype=torch.bfloat16, device="cuda")
        check(lib().sl_linear_small(ptr(x), T, K, ptr(w), N, ptr(y),
                                    torch.cuda.current_stream().cuda_stream), "sl_linear_small")
        torch.cuda.synchronize()
        ref = x.float() @ w.float().t()
        err = (y.float() - ref).abs()
        assert (err <= 1e-2 * ref.abs() + 1e-2 * ref.abs().max()).all(), (T, K, N, err.max().item())
