"""sl_fused_experts_noalloc: fused experts for callers that cannot allocate.

A caller that binds the C ABI directly, with no caching allocator, or a
serving process whose HBM is already claimed by its own pool, cannot hand
sl_fused_experts a workspace. The no-alloc entry point takes its scratch from
a fixed 32 MiB device array instead. This test calls both entry points through
the C ABI on the same inputs, twice in a row with different inputs (the shared
scratch keeps the first call's contents), and checks that:

* the two results are bit-identical (both run the same deterministic kernels,
  so any difference would be stale scratch leaking into the second call);
* both are within the fused-experts tolerance of the CPU oracle (2e-2
  relative, bf16, elementwise bound scaled by the output magnitude);
* every refused call (fp8 weights, a problem beyond the scratch, a null
  pointer) leaves the caller's status word untouched and launches nothing.

It lives in its own file, collected last, and works alone in a fresh process
or after the other tests.
"""

import pytest
import torch

from oracle import moe as omoe
from sluice_b200 import _lib

pytestmark = pytest.mark.gpu
RTOL = 2e-2


def _case(seed, T=8, H=2048, I=1408, S=48, E=64, k=6, n_sh=2):
    g = torch.Generator().manual_seed(seed)
    hs = torch.randn(T, H, generator=g).to(torch.bfloat16)
    w13 = (torch.randn(S, 2 * I, H, generator=g) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn(S, H, I, generator=g) * 0.02).to(torch.bfloat16)
    sh13 = (torch.randn(n_sh, 2 * I, H, generator=g) * 0.02).to(torch.bfloat16)
    sh2 = (torch.randn(n_sh, H, I, generator=g) * 0.02).to(torch.bfloat16)
    emap = torch.full((E,), -1, dtype=torch.int32)
    perm = torch.randperm(E, generator=g)
    emap[perm[:S]] = torch.randperm(S, generator=g).to(torch.int32)
    ti = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).to(torch.int32)
    tw = torch.rand(T, k, generator=g).float()
    cpu = dict(hs=hs, w13=w13, w2=w2, sh13=sh13, sh2=sh2, emap=emap, ti=ti, tw=tw)
    c = lambda t: t.cuda().contiguous()
    d = {n: c(t) for n, t in cpu.items()}
    d.update(T=T, H=H, I=I, S=S, E=E, k=k, n_sh=n_sh, cpu=cpu)
    return d


def _oracle(d):
    c = d["cpu"]
    routed = omoe.fused_experts(c["hs"], c["w13"], c["w2"], c["tw"], c["ti"], c["emap"])
    shared = sum(omoe.expert_mlp(c["hs"], c["sh13"][i], c["sh2"][i]).float()
                 for i in range(d["n_sh"])).to(torch.bfloat16)
    return omoe.layer_output(routed, shared, 1.0)


def _with_workspace(L, d, stream):
    out = torch.empty(d["T"], d["H"], dtype=torch.bfloat16, device="cuda")
    nbytes = L.sl_fused_experts_workspace_bytes(d["T"], d["k"], d["H"], d["I"], d["S"],
                                                d["n_sh"])
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    rc = L.sl_fused_experts(d["hs"].data_ptr(), d["T"], d["H"], d["I"], d["w13"].data_ptr(),
                            d["w2"].data_ptr(), d["S"], 0, d["tw"].data_ptr(),
                            d["ti"].data_ptr(), d["k"], d["emap"].data_ptr(), d["E"],
                            d["sh13"].data_ptr(), d["sh2"].data_ptr(), d["n_sh"], 1.0,
                            out.data_ptr(), ws.data_ptr(), nbytes, stream)
    assert rc == _lib.SL_OK
    return out, ws


def _no_alloc(L, d, stream, status, weight_dtype=0, hidden=True):
    out = torch.empty(d["T"], d["H"], dtype=torch.bfloat16, device="cuda")
    rc = L.sl_fused_experts_noalloc(d["hs"].data_ptr() if hidden else None, d["T"], d["H"],
                                    d["I"], d["w13"].data_ptr(), d["w2"].data_ptr(), d["S"],
                                    weight_dtype, d["tw"].data_ptr(), d["ti"].data_ptr(),
                                    d["k"], d["emap"].data_ptr(), d["E"],
                                    d["sh13"].data_ptr(), d["sh2"].data_ptr(), d["n_sh"], 1.0,
                                    out.data_ptr(), status.data_ptr(), stream)
    return rc, out


def _assert_close(got, ref):
    got, ref = got.float().cpu(), ref.float().cpu()
    assert torch.isfinite(got).all()
    err = (got - ref).abs()
    assert (err <= RTOL * ref.abs().max() + RTOL * ref.abs()).all(), err.max()


def test_no_alloc_matches_workspace_entry_point_twice_in_a_row():
    L = _lib.lib()
    torch.cuda.init()
    stream = torch.cuda.current_stream().cuda_stream
    status = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    # the second case is smaller (fewer tokens, fewer slots): rows the first
    # call left in the scratch must not reach its result
    for seed, kw in ((101, {}), (202, dict(T=3, S=40))):
        d = _case(seed, **kw)
        ref, ws = _with_workspace(L, d, stream)
        status.fill_(-1)
        rc, got = _no_alloc(L, d, stream, status)
        assert rc == _lib.SL_OK, _lib.status_text(rc)
        torch.cuda.synchronize()
        assert int(ws[:4].view(torch.int32)[0].item()) == _lib.SL_OK
        assert int(status.item()) == _lib.SL_OK
        assert torch.equal(got.view(torch.int16), ref.view(torch.int16)), \
            (got.float() - ref.float()).abs().max()
        oracle = _oracle(d)
        _assert_close(ref, oracle)
        _assert_close(got, oracle)


def test_no_alloc_refusals_launch_nothing():
    L = _lib.lib()
    stream = torch.cuda.current_stream().cuda_stream
    status = torch.full((1,), 77, dtype=torch.int32, device="cuda")
    d = _case(303, T=2)
    # fp8 weights are not served by this entry point
    rc, _ = _no_alloc(L, d, stream, status, weight_dtype=_lib.WEIGHTS_FP8_BLOCK128)
    assert rc == _lib.SL_ERR_UNSUPPORTED
    # a null input
    rc, _ = _no_alloc(L, d, stream, status, hidden=False)
    assert rc == _lib.SL_ERR_INVALID
    # a problem larger than the scratch
    need = L.sl_fused_experts_workspace_bytes(4096, 8, 7168, 2048, 256, 1)
    assert need > (32 << 20)
    rc = L.sl_fused_experts_noalloc(None, 4096, 7168, 2048, None, None, 256, 0, None, None,
                                    8, None, 256, None, None, 1, 1.0, None,
                                    status.data_ptr(), None)
    assert rc == _lib.SL_ERR_NO_SCRATCH
    assert b"32 MiB" in L.sl_status_string(rc)
    torch.cuda.synchronize()
    assert int(status.item()) == 77  # never written by a refused call
