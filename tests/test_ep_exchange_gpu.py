"""The expert-parallel exchange kernels on ONE GPU, through the C ABI.

Rank 0 of a two-rank world runs against a peer whose receive buffer and
signal words are ordinary local buffers: the test plays the peer by filling
its rows and raising its signal BEFORE the launch, so the kernel never waits
on another launch. Checked: the rows pushed into the peer's buffer, the
peer's signal, the unpacked / summed outputs, the alternation of the two
receive halves across calls, and the bounded wait — a signal that nothing
raises ends the call with SL_ERR_TIMEOUT and the context stays usable.
"""

import ctypes

import pytest
import torch

from sluice_b200 import _lib
from sluice_b200.ep import pack_routing

pytestmark = pytest.mark.gpu

T, H, K = 4, 256, 8


def _vp(*ptrs):
    return (ctypes.c_void_p * len(ptrs))(*ptrs)


def _rows(seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    tw = torch.rand(T, K, generator=g)
    ti = torch.randint(0, 64, (T, K), generator=g, dtype=torch.int32)
    return x.cuda(), tw.cuda(), ti.cuda()


def test_dispatch_pushes_signals_and_unpacks():
    L = _lib.lib()
    nd = L.sl_ep_dispatch_recv_bytes(2, T, H, K)
    row = 2 * H + 8 * K
    assert nd == 2 * 2 * T * row
    mine, peer = (torch.zeros(nd, dtype=torch.uint8, device="cuda") for _ in range(2))
    my_sig, peer_sig = (torch.zeros(16, dtype=torch.int32, device="cuda") for _ in range(2))
    book = torch.zeros(4, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    recv = _vp(mine.data_ptr(), peer.data_ptr())
    sig = _vp(my_sig.data_ptr(), peer_sig.data_ptr())
    half = 2 * T * row
    stream = torch.cuda.current_stream().cuda_stream
    for call, epoch in enumerate((1, 2)):
        x0, tw0, ti0 = _rows(10 + call)
        x1, tw1, ti1 = _rows(20 + call)
        h = (epoch & 1) * half
        mine[h + T * row:h + 2 * T * row] = pack_routing(x1, tw1, ti1).view(-1)
        my_sig[0 * 8 + 1] = epoch  # the peer has pushed this call's rows
        xo = torch.empty(2 * T, H, dtype=torch.bfloat16, device="cuda")
        wo = torch.empty(2 * T, K, dtype=torch.float32, device="cuda")
        io = torch.empty(2 * T, K, dtype=torch.int32, device="cuda")
        packed = pack_routing(x0, tw0, ti0)  # what the kernel must push
        _lib.check(L.sl_ep_dispatch(x0.data_ptr(), tw0.data_ptr(), ti0.data_ptr(), T, H, K, 0,
                                    2, recv, sig, book.data_ptr(), xo.data_ptr(),
                                    wo.data_ptr(), io.data_ptr(), status.data_ptr(), stream),
                   "dispatch")
        torch.cuda.synchronize()
        assert status.item() == _lib.SL_OK
        assert torch.equal(xo, torch.cat([x0, x1]))
        assert torch.equal(wo, torch.cat([tw0, tw1]))
        assert torch.equal(io, torch.cat([ti0, ti1]))
        assert torch.equal(peer[h:h + T * row], packed.view(-1))
        assert peer_sig[0].item() == epoch
        assert book[0].item() == 8 * epoch


def test_combine_sums_in_rank_order():
    L = _lib.lib()
    nc = L.sl_ep_combine_recv_bytes(2, T, H)
    assert nc == 2 * 2 * T * H * 4
    mine, peer = (torch.zeros(nc, dtype=torch.uint8, device="cuda") for _ in range(2))
    my_sig, peer_sig = (torch.zeros(16, dtype=torch.int32, device="cuda") for _ in range(2))
    book = torch.zeros(4, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    recv = _vp(mine.data_ptr(), peer.data_ptr())
    sig = _vp(my_sig.data_ptr(), peer_sig.data_ptr())
    slot = T * H * 4
    stream = torch.cuda.current_stream().cuda_stream
    g = torch.Generator().manual_seed(5)
    for epoch in (1, 2, 3):
        part = torch.randn(2 * T, H, generator=g).cuda()
        from_peer = torch.randn(T, H, generator=g).cuda()
        h = (epoch & 1) * 2 * slot
        mine[h + slot:h + 2 * slot] = from_peer.view(torch.uint8).view(-1)
        my_sig[1 * 8 + 1] = epoch
        out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
        # the third call folds in the decoder's residual add
        res = torch.randn(T, H, generator=g).to(torch.bfloat16).cuda() if epoch == 3 else None
        _lib.check(L.sl_ep_combine(part.data_ptr(), T, H, 0, 2, recv, sig, book.data_ptr(),
                                   None if res is None else res.data_ptr(), out.data_ptr(),
                                   status.data_ptr(), stream), "combine")
        torch.cuda.synchronize()
        assert status.item() == _lib.SL_OK
        moe = (part[:T] + from_peer).to(torch.bfloat16)
        assert torch.equal(out, moe if res is None else res + moe)
        assert torch.equal(peer[h:h + slot], part[T:].contiguous().view(torch.uint8).view(-1))
        assert peer_sig[8].item() == epoch
        assert book[1].item() == 8 * epoch


def test_wait_on_silent_peer_times_out():
    L = _lib.lib()
    nd = L.sl_ep_dispatch_recv_bytes(2, T, H, K)
    mine, peer = (torch.zeros(nd, dtype=torch.uint8, device="cuda") for _ in range(2))
    my_sig, peer_sig = (torch.zeros(16, dtype=torch.int32, device="cuda") for _ in range(2))
    book = torch.zeros(4, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    x0, tw0, ti0 = _rows(1)
    xo = torch.empty(2 * T, H, dtype=torch.bfloat16, device="cuda")
    wo = torch.empty(2 * T, K, dtype=torch.float32, device="cuda")
    io = torch.empty(2 * T, K, dtype=torch.int32, device="cuda")
    _lib.check(L.sl_ep_dispatch(x0.data_ptr(), tw0.data_ptr(), ti0.data_ptr(), T, H, K, 0, 2,
                                _vp(mine.data_ptr(), peer.data_ptr()),
                                _vp(my_sig.data_ptr(), peer_sig.data_ptr()), book.data_ptr(),
                                xo.data_ptr(), wo.data_ptr(), io.data_ptr(), status.data_ptr(),
                                torch.cuda.current_stream().cuda_stream), "dispatch")
    torch.cuda.synchronize()
    assert status.item() == _lib.SL_ERR_TIMEOUT
    assert peer_sig[0].item() == 1  # this rank still signalled its own pushes
    assert torch.equal(xo[:T], x0)  # own rows come from the local input
    assert (torch.ones(8, device="cuda") * 2).sum().item() == 16.0  # context usable


def test_exchange_rejects_bad_arguments():
    L = _lib.lib()
    z = torch.zeros(64, dtype=torch.int32, device="cuda")
    p = z.data_ptr()
    s = torch.cuda.current_stream().cuda_stream
    recv = _vp(p, p)
    d = lambda *a: L.sl_ep_dispatch(p, p, p, *a)
    assert d(T, H, K, 2, 2, recv, recv, p, p, p, p, p, s) == _lib.SL_ERR_INVALID
    assert d(T, H, K, 0, 9, recv, recv, p, p, p, p, p, s) == _lib.SL_ERR_INVALID
    assert d(T, 100, 3, 0, 2, recv, recv, p, p, p, p, p, s) \
        in (_lib.SL_ERR_INVALID, _lib.SL_ERR_UNSUPPORTED)
    assert d(T, H, 3, 0, 2, recv, recv, p, p, p, p, p, s) == _lib.SL_ERR_UNSUPPORTED  # odd topk
    assert L.sl_ep_dispatch(p + 4, p, p, T, H, K, 0, 2, recv, recv, p, p, p, p, p, s) \
        == _lib.SL_ERR_INVALID  # hidden rows not 16-byte aligned
    assert L.sl_ep_combine(p, T, H, 0, 2, _vp(p, None), recv, p, None, p, p, s) \
        == _lib.SL_ERR_INVALID
