"""The routed expert-parallel exchange kernels on ONE GPU, through the C ABI.

Rank 0 of a two-rank world (64 experts: rank 0 owns 0..31, rank 1 owns
32..63) runs against a peer whose receive buffer and signal words are
ordinary local buffers: the test plays the peer by writing what the peer
would push and raising its signal BEFORE the launch, so the kernel never
waits on another launch. Checked: only tokens with an expert on the peer are
pushed to it (packed rows in token order, with the row count), the peer's
signal, the unpacked rows (own tokens first, then the peer's, then empty
rows with id -1), the routed combine (each received row's partial back to
its home token, sums only over the ranks a token was sent to), the
alternation of the two receive halves across calls, and the bounded wait —
a signal that nothing raises ends the call with SL_ERR_TIMEOUT and the
context stays usable.
"""

import ctypes

import pytest
import torch

from sluice_b200 import _lib

pytestmark = pytest.mark.gpu

T, H, K, G, WORLD = 4, 256, 8, 64, 2
PER = G // WORLD
HDR = 128                                   # bytes before a dispatch half's rows
ROW = (2 * H + 8 * K + 4 + 15) // 16 * 16   # hidden | weights | ids | token | pad


def _vp(*ptrs):
    return (ctypes.c_void_p * len(ptrs))(*ptrs)


def _rows(seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    tw = torch.rand(T, K, generator=g)
    ti = torch.randint(0, G, (T, K), generator=g, dtype=torch.int32)
    ti[0, :] = 3            # token 0 stays home (rank 0's experts only)
    ti[1, :] = 40           # token 1 only needs rank 1
    return x.cuda(), tw.cuda(), ti.cuda()


def _sent_to(ti, dest):
    """Tokens that own rank (world 2) sends to `dest`, in token order."""
    owners = (ti.long() // PER)
    return [t for t in range(ti.shape[0]) if bool((owners[t] == dest).any())]


def _packed(x, tw, ti, toks):
    """The rows the dispatch packs for tokens `toks` (ROW bytes each)."""
    out = torch.zeros(len(toks), ROW, dtype=torch.uint8, device=x.device)
    for i, t in enumerate(toks):
        parts = [x[t].view(torch.uint8), tw[t].contiguous().view(torch.uint8),
                 ti[t].contiguous().view(torch.uint8),
                 torch.tensor([t], dtype=torch.int32, device=x.device).view(torch.uint8)]
        row = torch.cat(parts)
        out[i, :row.numel()] = row
    return out


def _buffers(nbytes):
    mine, peer = (torch.zeros(nbytes, dtype=torch.uint8, device="cuda") for _ in range(2))
    my_sig, peer_sig = (torch.zeros(16, dtype=torch.int32, device="cuda") for _ in range(2))
    book = torch.zeros(4, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    return mine, peer, my_sig, peer_sig, book, status


def test_dispatch_routes_pushes_signals_and_unpacks():
    L = _lib.lib()
    nd = L.sl_ep_dispatch_recv_bytes(WORLD, T, H, K)
    half = HDR + WORLD * T * ROW
    assert nd == 2 * half
    mine, peer, my_sig, peer_sig, book, status = _buffers(nd)
    recv = _vp(mine.data_ptr(), peer.data_ptr())
    sig = _vp(my_sig.data_ptr(), peer_sig.data_ptr())
    stream = torch.cuda.current_stream().cuda_stream
    for call, epoch in enumerate((1, 2)):
        x0, tw0, ti0 = _rows(10 + call)
        x1, tw1, ti1 = _rows(20 + call)
        h = (epoch & 1) * half
        # what the peer (rank 1) pushes to rank 0: its tokens with an expert in 0..31
        from_peer = _sent_to(ti1, 0)
        mine[h:h + HDR] = 0
        mine[h:h + 8].view(torch.int32)[1] = len(from_peer)
        s1 = h + HDR + 1 * T * ROW
        mine[s1:s1 + len(from_peer) * ROW] = _packed(x1, tw1, ti1, from_peer).view(-1)
        my_sig[0 * 8 + 1] = epoch
        n = WORLD * T
        xo = torch.zeros(n, H, dtype=torch.bfloat16, device="cuda")
        wo = torch.full((n, K), 7.0, dtype=torch.float32, device="cuda")
        io = torch.full((n, K), 7, dtype=torch.int32, device="cuda")
        so = torch.full((n,), 7, dtype=torch.int32, device="cuda")
        _lib.check(L.sl_ep_dispatch(x0.data_ptr(), tw0.data_ptr(), ti0.data_ptr(), T, H, K, G,
                                    0, WORLD, recv, sig, book.data_ptr(), xo.data_ptr(),
                                    wo.data_ptr(), io.data_ptr(), so.data_ptr(),
                                    status.data_ptr(), stream), "dispatch")
        torch.cuda.synchronize()
        assert status.item() == _lib.SL_OK
        # pushed: only tokens with an expert on rank 1, in token order
        to_peer = _sent_to(ti0, 1)
        assert 1 in to_peer and 0 not in to_peer
        assert peer[h:h + 8].view(torch.int32)[0].item() == len(to_peer)
        s0 = h + HDR
        assert torch.equal(peer[s0:s0 + len(to_peer) * ROW].view(len(to_peer), ROW),
                           _packed(x0, tw0, ti0, to_peer))
        assert peer_sig[0].item() == epoch
        assert book[0].item() == 8 * epoch
        # unpacked: own rows, the peer's rows, empty rows
        m = len(from_peer)
        idx = torch.tensor(from_peer, dtype=torch.long, device="cuda")
        assert torch.equal(xo[:T], x0)
        assert torch.equal(xo[T:T + m], x1[idx])
        assert torch.equal(wo[:T], tw0) and torch.equal(wo[T:T + m], tw1[idx])
        assert torch.equal(io[:T], ti0) and torch.equal(io[T:T + m], ti1[idx])
        assert (io[T + m:] == -1).all() and (wo[T + m:] == 0).all()
        src = so.cpu().tolist()
        assert src[:T] == list(range(T))
        assert src[T:T + m] == [(1 << 16) | t for t in from_peer]
        assert all(v == -1 for v in src[T + m:])


def test_combine_returns_rows_home_and_sums_routed_partials():
    L = _lib.lib()
    nc = L.sl_ep_combine_recv_bytes(WORLD, T, H)
    assert nc == 2 * WORLD * T * H * 4
    mine, peer, my_sig, peer_sig, book, status = _buffers(nc)
    recv = _vp(mine.data_ptr(), peer.data_ptr())
    sig = _vp(my_sig.data_ptr(), peer_sig.data_ptr())
    slot = T * H * 4
    stream = torch.cuda.current_stream().cuda_stream
    g = torch.Generator().manual_seed(5)
    for epoch in (1, 2, 3):
        _, _, ti0 = _rows(30 + epoch)    # this rank's tokens' ids
        _, _, ti1 = _rows(40 + epoch)
        from_peer = _sent_to(ti1, 0)     # rows the dispatch gave rank 0 from rank 1
        m = len(from_peer)
        part = torch.randn(WORLD * T, H, generator=g).cuda()
        src = torch.full((WORLD * T,), -1, dtype=torch.int32)
        src[:T] = torch.arange(T, dtype=torch.int32)
        src[T:T + m] = torch.tensor([(1 << 16) | t for t in from_peer], dtype=torch.int32)
        src = src.cuda()
        # what rank 1 sends back: partials of rank 0's tokens it received
        back = torch.randn(T, H, generator=g).cuda()
        h = (epoch & 1) * WORLD * slot
        mine[h + slot:h + 2 * slot] = back.view(torch.uint8).view(-1)
        my_sig[1 * 8 + 1] = epoch
        peer[h:h + slot] = 0
        out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
        # the third call folds in the decoder's residual add
        res = torch.randn(T, H, generator=g).to(torch.bfloat16).cuda() if epoch == 3 else None
        _lib.check(L.sl_ep_combine(part.data_ptr(), src.data_ptr(), ti0.data_ptr(), T, H, K, G,
                                   0, WORLD, recv, sig, book.data_ptr(),
                                   None if res is None else res.data_ptr(), out.data_ptr(),
                                   status.data_ptr(), stream), "combine")
        torch.cuda.synchronize()
        assert status.item() == _lib.SL_OK
        went = torch.tensor([bool(((ti0[t].long() // PER) == 1).any()) for t in range(T)],
                            device="cuda")
        moe = (part[:T] + torch.where(went[:, None], back, torch.zeros_like(back))) \
            .to(torch.bfloat16)
        assert torch.equal(out, moe if res is None else res + moe)
        # each received row's partial went back to its token's row of slot 0
        pushed = peer[h:h + slot].view(torch.float32).view(T, H)
        for j, t in enumerate(from_peer):
            assert torch.equal(pushed[t], part[T + j])
        assert peer_sig[8].item() == epoch
        assert book[1].item() == 8 * epoch


def test_wait_on_silent_peer_times_out():
    L = _lib.lib()
    nd = L.sl_ep_dispatch_recv_bytes(WORLD, T, H, K)
    mine, peer, my_sig, peer_sig, book, status = _buffers(nd)
    x0, tw0, ti0 = _rows(1)
    n = WORLD * T
    xo = torch.empty(n, H, dtype=torch.bfloat16, device="cuda")
    wo = torch.empty(n, K, dtype=torch.float32, device="cuda")
    io = torch.empty(n, K, dtype=torch.int32, device="cuda")
    so = torch.empty(n, dtype=torch.int32, device="cuda")
    _lib.check(L.sl_ep_dispatch(x0.data_ptr(), tw0.data_ptr(), ti0.data_ptr(), T, H, K, G, 0,
                                WORLD, _vp(mine.data_ptr(), peer.data_ptr()),
                                _vp(my_sig.data_ptr(), peer_sig.data_ptr()), book.data_ptr(),
                                xo.data_ptr(), wo.data_ptr(), io.data_ptr(), so.data_ptr(),
                                status.data_ptr(), torch.cuda.current_stream().cuda_stream),
               "dispatch")
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
    d = lambda T_, H_, K_, G_, r, w: L.sl_ep_dispatch(p, p, p, T_, H_, K_, G_, r, w, recv, recv,
                                                      p, p, p, p, p, p, s)
    assert d(T, H, K, G, 2, 2) == _lib.SL_ERR_INVALID          # rank outside the world
    assert d(T, H, K, G, 0, 9) == _lib.SL_ERR_INVALID          # more ranks than supported
    assert d(T, 100, K, G, 0, 2) == _lib.SL_ERR_INVALID        # H not a multiple of 8
    assert d(T, H, K, 63, 0, 2) == _lib.SL_ERR_UNSUPPORTED     # experts do not shard evenly
    assert d(2048, H, K, G, 0, 2) == _lib.SL_ERR_UNSUPPORTED   # more tokens than routed
    assert L.sl_ep_dispatch(p + 4, p, p, T, H, K, G, 0, 2, recv, recv, p, p, p, p, p, p, s) \
        == _lib.SL_ERR_INVALID  # hidden rows not 16-byte aligned
    assert L.sl_ep_combine(p, p, p, T, H, K, G, 0, 2, _vp(p, None), recv, p, None, p, p, s) \
        == _lib.SL_ERR_INVALID
