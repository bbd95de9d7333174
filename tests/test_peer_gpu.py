"""The NVLink peer-memory exchange (libmuda_peer, mb200_peer.h) on one GPU.

Two exchange buffers on the same device stand in for two ranks.  The kernel never
waits on another kernel here: a peer's announcement is either written from the host
before the call (the pull then finds it at once) or never written, so that the
bounded wait runs out (about one second), records the peer in the status word and
leaves the context usable.  The multi-GPU path itself runs in the distributed SpMV
bench, whose result is checked against the NCCL exchange.
"""

import ctypes as C
import time

import numpy as np
import pytest

from muda_b200 import capi

pytestmark = pytest.mark.gpu


class _Raw:
    """A torch view of raw device memory (CUDA array interface)."""

    def __init__(self, ptr: int, n: int, typestr: str):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr,
                                         "data": (ptr, False), "version": 3}


def _view(torch, ptr, n, typestr="<f4"):
    return torch.as_tensor(_Raw(ptr, n, typestr), device="cuda")


def _alloc(L, count):
    base, handle = C.c_void_p(), (C.c_ubyte * capi.MB200_PEER_HANDLE_BYTES)()
    assert L.mb200PeerAlloc(count, C.byref(base), handle) == 0
    assert any(bytes(handle))
    return base


def _buffer(L, base, count, epoch):
    return int(L.mb200PeerBuffer(base, count, epoch))


@pytest.mark.parametrize("block", [1000, 1001])
def test_single_rank_copies_own_block(cuda, built, block):
    torch = cuda
    L = capi.peer()
    base = _alloc(L, block)
    x = torch.arange(block, dtype=torch.float32, device="cuda") + 0.5
    bases = (C.c_void_p * 1)(base)
    for epoch in (1, 2):
        stream = torch.cuda.current_stream().cuda_stream
        assert L.mb200PeerAllgather(bases, 1, 0, block, block, epoch, C.c_void_p(x.data_ptr()),
                                    C.c_void_p(stream)) == 0
        got = _view(torch, _buffer(L, base, block, epoch), block).clone()
        torch.cuda.synchronize()
        assert torch.equal(got, x)
    st = C.c_uint(7)
    assert L.mb200PeerTakeStatus(base, C.byref(st)) == 0 and st.value == 0
    assert L.mb200PeerFree(base) == 0


@pytest.mark.parametrize("block", [8192, 4099])
def test_pull_after_announcement(cuda, built, block):
    """Rank 0 of two: rank 1's announcement of epoch 1 is already in rank 0's header,
    so the pull copies rank 1's block at once (16-byte path for block % 4 == 0)."""
    torch = cuda
    L = capi.peer()
    count = 2 * block
    own, peer = _alloc(L, count), _alloc(L, count)
    data = torch.linspace(-3.0, 7.0, block, dtype=torch.float32, device="cuda")
    _view(torch, _buffer(L, peer, count, 1) + block * 4, block).copy_(data)
    _view(torch, own.value + 4, 1, "<u4").fill_(1)  # header word 1: rank 1 announced epoch 1
    x0 = torch.full((block,), 2.25, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    bases = (C.c_void_p * 2)(own, peer)
    stream = torch.cuda.current_stream().cuda_stream
    assert L.mb200PeerAllgather(bases, 2, 0, count, block, 1, C.c_void_p(x0.data_ptr()),
                                C.c_void_p(stream)) == 0
    full = _view(torch, _buffer(L, own, count, 1), count).clone()
    torch.cuda.synchronize()
    assert torch.equal(full[:block], x0)
    assert torch.equal(full[block:], data)
    # rank 0 announced epoch 1 into rank 1's header, word 0
    assert int(_view(torch, peer.value, 1, "<u4").item()) == 1
    st = C.c_uint(7)
    assert L.mb200PeerTakeStatus(own, C.byref(st)) == 0 and st.value == 0
    for b in (own, peer):
        assert L.mb200PeerFree(b) == 0


def test_wait_runs_out_and_reports(cuda, built):
    """Nothing announces rank 1: the wait ends after about a second with bit 1 set in
    the status word, rank 1's block is left untouched and the device stays usable."""
    torch = cuda
    L = capi.peer()
    block = 4096
    count = 2 * block
    own, peer = _alloc(L, count), _alloc(L, count)
    x0 = torch.ones(block, dtype=torch.float32, device="cuda")
    bases = (C.c_void_p * 2)(own, peer)
    stream = torch.cuda.current_stream().cuda_stream
    torch.cuda.synchronize()
    t0 = time.monotonic()
    assert L.mb200PeerAllgather(bases, 2, 0, count, block, 1, C.c_void_p(x0.data_ptr()),
                                C.c_void_p(stream)) == 0
    st = C.c_uint(0)
    assert L.mb200PeerTakeStatus(own, C.byref(st)) == 0
    waited = time.monotonic() - t0
    assert st.value == 1 << 1
    assert 0.5 < waited < 30.0
    full = _view(torch, _buffer(L, own, count, 1), count).cpu().numpy()
    np.testing.assert_array_equal(full[:block], 1.0)
    np.testing.assert_array_equal(full[block:], 0.0)
    # the context is still usable and the status word was cleared
    assert float(torch.ones(4, device="cuda").sum().item()) == 4.0
    assert L.mb200PeerTakeStatus(own, C.byref(st)) == 0 and st.value == 0
    for b in (own, peer):
        assert L.mb200PeerFree(b) == 0


def test_argument_errors(cuda, built):
    L = capi.peer()
    base = _alloc(L, 16)
    bases = (C.c_void_p * 1)(base)
    x = C.c_void_p(base.value + capi.MB200_PEER_HEADER_BYTES)
    assert L.mb200PeerAllgather(bases, 1, 0, 16, 16, 0, x, None) == capi.MB200_PEER_INVALID_VALUE
    assert L.mb200PeerAllgather(bases, 1, 1, 16, 16, 1, x, None) == capi.MB200_PEER_INVALID_VALUE
    assert L.mb200PeerAllgather(bases, 1, 0, 16, 17, 1, x, None) == capi.MB200_PEER_INVALID_VALUE
    assert L.mb200PeerAllgather(bases, 33, 0, 16, 16, 1, x, None) == capi.MB200_PEER_INVALID_VALUE
    assert L.mb200PeerAlloc(0, C.byref(C.c_void_p()), (C.c_ubyte * 64)()) == \
        capi.MB200_PEER_INVALID_VALUE
    assert L.mb200PeerFree(base) == 0
