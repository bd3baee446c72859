"""The peer-memory exchange's device-side bounds (bs_ep_p2p_dispatch/return)
on one GPU: a world of one rank, whose only peer is itself, so every flag the
kernels wait on is raised earlier on the same stream.

* a rank that dispatches more rows than the exchange was sized for
  (expert_offsets[E] > src_rows) sends nothing, records BS_ERR_CAPACITY in
  the status word and leaves the receive buffer untouched;
* a correctly sized call afterwards delivers every row (expert-major) and
  returns every result row to its dispatch position.
"""

import ctypes

import pytest
import torch

from blockstreamer_b200 import _lib, kernels

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


class _OneRankExchange:
    def __init__(self, E, H, src_rows):
        self.lib = _lib.load()
        self.E, self.H, self.src, self.cap = E, H, src_rows, src_rows
        self.nbytes = self.lib.bs_ep_p2p_bytes(1, E, H, self.cap, self.src)
        base, handle = ctypes.c_void_p(), (ctypes.c_char * 64)()
        _lib.call("bs_ep_p2p_alloc", self.nbytes, ctypes.byref(base), handle)
        self.base = base.value
        self.bases = torch.tensor([self.base], dtype=torch.int64, device=DEV)
        ro, yo = ctypes.c_size_t(), ctypes.c_size_t()
        _lib.call("bs_ep_p2p_layout", 1, E, H, self.cap, self.src, ctypes.byref(ro), ctypes.byref(yo))
        from blockstreamer_b200.expert_parallel import _DeviceBytes
        raw = torch.as_tensor(_DeviceBytes(self.base, self.nbytes), device=DEV)
        self.recv = raw[ro.value: ro.value + self.cap * H * 2].view(torch.bfloat16).view(self.cap, H)
        self.yback = raw[yo.value: yo.value + self.src * H * 2].view(torch.bfloat16).view(self.src, H)
        self.local = torch.zeros(E + 1, dtype=torch.int32, device=DEV)

    def dispatch(self, x, d):
        st = torch.cuda.current_stream().cuda_stream
        return self.lib.bs_ep_p2p_dispatch(
            ctypes.c_void_p(x.data_ptr()), self.H, ctypes.c_void_p(d.expert_offsets.data_ptr()),
            ctypes.c_void_p(d.token_of_row.data_ptr()), ctypes.c_void_p(self.base),
            ctypes.c_void_p(self.bases.data_ptr()), 1, self.E, 0, self.cap, self.src,
            ctypes.c_void_p(self.local.data_ptr()), ctypes.c_void_p(st))

    def give_back(self, y):
        st = torch.cuda.current_stream().cuda_stream
        return self.lib.bs_ep_p2p_return(ctypes.c_void_p(y.data_ptr()), self.H, ctypes.c_void_p(self.base),
                                         ctypes.c_void_p(self.bases.data_ptr()), 1, self.E, 0, self.cap,
                                         self.src, ctypes.c_void_p(st))

    def free(self):
        torch.cuda.synchronize()
        _lib.call("bs_ep_p2p_free", ctypes.c_void_p(self.base))


def _tokens(T, E, k, H, seed):
    g = torch.Generator().manual_seed(seed)
    idx = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).to(torch.int32).to(DEV)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16).to(DEV)
    return idx, x


def test_exchange_rejects_more_rows_than_src_rows_without_writing():
    T, E, k, H = 96, 4, 2, 256
    assert kernels.device_status(clear=True) == 0
    ex = _OneRankExchange(E, H, src_rows=T * k - 1)   # one row too few
    try:
        ex.recv.fill_(7.0)
        ex.yback.fill_(5.0)
        idx, x = _tokens(T, E, k, H, 1)
        d = kernels.dispatch(idx, E)
        assert ex.dispatch(x, d) == _lib.BS_OK          # the size error is found on the device
        assert kernels.device_status(clear=True) == _lib.BS_ERR_CAPACITY
        assert bool((ex.recv == 7.0).all()), "rows were written past the exchange's size"
        assert int(ex.local[-1]) == 0                    # the peers saw zero rows from this rank
        y = torch.randn(ex.cap, H, device=DEV).to(torch.bfloat16)
        assert ex.give_back(y) == _lib.BS_OK
        torch.cuda.synchronize()
        assert bool((ex.yback == 5.0).all())
        assert kernels.device_status(clear=True) == 0
    finally:
        ex.free()


def test_exchange_single_rank_round_trip():
    T, E, k, H = 96, 4, 2, 256
    assert kernels.device_status(clear=True) == 0
    ex = _OneRankExchange(E, H, src_rows=T * k)
    try:
        idx, x = _tokens(T, E, k, H, 2)
        d = kernels.dispatch(idx, E, x)
        for _ in range(2):   # the second call checks the epoch bookkeeping
            ex.recv.zero_()
            assert ex.dispatch(x, d) == _lib.BS_OK
            torch.cuda.synchronize()
            assert kernels.device_status(clear=True) == 0
            assert torch.equal(ex.local, d.expert_offsets)
            assert torch.equal(ex.recv, d.x_perm)          # one rank: recv is the dispatch order
            y = torch.randn(ex.cap, H, device=DEV).to(torch.bfloat16)
            assert ex.give_back(y) == _lib.BS_OK
            torch.cuda.synchronize()
            assert kernels.device_status(clear=True) == 0
            assert torch.equal(ex.yback, y)
    finally:
        ex.free()
