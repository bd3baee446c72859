"""The allocation-free dispatch entry point (bs_dispatch_noalloc).

Callers that cannot allocate device memory where they dispatch tokens
(serving loops that must not stall on the synchronization cudaMalloc implies,
runtimes whose pools own all device memory, or ctypes/cgo/JNI hosts without
an allocator) use this entry point: its scratch lives in a fixed device array
of the library.  These tests call it through the C ABI and check it against
bs_dispatch (the workspace form) on two calls in a row — the second call must
not be affected by what the first left in the shared array.  This file sorts
last so that a run stopping at the first failure has run every other test.
"""

import ctypes

import pytest
import torch

from blockstreamer_b200 import _lib

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _run(fn, idx, E, x, workspace=None):
    T, k = idx.shape
    S = T * k
    H = x.shape[1]
    off = torch.full((E + 1,), -7, dtype=torch.int32, device=DEV)
    ros = torch.full((S,), -7, dtype=torch.int32, device=DEV)
    tor = torch.full((S,), -7, dtype=torch.int32, device=DEV)
    xp = torch.zeros(S, H, dtype=x.dtype, device=DEV)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    dt = _lib.BS_I32 if idx.dtype == torch.int32 else _lib.BS_I64
    if fn == "bs_dispatch":
        _lib.call(fn, _p(idx), dt, T, k, E, _p(x), H, _p(off), _p(ros), _p(tor), _p(xp),
                  _p(workspace), workspace.numel(), st)
    else:
        _lib.call(fn, _p(idx), dt, T, k, E, _p(x), H, _p(off), _p(ros), _p(tor), _p(xp), st)
    torch.cuda.synchronize()
    return off.cpu(), ros.cpu(), tor.cpu(), xp.cpu()


def _case(T, E, k, H, seed):
    g = torch.Generator().manual_seed(seed)
    idx = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).to(torch.int32)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    return idx.to(DEV), x.to(DEV)


def test_noalloc_dispatch_matches_workspace_dispatch_twice():
    lib = _lib.load()
    # a large call, then a smaller one that leaves stale counts beyond its own blocks
    for (T, E, k, H, seed) in [(8192, 128, 4, 256, 1), (1000, 32, 2, 64, 2)]:
        idx, x = _case(T, E, k, H, seed)
        ws_bytes = lib.bs_dispatch_workspace_bytes(T, k, E)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=DEV)
        want = _run("bs_dispatch", idx, E, x, ws)
        got = _run("bs_dispatch_noalloc", idx, E, x)
        for a, b in zip(got, want):
            assert torch.equal(a, b)
        assert int(got[0][-1]) == T * k


def test_noalloc_dispatch_rejects_sizes_beyond_its_scratch():
    idx = torch.zeros(1, 1, dtype=torch.int32, device=DEV)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    lib = _lib.load()
    # T = 2**20 tokens with 512 experts needs 4 MiB of scratch (> 512 KiB)
    status = lib.bs_dispatch_noalloc(_p(idx), _lib.BS_I32, 1 << 20, 1, 512, None, 0, _p(idx),
                                     _p(idx), _p(idx), None, st)
    assert status == _lib.BS_ERR_CAPACITY
    assert b"512" in lib.bs_last_error_string() or b"524288" in lib.bs_last_error_string()
