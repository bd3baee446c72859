"""ctypes binding of libbs_moe.so, the sm_100a C ABI declared in include/bs_moe.h.

The library is built in-tree (``blockstreamer_b200/libbs_moe.so``) by
``blockstreamer_b200.build.build()``.  Loading fails loudly when it is missing:
there is no CPU or PyTorch fallback for any operation of this package.
"""

from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libbs_moe.so")

BS_OK = 0
BS_ERR_INVALID_ARGUMENT = 1
BS_ERR_MISALIGNED = 2
BS_ERR_CAPACITY = 3
BS_ERR_CUDA = 4
BS_ERR_TIMEOUT = 5
BS_ERR_UNSUPPORTED = 6

BS_BF16, BS_F32, BS_I32, BS_I64 = 0, 1, 2, 3
ALGO_AUTO, ALGO_GEMV, ALGO_TCGEN05, ALGO_MX, ALGO_FUSED, ALGO_TCGEN05_PAIR = 0, 1, 2, 3, 4, 5

_c = ctypes
_vp, _i64, _i32, _f32, _sz = _c.c_void_p, _c.c_int64, _c.c_int, _c.c_float, _c.c_size_t

# name -> (restype, argtypes); mirrors include/bs_moe.h
SIGNATURES = {
    "bs_version": (_i32, []),
    "bs_last_error_string": (_c.c_char_p, []),
    "bs_device_status": (_i32, [_c.POINTER(_c.c_int), _i32, _vp]),
    "bs_dequant_mxfp4": (_i32, [_vp, _vp, _i64, _i64, _i64, _i32, _vp, _vp]),
    "bs_router_workspace_bytes": (_sz, [_i64, _i64, _i64, _i32]),
    "bs_router": (_i32, [_vp, _i32, _vp, _vp, _i32, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _i32, _vp,
                         _sz, _vp]),
    "bs_dispatch_workspace_bytes": (_sz, [_i64, _i64, _i64]),
    "bs_dispatch": (_i32, [_vp, _i32, _i64, _i64, _i64, _vp, _i64, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "bs_dispatch_noalloc": (_i32, [_vp, _i32, _i64, _i64, _i64, _vp, _i64, _vp, _vp, _vp, _vp, _vp]),
    "bs_moe_gate_up": (_i32, [_vp, _vp, _i64, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _i32, _f32,
                              _f32, _vp, _i32, _vp]),
    "bs_moe_down": (_i32, [_vp, _vp, _i64, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _i32, _vp, _i32, _vp]),
    "bs_ep_regroup": (_i32, [_vp, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _vp, _vp]),
    "bs_gather_rows": (_i32, [_vp, _vp, _i64, _i64, _vp, _vp]),
    "bs_ep_p2p_bytes": (_sz, [_i64, _i64, _i64, _i64, _i64]),
    "bs_ep_p2p_layout": (_i32, [_i64, _i64, _i64, _i64, _i64, _c.POINTER(_sz), _c.POINTER(_sz)]),
    "bs_ep_p2p_alloc": (_i32, [_sz, _c.POINTER(_vp), _vp]),
    "bs_ep_p2p_open": (_i32, [_vp, _c.POINTER(_vp)]),
    "bs_ep_p2p_close": (_i32, [_vp]),
    "bs_ep_p2p_free": (_i32, [_vp]),
    "bs_ep_p2p_dispatch": (_i32, [_vp, _i64, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _vp, _vp]),
    "bs_ep_p2p_return": (_i32, [_vp, _i64, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _vp]),
    "bs_combine": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _vp, _vp]),
    "bs_mxfp4_matmul": (_i32, [_vp, _i64, _i64, _vp, _vp, _i64, _vp, _vp, _i32, _vp]),
    "bs_moe_workspace_bytes": (_sz, [_i64, _i64, _i64, _i64, _i64]),
    "bs_moe_decode": (_i32, [_vp, _i64, _i64, _i64, _i64, _i64, _vp, _vp, _i32, _vp, _vp,
                             _vp, _vp, _vp, _vp, _vp, _vp, _i32, _f32, _f32, _vp, _vp, _sz, _vp]),
    "bs_rmsnorm": (_i32, [_vp, _i64, _i64, _vp, _i32, _f32, _vp, _vp]),
    "bs_moe_block_workspace_bytes": (_sz, [_i64, _i64, _i64, _i64, _i64]),
    "bs_moe_block_forward": (_i32, [_vp, _i64, _i64, _i64, _i64, _i64, _vp, _i32, _f32, _vp, _vp, _i32, _vp,
                                    _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _f32, _f32, _vp, _vp, _sz, _i32,
                                    _vp]),
    "bs_moe_backward_workspace_bytes": (_sz, [_i64, _i64, _i64, _i64, _i64]),
    "bs_moe_backward": (_i32, [_vp, _i64, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _i32, _vp, _vp, _vp, _vp, _vp,
                               _vp, _i32, _f32, _f32, _vp, _vp, _vp, _sz, _vp]),
    "bs_router_backward": (_i32, [_vp, _i32, _i64, _i64, _i64, _i64, _vp, _i32, _vp, _vp, _vp, _vp, _vp, _vp,
                                  _vp]),
    "bs_mxfp4_matmul_backward_workspace_bytes": (_sz, [_i64, _i64]),
    "bs_mxfp4_matmul_backward": (_i32, [_vp, _i64, _i64, _vp, _vp, _i64, _vp, _vp, _sz, _vp]),
    "bs_moe_forward": (_i32, [_vp, _i64, _i64, _i64, _i64, _i64, _vp, _vp, _i32, _vp, _vp,
                              _vp, _vp, _vp, _vp, _vp, _vp, _i32, _f32, _f32, _vp, _vp, _sz, _i32, _vp]),
}

_lock = threading.Lock()
_lib = None


class BSError(RuntimeError):
    """A C-ABI call returned an error status."""

    def __init__(self, fn: str, status: int, message: str):
        super().__init__(f"{fn} failed with status {status}: {message}")
        self.status = status


def load(path: str | None = None) -> ctypes.CDLL:
    """Load (once) and type the library; raises if it was not built."""
    global _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = path or LIB_PATH
        if not os.path.exists(p):
            raise RuntimeError(
                f"{p} is missing: build it with blockstreamer_b200.build.build() "
                "(there is no fallback implementation)")
        lib = ctypes.CDLL(p)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if path is None:
            _lib = lib
        return lib


def call(name: str, *args) -> None:
    """Call an int-returning entry point and raise on a non-zero status."""
    lib = load()
    status = getattr(lib, name)(*args)
    if status != BS_OK:
        msg = lib.bs_last_error_string().decode(errors="replace")
        if status in (BS_ERR_INVALID_ARGUMENT, BS_ERR_MISALIGNED, BS_ERR_CAPACITY):
            raise ValueError(f"{name}: {msg}")
        raise BSError(name, status, msg)
