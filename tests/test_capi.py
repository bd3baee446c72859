"""The C-ABI library loads, exports every symbol include/bs_moe.h declares, and
rejects bad arguments before touching a device (no GPU needed)."""

import ctypes
import os
import re

import pytest

from conftest import REPO
from blockstreamer_b200 import _lib

HEADER = os.path.join(REPO, "include", "bs_moe.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(bs_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_expected_entry_points():
    names = declared_functions()
    for n in ("bs_dequant_mxfp4", "bs_router", "bs_dispatch", "bs_moe_gate_up", "bs_moe_down",
              "bs_combine", "bs_mxfp4_matmul", "bs_moe_forward", "bs_last_error_string"):
        assert n in names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for n in declared_functions():
        assert hasattr(lib, n), n
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"


def test_version_and_error_string():
    lib = _lib.load()
    assert lib.bs_version() >= 1
    assert isinstance(lib.bs_last_error_string(), bytes)


def _err(lib):
    return lib.bs_last_error_string().decode()


def test_null_and_misaligned_pointers_are_rejected():
    lib = _lib.load()
    assert lib.bs_dequant_mxfp4(None, None, 1, 1, 1, 1, None, None) == _lib.BS_ERR_INVALID_ARGUMENT
    assert "null" in _err(lib)
    bad = ctypes.c_void_p(0x1001)
    good = ctypes.c_void_p(0x1000)
    assert lib.bs_dequant_mxfp4(bad, good, 1, 1, 1, 1, good, None) == _lib.BS_ERR_MISALIGNED
    assert "aligned" in _err(lib)


def test_bad_shapes_are_rejected():
    lib = _lib.load()
    p = ctypes.c_void_p(0x1000)
    # contraction not a multiple of 32
    st = lib.bs_moe_gate_up(p, p, 4, 4, 2, 48, 64, p, p, p, 0, 1.702, 7.0, p, 0, None)
    assert st == _lib.BS_ERR_INVALID_ARGUMENT and "multiple of 32" in _err(lib)
    # top_k larger than the expert count
    st = lib.bs_router(p, 0, p, p, 1, 4, 64, 4, 8, None, p, p, 2, None, 0, None)
    assert st == _lib.BS_ERR_INVALID_ARGUMENT
    # unknown dtype code
    st = lib.bs_router(p, 7, p, p, 1, 4, 64, 8, 2, None, p, p, 2, None, 0, None)
    assert st == _lib.BS_ERR_INVALID_ARGUMENT


def test_workspace_capacity_is_checked():
    lib = _lib.load()
    p = ctypes.c_void_p(0x1000)
    need = lib.bs_dispatch_workspace_bytes(1024, 4, 128)
    assert need > 0
    st = lib.bs_dispatch(p, 2, 1024, 4, 128, None, 0, p, p, p, None, p, need - 1, None)
    assert st == _lib.BS_ERR_CAPACITY


def test_workspace_size_formula():
    lib = _lib.load()
    small = lib.bs_moe_workspace_bytes(64, 256, 256, 8, 2)
    big = lib.bs_moe_workspace_bytes(8192, 2880, 2880, 128, 4)
    assert 0 < small < big
    # x_perm + h + y for T*k rows dominate
    assert big >= 8192 * 4 * (2880 + 2880 + 2880) * 2


def test_python_raises_valueerror_with_message():
    with pytest.raises(ValueError, match="null pointer"):
        _lib.call("bs_dequant_mxfp4", None, None, 1, 1, 1, 1, None, None)


def test_expert_parallel_exchange_layout():
    """bs_ep_p2p_bytes / bs_ep_p2p_layout (host arithmetic, no GPU): the receive
    area holds cap_rows rows and the result area src_rows rows, 256-byte aligned
    and disjoint, inside the buffer; argument checks reject bad rank/expert
    counts before any device work."""
    lib = _lib.load()
    for R, E, H, T, k in ((2, 128, 2880, 4096, 4), (8, 128, 2880, 1024, 4), (4, 16, 512, 64, 2)):
        src_rows = T * k
        cap = R * src_rows
        total = lib.bs_ep_p2p_bytes(R, E, H, cap, src_rows)
        ro, yo = ctypes.c_size_t(), ctypes.c_size_t()
        assert lib.bs_ep_p2p_layout(R, E, H, cap, src_rows, ctypes.byref(ro), ctypes.byref(yo)) == 0
        assert ro.value % 256 == 0 and yo.value % 256 == 0
        assert ro.value >= R * E * 4                       # flags and the counts matrix come first
        assert yo.value >= ro.value + cap * H * 2           # recv, then yback
        assert total >= yo.value + src_rows * H * 2
    base = ctypes.c_void_p(16)
    st = lib.bs_ep_p2p_dispatch(base, 2880, base, base, base, base, 3, 128, 0, 3, 1, base, None)
    assert st == _lib.BS_ERR_INVALID_ARGUMENT or st == _lib.BS_ERR_UNSUPPORTED   # 128 experts over 3 ranks


def test_norm_and_block_entry_points_reject_bad_arguments():
    """bs_rmsnorm / bs_moe_block_forward check pointers, sizes, dtypes, aliasing
    and workspace capacity before any device work."""
    lib = _lib.load()
    p = ctypes.c_void_p(0x1000)
    q = ctypes.c_void_p(0x2000)
    assert lib.bs_rmsnorm(None, 4, 64, p, _lib.BS_F32, 1e-5, p, None) == _lib.BS_ERR_INVALID_ARGUMENT
    assert lib.bs_rmsnorm(p, 4, 60, p, _lib.BS_F32, 1e-5, q, None) == _lib.BS_ERR_INVALID_ARGUMENT  # H % 8
    assert lib.bs_rmsnorm(p, 4, 64, p, _lib.BS_I32, 1e-5, q, None) == _lib.BS_ERR_INVALID_ARGUMENT  # dtype
    assert lib.bs_rmsnorm(ctypes.c_void_p(0x1008), 4, 64, p, _lib.BS_F32, 1e-5, q, None) == _lib.BS_ERR_MISALIGNED
    args = [4, 64, 64, 8, 2, p, _lib.BS_F32, 1e-5, p, p, _lib.BS_F32, p, p, p, p, p, p, p, p, _lib.BS_BF16,
            1.702, 7.0]
    # out aliasing x (x is the residual)
    assert lib.bs_moe_block_forward(p, *args, p, q, 1 << 30, 0, None) == _lib.BS_ERR_INVALID_ARGUMENT
    assert "alias" in _err(lib)
    # workspace too small
    need = lib.bs_moe_block_workspace_bytes(4, 64, 64, 8, 2)
    assert need > lib.bs_moe_workspace_bytes(4, 64, 64, 8, 2)
    assert lib.bs_moe_block_forward(p, *args, q, q, need - 1, 0, None) == _lib.BS_ERR_CAPACITY
