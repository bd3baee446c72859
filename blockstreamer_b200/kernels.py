"""Typed torch wrappers over the C ABI (include/bs_moe.h).

Every function launches on ``torch.cuda.current_stream()`` of its inputs'
device, allocates outputs and workspaces through the torch caching allocator
(so ``record_stream`` semantics hold for callers such as StreamedModel's pool),
reads ``data_ptr()`` on every call (no cached pointers), and never mutates its
inputs.  All tensors must be CUDA tensors: there is no CPU path.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib
from ._lib import ALGO_AUTO, ALGO_FUSED, ALGO_GEMV, ALGO_MX, ALGO_TCGEN05, ALGO_TCGEN05_PAIR  # noqa: F401  (re-exported)

_DT = {torch.bfloat16: _lib.BS_BF16, torch.float32: _lib.BS_F32,
       torch.int32: _lib.BS_I32, torch.int64: _lib.BS_I64}

ALPHA = 1.702
LIMIT = 7.0


def _p(t: torch.Tensor | None):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _stream(t: torch.Tensor):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _cuda(name: str, *ts: torch.Tensor | None) -> torch.device:
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError(f"{name}: blockstreamer_b200 runs on CUDA tensors only (got {t.device})")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"{name}: tensors on {dev} and {t.device}")
    return dev


def _contig(name: str, t: torch.Tensor) -> torch.Tensor:
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    return t


def device_status(device=None, clear: bool = True) -> int:
    """Status word kernels on ``device`` recorded (0 = none); synchronizes."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    out = ctypes.c_int(0)
    with torch.cuda.device(dev):
        _lib.call("bs_device_status", ctypes.byref(out), int(clear),
                  ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
    return out.value


def dequant_mxfp4(blocks: torch.Tensor, scales: torch.Tensor, transpose: bool = True) -> torch.Tensor:
    """[E, rows, G, 16] u8 + [E, rows, G] u8 -> bf16 [E, G*32, rows] (transpose) or [E, rows, G*32]."""
    _cuda("dequant_mxfp4", blocks, scales)
    if blocks.dim() != 4 or blocks.shape[-1] != 16 or tuple(scales.shape) != tuple(blocks.shape[:3]):
        raise ValueError(f"blocks {tuple(blocks.shape)} / scales {tuple(scales.shape)}: expected "
                         "[E, rows, G, 16] and [E, rows, G]")
    if blocks.dtype != torch.uint8 or scales.dtype != torch.uint8:
        raise ValueError("blocks and scales must be uint8")
    E, R, G, _ = blocks.shape
    blocks, scales = _contig("blocks", blocks), _contig("scales", scales)
    shape = (E, G * 32, R) if transpose else (E, R, G * 32)
    out = torch.empty(shape, dtype=torch.bfloat16, device=blocks.device)
    with torch.cuda.device(blocks.device):
        _lib.call("bs_dequant_mxfp4", _p(blocks), _p(scales), E, R, G, int(transpose), _p(out), _stream(blocks))
    return out


def router(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, top_k: int,
           return_logits: bool = False, index_dtype: torch.dtype = torch.int64,
           use_workspace: bool = True, out_scores: torch.Tensor | None = None,
           out_indices: torch.Tensor | None = None, workspace: torch.Tensor | None = None):
    """GptOssTopKRouter.forward: returns (logits | None, scores [T,k] f32, indices [T,k]).

    With ``use_workspace`` (default) the library may use its tensor-core form;
    without, the fp32 CUDA-core form runs.  ``out_*`` and ``workspace`` let a
    caller reuse buffers across calls.
    """
    _cuda("router", x, weight, bias)
    T, H = x.shape
    E = weight.shape[0]
    if weight.shape != (E, H) or bias.shape != (E,):
        raise ValueError(f"router weight {tuple(weight.shape)} / bias {tuple(bias.shape)} vs hidden {H}")
    if weight.dtype != bias.dtype:
        raise ValueError("router weight and bias must share a dtype")
    x, weight, bias = _contig("x", x), _contig("weight", weight), _contig("bias", bias)
    dev = x.device
    logits = torch.empty(T, E, dtype=torch.float32, device=dev) if return_logits else None
    scores = out_scores if out_scores is not None else torch.empty(T, top_k, dtype=torch.float32, device=dev)
    idx = out_indices if out_indices is not None else torch.empty(T, top_k, dtype=index_dtype, device=dev)
    index_dtype = idx.dtype
    ws, ws_bytes = None, 0
    if use_workspace:
        ws_bytes = _lib.load().bs_router_workspace_bytes(T, H, E, _DT[weight.dtype])
        ws = workspace if workspace is not None and workspace.numel() >= ws_bytes else \
            torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
        ws_bytes = ws.numel()
    with torch.cuda.device(dev):
        _lib.call("bs_router", _p(x), _DT[x.dtype], _p(weight), _p(bias), _DT[weight.dtype],
                  T, H, E, top_k, _p(logits), _p(scores), _p(idx), _DT[index_dtype], _p(ws), ws_bytes,
                  _stream(x))
    return logits, scores, idx


@dataclass
class Dispatch:
    expert_offsets: torch.Tensor   # [E+1] int32
    row_of_slot: torch.Tensor      # [T*k] int32
    token_of_row: torch.Tensor     # [T*k] int32
    x_perm: torch.Tensor | None    # [T*k, H] bf16


def dispatch(indices: torch.Tensor, num_experts: int, x: torch.Tensor | None = None,
             out: Dispatch | None = None, workspace: torch.Tensor | None = None) -> Dispatch:
    """Group the (token, slot) pairs by expert; optionally gather x rows.
    ``out`` (a previous result of the same shapes) and ``workspace`` are reused when given."""
    _cuda("dispatch", indices, x)
    T, k = indices.shape
    indices = _contig("indices", indices)
    dev = indices.device
    S = T * k
    if out is not None:
        offsets, row_of_slot, token_of_row, x_perm = (out.expert_offsets, out.row_of_slot,
                                                      out.token_of_row, out.x_perm)
    else:
        offsets = torch.empty(num_experts + 1, dtype=torch.int32, device=dev)
        row_of_slot = torch.empty(S, dtype=torch.int32, device=dev)
        token_of_row = torch.empty(S, dtype=torch.int32, device=dev)
        x_perm = None
    H = 0
    if x is not None:
        x = _contig("x", x)
        H = x.shape[1]
        if x_perm is None:
            x_perm = torch.empty(S, H, dtype=x.dtype, device=dev)
    else:
        x_perm = None
    lib = _lib.load()
    ws_bytes = lib.bs_dispatch_workspace_bytes(T, k, num_experts)
    ws = workspace if workspace is not None and workspace.numel() >= ws_bytes else \
        torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
    ws_bytes = ws.numel()
    with torch.cuda.device(dev):
        _lib.call("bs_dispatch", _p(indices), _DT[indices.dtype], T, k, num_experts, _p(x), H,
                  _p(offsets), _p(row_of_slot), _p(token_of_row), _p(x_perm), _p(ws), ws_bytes,
                  _stream(indices))
    return Dispatch(offsets, row_of_slot, token_of_row, x_perm)


def _bias_code(bias: torch.Tensor | None) -> int:
    if bias is None:
        return _lib.BS_BF16
    if bias.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("bias must be bf16 or f32")
    return _DT[bias.dtype]


def moe_gate_up(x_perm, expert_offsets, blocks, scales, bias, alpha=ALPHA, limit=LIMIT,
                algo=ALGO_AUTO, max_rows_per_expert=None, out: torch.Tensor | None = None) -> torch.Tensor:
    """h [rows, I] = SwiGLU(x_perm @ dequant(W_gu[e]) + b_gu[e]) per expert segment."""
    _cuda("moe_gate_up", x_perm, expert_offsets, blocks, scales, bias)
    S, H = x_perm.shape
    E, two_i, G, _ = blocks.shape
    if G * 32 != H or two_i % 2:
        raise ValueError(f"gate_up blocks {tuple(blocks.shape)} do not match hidden size {H}")
    I = two_i // 2
    h = out if out is not None else torch.empty(S, I, dtype=torch.bfloat16, device=x_perm.device)
    mr = S if max_rows_per_expert is None else max_rows_per_expert
    with torch.cuda.device(x_perm.device):
        _lib.call("bs_moe_gate_up", _p(x_perm), _p(expert_offsets), S, mr, E, H, I, _p(blocks),
                  _p(scales), _p(bias), _bias_code(bias), float(alpha), float(limit), _p(h), algo,
                  _stream(x_perm))
    return h


def moe_down(h, expert_offsets, blocks, scales, bias, algo=ALGO_AUTO, max_rows_per_expert=None,
             out: torch.Tensor | None = None) -> torch.Tensor:
    """y [rows, H] = h @ dequant(W_d[e]) + b_d[e] per expert segment."""
    _cuda("moe_down", h, expert_offsets, blocks, scales, bias)
    S, I = h.shape
    E, H, G, _ = blocks.shape
    if G * 32 != I:
        raise ValueError(f"down blocks {tuple(blocks.shape)} do not match intermediate size {I}")
    y = out if out is not None else torch.empty(S, H, dtype=torch.bfloat16, device=h.device)
    mr = S if max_rows_per_expert is None else max_rows_per_expert
    with torch.cuda.device(h.device):
        _lib.call("bs_moe_down", _p(h), _p(expert_offsets), S, mr, E, H, I, _p(blocks), _p(scales),
                  _p(bias), _bias_code(bias), _p(y), algo, _stream(h))
    return y


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, out: torch.Tensor | None = None) -> torch.Tensor:
    """GptOssRMSNorm: bf16(weight * (x * rsqrt(mean(x^2) + eps))) per row (bs_rmsnorm)."""
    _cuda("rmsnorm", x, weight)
    if x.dtype != torch.bfloat16 or weight.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("rmsnorm: x must be bf16 and weight bf16 or f32")
    x = _contig("x", x)
    T, H = x.shape
    out = out if out is not None else torch.empty_like(x)
    with torch.cuda.device(x.device):
        _lib.call("bs_rmsnorm", _p(x), T, H, _p(_contig("weight", weight)), _DT[weight.dtype], float(eps),
                  _p(out), _stream(x))
    return out


def combine(y: torch.Tensor, row_of_slot: torch.Tensor, weights: torch.Tensor, num_tokens: int,
            out: torch.Tensor | None = None) -> torch.Tensor:
    """out[t] = sum_s weights[t,s] * y[row_of_slot[t*k+s]] (fp32 sum, bf16 out)."""
    _cuda("combine", y, row_of_slot, weights)
    k = row_of_slot.numel() // max(num_tokens, 1)
    H = y.shape[1]
    w = weights.float().contiguous()
    out = out if out is not None else torch.empty(num_tokens, H, dtype=torch.bfloat16, device=y.device)
    with torch.cuda.device(y.device):
        _lib.call("bs_combine", _p(y), _p(row_of_slot), _p(w), num_tokens, k, H, _p(out), _stream(y))
    return out


def ep_regroup(recv_counts: torch.Tensor, x_recv: torch.Tensor, out: torch.Tensor | None = None):
    """Expert-major regroup of all-to-all-received rows (see bs_ep_regroup).

    recv_counts [R, El] int32 on the device; returns (x_grouped, expert_offsets [El+1], row_map)."""
    _cuda("ep_regroup", recv_counts, x_recv)
    R, El = recv_counts.shape
    rows, H = x_recv.shape
    dev = x_recv.device
    x_grouped = out if out is not None else torch.empty_like(x_recv)
    offsets = torch.empty(El + 1, dtype=torch.int32, device=dev)
    row_map = torch.empty(max(rows, 1), dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        _lib.call("bs_ep_regroup", _p(_contig("recv_counts", recv_counts.to(torch.int32))), R, El,
                  _p(_contig("x_recv", x_recv)), rows, H, _p(x_grouped), _p(offsets), _p(row_map),
                  _stream(x_recv))
    return x_grouped, offsets, row_map[:rows]


def gather_rows(src: torch.Tensor, row_map: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """dst[i] = src[row_map[i]] (rows of bf16)."""
    _cuda("gather_rows", src, row_map)
    rows = row_map.numel()
    H = src.shape[1]
    dst = out if out is not None else torch.empty(rows, H, dtype=src.dtype, device=src.device)
    with torch.cuda.device(src.device):
        _lib.call("bs_gather_rows", _p(_contig("src", src)), _p(_contig("row_map", row_map)), rows, H,
                  _p(dst), _stream(src))
    return dst


def mxfp4_matmul(x: torch.Tensor, blocks: torch.Tensor, scales: torch.Tensor,
                 bias: torch.Tensor | None = None, algo=ALGO_AUTO) -> torch.Tensor:
    """x [m, K] bf16 @ dequant(W) for one expert W = blocks [N, K/32, 16] -> [m, N] bf16."""
    _cuda("mxfp4_matmul", x, blocks, scales, bias)
    if x.dtype != torch.bfloat16:
        raise ValueError("mxfp4_matmul: x must be bf16")
    m, K = x.shape
    N, G, _ = blocks.shape
    if G * 32 != K:
        raise ValueError(f"blocks {tuple(blocks.shape)} do not match K={K}")
    x = _contig("x", x)
    out = torch.empty(m, N, dtype=torch.bfloat16, device=x.device)
    with torch.cuda.device(x.device):
        _lib.call("bs_mxfp4_matmul", _p(x), m, K, _p(_contig("blocks", blocks)),
                  _p(_contig("scales", scales)), N, _p(bias), _p(out), algo, _stream(x))
    return out


def moe_block_forward(x: torch.Tensor, norm_weight: torch.Tensor, eps: float, gate_up_blocks,
                      gate_up_scales, gate_up_bias, down_blocks, down_scales, down_bias, top_k: int,
                      router_weight, router_bias, alpha=ALPHA, limit=LIMIT, algo=ALGO_AUTO):
    """x + MoE(RMSNorm(x)) through bs_moe_block_forward: returns (out, scores f32, indices int32)."""
    _cuda("moe_block_forward", x, norm_weight, gate_up_blocks, gate_up_scales, down_blocks, down_scales,
          router_weight)
    if x.dtype != torch.bfloat16:
        raise ValueError("moe_block_forward: hidden states must be bf16")
    x = _contig("x", x)
    T, H = x.shape
    E, two_i = gate_up_blocks.shape[:2]
    I = two_i // 2
    dev = x.device
    idx = torch.empty(T, top_k, dtype=torch.int32, device=dev)
    sc = torch.empty(T, top_k, dtype=torch.float32, device=dev)
    lib = _lib.load()
    ws = torch.empty(max(lib.bs_moe_block_workspace_bytes(T, H, I, E, top_k), 16), dtype=torch.uint8, device=dev)
    out = torch.empty_like(x)
    bias_code = _bias_code(gate_up_bias)
    if down_bias is not None and down_bias.dtype != gate_up_bias.dtype:
        down_bias = down_bias.to(gate_up_bias.dtype)
    with torch.cuda.device(dev):
        _lib.call("bs_moe_block_forward", _p(x), T, H, I, E, top_k, _p(_contig("norm_weight", norm_weight)),
                  _DT[norm_weight.dtype], float(eps), _p(router_weight), _p(router_bias),
                  _DT[router_weight.dtype], _p(sc), _p(idx), _p(gate_up_blocks), _p(gate_up_scales),
                  _p(gate_up_bias), _p(down_blocks), _p(down_scales), _p(down_bias), bias_code, float(alpha),
                  float(limit), _p(out), _p(ws), ws.numel(), algo, _stream(x))
    return out, sc, idx


def moe_forward(x: torch.Tensor, gate_up_blocks, gate_up_scales, gate_up_bias, down_blocks,
                down_scales, down_bias, top_k: int, router_weight=None, router_bias=None,
                indices=None, scores=None, alpha=ALPHA, limit=LIMIT, algo=ALGO_AUTO,
                workspace: torch.Tensor | None = None):
    """Whole layer through bs_moe_forward.

    With router weights: computes the routing and returns (out, scores f32, indices int32).
    Without: ``indices`` [T,k] and ``scores`` [T,k] are the caller's routing.
    """
    _cuda("moe_forward", x, gate_up_blocks, gate_up_scales, down_blocks, down_scales,
          router_weight, indices, scores)
    if x.dtype != torch.bfloat16:
        raise ValueError("moe_forward: hidden states must be bf16")
    x = _contig("x", x)
    T, H = x.shape
    E, two_i = gate_up_blocks.shape[:2]
    I = two_i // 2
    dev = x.device
    if router_weight is None:
        if indices is None or scores is None:
            raise ValueError("moe_forward: give router weights or (indices, scores)")
        idx = indices.to(torch.int32).contiguous()
        sc = scores.float().contiguous()
    else:
        idx = torch.empty(T, top_k, dtype=torch.int32, device=dev)
        sc = torch.empty(T, top_k, dtype=torch.float32, device=dev)
    lib = _lib.load()
    ws_bytes = lib.bs_moe_workspace_bytes(T, H, I, E, top_k)
    if workspace is None or workspace.numel() < ws_bytes:
        workspace = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=dev)
    out = torch.empty_like(x)
    rdt = _DT[router_weight.dtype] if router_weight is not None else _lib.BS_F32
    bias_code = _bias_code(gate_up_bias)
    if down_bias is not None and down_bias.dtype != gate_up_bias.dtype:
        down_bias = down_bias.to(gate_up_bias.dtype)
    with torch.cuda.device(dev):
        _lib.call("bs_moe_forward", _p(x), T, H, I, E, top_k,
                  _p(router_weight), _p(router_bias), rdt, _p(sc), _p(idx),
                  _p(gate_up_blocks), _p(gate_up_scales), _p(gate_up_bias),
                  _p(down_blocks), _p(down_scales), _p(down_bias), bias_code,
                  float(alpha), float(limit), _p(out), _p(workspace), workspace.numel(), algo,
                  _stream(x))
    return out, sc, idx


def moe_backward(x: torch.Tensor, indices: torch.Tensor, weights: torch.Tensor, grad_out: torch.Tensor,
                 gate_up_blocks, gate_up_scales, gate_up_bias, down_blocks, down_scales, down_bias,
                 alpha=ALPHA, limit=LIMIT):
    """dL/dx [T,H] f32 and dL/d routing weights [T,k] f32 of the expert layer
    (bs_moe_backward): transposed tcgen05 grouped GEMMs over the packed
    weights, no host synchronization."""
    _cuda("moe_backward", x, indices, weights, grad_out, gate_up_blocks, gate_up_scales, down_blocks, down_scales)
    if x.dtype != torch.bfloat16:
        raise ValueError("moe_backward: x must be bf16")
    if grad_out.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("moe_backward: grad_out must be bf16 or f32")
    x = _contig("x", x)
    T, H = x.shape
    k = indices.shape[1]
    E, two_i = gate_up_blocks.shape[:2]
    I = two_i // 2
    dev = x.device
    idx = indices.to(torch.int32).contiguous()
    w = weights.float().contiguous()
    go = _contig("grad_out", grad_out)
    gx = torch.empty(T, H, dtype=torch.float32, device=dev)
    gw = torch.empty(T, k, dtype=torch.float32, device=dev)
    ws = torch.empty(max(_lib.load().bs_moe_backward_workspace_bytes(T, H, I, E, k), 16), dtype=torch.uint8,
                     device=dev)
    bias_code = _bias_code(gate_up_bias)
    if down_bias is not None and down_bias.dtype != gate_up_bias.dtype:
        down_bias = down_bias.to(gate_up_bias.dtype)
    with torch.cuda.device(dev):
        _lib.call("bs_moe_backward", _p(x), T, H, I, E, k, _p(idx), _p(w), _p(go), _DT[go.dtype],
                  _p(gate_up_blocks), _p(gate_up_scales), _p(gate_up_bias), _p(down_blocks), _p(down_scales),
                  _p(down_bias), bias_code, float(alpha), float(limit), _p(gx), _p(gw), _p(ws), ws.numel(),
                  _stream(x))
    return gx, gw


def router_backward(x: torch.Tensor, weight: torch.Tensor, scores: torch.Tensor, indices: torch.Tensor,
                    grad_scores: torch.Tensor, want_weight_grad: bool = False, want_bias_grad: bool = False):
    """Backward of the router (bs_router_backward): returns (dL/dx f32 [T,H],
    dL/dW f32 [E,H] or None, dL/db f32 [E] or None)."""
    _cuda("router_backward", x, weight, scores, indices, grad_scores)
    x = _contig("x", x)
    T, H = x.shape
    E = weight.shape[0]
    k = indices.shape[1]
    dev = x.device
    gx = torch.zeros(T, H, dtype=torch.float32, device=dev)
    gW = torch.zeros(E, H, dtype=torch.float32, device=dev) if want_weight_grad else None
    gb = torch.zeros(E, dtype=torch.float32, device=dev) if want_bias_grad else None
    with torch.cuda.device(dev):
        _lib.call("bs_router_backward", _p(x), _DT[x.dtype], T, H, E, k, _p(_contig("weight", weight)),
                  _DT[weight.dtype], _p(scores.float().contiguous()), _p(indices.to(torch.int32).contiguous()),
                  _p(grad_scores.float().contiguous()), _p(gx), _p(gW), _p(gb), _stream(x))
    return gx, gW, gb


def mxfp4_matmul_backward(grad_out: torch.Tensor, blocks: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """dL/dx [m, K] bf16 of x @ dequant(W) for one expert W = blocks [N, K/32, 16]
    (bs_mxfp4_matmul_backward: the transposed tcgen05 GEMM, no dense weight)."""
    _cuda("mxfp4_matmul_backward", grad_out, blocks, scales)
    go = _contig("grad_out", grad_out.to(torch.bfloat16))
    m, N = go.shape
    K = blocks.shape[1] * 32
    out = torch.empty(m, K, dtype=torch.bfloat16, device=go.device)
    lib = _lib.load()
    ws = torch.empty(max(lib.bs_mxfp4_matmul_backward_workspace_bytes(N, K), 16), dtype=torch.uint8,
                     device=go.device)
    with torch.cuda.device(go.device):
        _lib.call("bs_mxfp4_matmul_backward", _p(go), m, N, _p(_contig("blocks", blocks)),
                  _p(_contig("scales", scales)), K, _p(out), _p(ws), ws.numel(), _stream(go))
    return out
