"""GPU parity of the backward kernels (the training path the reference gets from
autograd through block_streamer/gptoss.py:45-75, 137-177 and transformers'
GptOssTopKRouter, modeling_gpt_oss.py:126-130):

* the transposed tcgen05 grouped GEMM through bs_mxfp4_matmul_backward
  against dL/dx = grad @ W computed in fp32 from the dequantized weight;
* bs_moe_backward (dL/dx, dL/d routing weights) against torch autograd
  through the fp32 oracle, on uniform routing and on a skewed routing whose
  hot expert spans several 320-row token chunks (the 128 x 256 + 128 x 64 MMA
  pair and multi-chunk paths);
* bs_router_backward (dL/dx, dL/dW, dL/db) against autograd through
  F.linear + topk + softmax in fp32.

Tolerances: relative L2 <= 1e-2 (the intermediates are bf16, as in the
reference's own bf16 autograd).  The oracle runs on the GPU's copy of the
inputs in fp32 (TF32 off).
"""

import ctypes

import pytest
import torch

from blockstreamer_b200 import _lib, kernels
from blockstreamer_b200.synthetic import CASES, LayerShape, make_layer, make_tokens
from oracle import moe as omoe

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
NAMES = ("gate_up_proj_blocks", "gate_up_proj_scales", "gate_up_proj_bias", "down_proj_blocks",
         "down_proj_scales", "down_proj_bias")


@pytest.fixture(autouse=True)
def _true_fp32():
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32 = prev


def experts_of(p):
    return {k.split(".", 1)[1]: v for k, v in p.items() if k.startswith("experts.")}


def rel(a, b):
    return omoe.rel_l2(a.detach().float().cpu(), b.detach().float().cpu())


@pytest.mark.parametrize("m,N,K", [(8, 64, 128), (300, 5760, 2880), (333, 2880, 2880), (1000, 128, 256)])
def test_mxfp4_matmul_backward_vs_dense(m, N, K):
    g = torch.Generator().manual_seed(m + N)
    blocks = torch.randint(0, 256, (N, K // 32, 16), dtype=torch.uint8, generator=g).to(DEV)
    scales = torch.randint(118, 132, (N, K // 32), dtype=torch.uint8, generator=g).to(DEV)
    grad = torch.randn(m, N, generator=g).to(torch.bfloat16).to(DEV)
    w = omoe.dequant_expert(blocks, scales, torch.float32)          # [K, N]
    ref = grad.float() @ w.t()
    got = kernels.mxfp4_matmul_backward(grad, blocks, scales)
    r = rel(got, ref)
    print(f"m={m} N={N} K={K}: rel_l2 {r:.2e}")
    assert r <= 4e-3
    assert kernels.device_status(clear=True) == 0


def _moe_backward_case(shape, case_id, T, idx, w):
    p = make_layer(shape, case_id, device=DEV)
    pe = experts_of(p)
    x = make_tokens(T, shape.hidden, case_id, device=DEV)
    gout = torch.randn(T, shape.hidden, generator=torch.Generator(device=DEV).manual_seed(case_id),
                       device=DEV).to(torch.bfloat16)
    gx, gw = kernels.moe_backward(x, idx.to(DEV), w.to(DEV), gout, *[pe[n] for n in NAMES])
    torch.cuda.synchronize()
    assert kernels.device_status(clear=True) == 0
    xr = x.float().requires_grad_()
    wr = w.to(DEV).float().requires_grad_()
    ref = omoe.experts_fp32(xr, idx.to(DEV).long(), wr, pe)
    ref.backward(gout.float())
    rx, rw = rel(gx, xr.grad), rel(gw, wr.grad)
    print(f"T={T} E={shape.experts}: dx rel_l2 {rx:.2e}  dw rel_l2 {rw:.2e}")
    assert rx <= 1e-2 and rw <= 1e-2


def test_moe_backward_20b_uniform_routing():
    shape = CASES["gptoss20b"]
    T, E, k = 512, shape.experts, shape.top_k
    g = torch.Generator().manual_seed(1)
    idx = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).to(torch.int32)
    w = torch.softmax(torch.randn(T, k, generator=g), -1)
    _moe_backward_case(shape, 2, T, idx, w)


def test_moe_backward_skewed_multichunk():
    """Expert 3 takes every token (700 rows: three token chunks), the rest spread."""
    shape = LayerShape(512, 512, 16, 2, 120, 128)
    T = 700
    idx = torch.zeros(T, 2, dtype=torch.int32)
    idx[:, 0] = 3
    idx[:, 1] = torch.arange(T, dtype=torch.int32) % 5 + 6
    w = torch.softmax(torch.randn(T, 2, generator=torch.Generator().manual_seed(4)), -1)
    _moe_backward_case(shape, 41, T, idx, w)


def test_moe_backward_c_abi_rejects_unsupported_shapes():
    lib = _lib.load()
    z = ctypes.c_void_p(16)
    # H = 96 is not a multiple of 64 (the transposed GEMM's weight-row stages)
    st = lib.bs_moe_backward(z, 4, 96, 64, 4, 2, z, z, z, _lib.BS_BF16, z, z, z, z, z, z, _lib.BS_BF16, 1.702, 7.0,
                             z, z, z, 1 << 20, None)
    assert st == _lib.BS_ERR_INVALID_ARGUMENT


@pytest.mark.parametrize("wdt", [torch.float32, torch.bfloat16])
def test_router_backward_vs_autograd(wdt):
    T, H, E, k = 96, 2880, 128, 4
    g = torch.Generator().manual_seed(7)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16).to(DEV)
    W = (torch.randn(E, H, generator=g) * 0.02).to(wdt).to(DEV)
    b = (torch.randn(E, generator=g) * 0.01).to(wdt).to(DEV)
    _, sc, idx = kernels.router(x, W, b, k, index_dtype=torch.int32)
    ds = torch.randn(T, k, generator=g).to(DEV)
    gx, gW, gb = kernels.router_backward(x, W, sc, idx, ds, want_weight_grad=True, want_bias_grad=True)
    xr = x.float().requires_grad_()
    Wr = W.float().requires_grad_()
    br = b.float().requires_grad_()
    logits = torch.nn.functional.linear(xr, Wr, br)
    top_v = logits.gather(1, idx.long())                 # the kernel's selection
    torch.softmax(top_v, dim=1).backward(ds)
    rx, rW, rb = rel(gx, xr.grad), rel(gW, Wr.grad), rel(gb, br.grad)
    print(f"router {wdt}: dx {rx:.2e} dW {rW:.2e} db {rb:.2e}")
    # a bf16 router rounds its logits to bf16 (as the reference computes them
    # in the weight dtype), which moves the softmax Jacobian by ~2^-9
    tol = 1e-4 if wdt == torch.float32 else 1e-2
    assert rx <= tol and rW <= tol and rb <= tol
    assert kernels.device_status(clear=True) == 0
