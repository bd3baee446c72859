"""Drop-in gpt-oss MoE modules backed by the sm_100a kernels.

Mirrors ``block_streamer/gptoss.py`` (hareramray/BlockStreamer) and the
transformers gpt-oss MLP it plugs into:

* ``dequantize_expert`` / ``mxfp4_matmul``       — gptoss.py:24-42, 45-75
* ``B200MXFP4Experts``                           — gptoss.py:78-177 (``MXFP4Experts``)
* ``install_b200_experts``                       — gptoss.py:180-189 (``install_mxfp4_experts``)
* ``B200GptOssMLP`` / ``install_b200_mlp``       — transformers models/gpt_oss/
  modeling_gpt_oss.py:117-146 (``GptOssTopKRouter`` + ``GptOssMLP``) with the
  experts above, as one fused layer.

Parameter names, shapes and dtypes are the checkpoint's, so
``StreamedModel``'s ``functional_call(..., strict=True)`` binds staged state to
these modules unchanged.  The modules read ``data_ptr()`` on every call, launch
on the current stream, allocate workspaces with the caching allocator and
never mutate their parameters.
"""

from __future__ import annotations

import torch
from torch import Tensor, nn

from . import kernels


def dequantize_expert(blocks: Tensor, scales: Tensor, dtype: torch.dtype = torch.bfloat16) -> Tensor:
    """Dequantize one expert's packed MXFP4 weight to a dense [groups*32, rows] matrix.

    Same contract as the reference (gptoss.py:24-42): ``blocks`` is
    [1, rows, groups, 16] uint8 and ``scales`` [1, rows, groups]; a missing
    leading expert dimension raises ``ValueError``.  Bit-exact with the
    reference for every byte and scale.
    """
    if blocks.dim() != 4:
        raise ValueError(f"Expected [1, rows, groups, 16] packed blocks, got {tuple(blocks.shape)}")
    dense = kernels.dequant_mxfp4(blocks, scales, transpose=True)
    if dtype != torch.bfloat16:
        # every dequantized value has at most two significant bits, so the bf16
        # result converts exactly to wider float types
        dense = dense.to(dtype)
    return dense.squeeze(0)


class _MXFP4Matmul(torch.autograd.Function):
    """x @ dequantize(blocks, scales) without a dense weight in either direction.

    Forward: the fused dequant-GEMM kernel.  Backward (dL/dx, the role of
    gptoss.py:64-71): the transposed tcgen05 GEMM over the packed codes
    (bs_mxfp4_matmul_backward); nothing is saved but the packed tensors."""

    @staticmethod
    def forward(ctx, x: Tensor, blocks: Tensor, scales: Tensor) -> Tensor:
        ctx.save_for_backward(blocks, scales)
        ctx.x_dtype = x.dtype
        lead = x.shape[:-1]
        out = kernels.mxfp4_matmul(x.reshape(-1, x.shape[-1]).to(torch.bfloat16).contiguous(),
                                   blocks.squeeze(0), scales.squeeze(0))
        return out.reshape(*lead, out.shape[-1]).to(x.dtype)

    @staticmethod
    def backward(ctx, grad: Tensor):
        blocks, scales = ctx.saved_tensors
        if not ctx.needs_input_grad[0]:
            return None, None, None
        lead = grad.shape[:-1]
        gx = kernels.mxfp4_matmul_backward(grad.reshape(-1, grad.shape[-1]), blocks.squeeze(0), scales.squeeze(0))
        return gx.reshape(*lead, gx.shape[-1]).to(ctx.x_dtype), None, None


def mxfp4_matmul(x: Tensor, blocks: Tensor, scales: Tensor) -> Tensor:
    """gptoss.py:74-75: ``x @ dequantize_expert(blocks, scales)`` for blocks [1, N, G, 16]."""
    if blocks.dim() != 4:
        raise ValueError(f"Expected [1, rows, groups, 16] packed blocks, got {tuple(blocks.shape)}")
    return _MXFP4Matmul.apply(x, blocks, scales)


class _ExpertsFunction(torch.autograd.Function):
    """The expert layer as one differentiable op over the library's kernels.

    Forward: bs_moe_forward with the caller's routing.  Backward (what the
    reference gets from autograd through its per-expert loop,
    gptoss.py:137-177 with 64-71): bs_moe_backward -- dL/dx and dL/d routing
    weights from the recomputed intermediates and two transposed grouped
    GEMMs, with no host synchronization.  Only x (bf16), the routing and the
    module are kept for backward."""

    @staticmethod
    def forward(ctx, x: Tensor, weights: Tensor, indices: Tensor, m: "B200MXFP4Experts") -> Tensor:
        xb = x.to(torch.bfloat16).contiguous()
        idx = indices.to(torch.int32).contiguous()
        w = weights.float().contiguous()
        out, _, _ = kernels.moe_forward(
            xb, m.gate_up_proj_blocks, m.gate_up_proj_scales, m.gate_up_proj_bias, m.down_proj_blocks,
            m.down_proj_scales, m.down_proj_bias, idx.shape[1], indices=idx, scores=w, alpha=m.alpha,
            limit=m.limit, algo=m.algo)
        ctx.save_for_backward(xb, idx, w)
        ctx.m = m
        ctx.dtypes = (x.dtype, weights.dtype)
        return out.to(x.dtype)

    @staticmethod
    def backward(ctx, grad: Tensor):
        xb, idx, w = ctx.saved_tensors
        m = ctx.m
        g = grad.contiguous() if grad.dtype in (torch.bfloat16, torch.float32) else grad.float().contiguous()
        gx, gw = kernels.moe_backward(xb, idx, w, g, m.gate_up_proj_blocks, m.gate_up_proj_scales,
                                      m.gate_up_proj_bias, m.down_proj_blocks, m.down_proj_scales,
                                      m.down_proj_bias, alpha=m.alpha, limit=m.limit)
        dx = gx.to(ctx.dtypes[0]) if ctx.needs_input_grad[0] else None
        dw = gw.to(ctx.dtypes[1]) if ctx.needs_input_grad[1] else None
        return dx, dw, None, None


class _RouterFunction(torch.autograd.Function):
    """GptOssTopKRouter (modeling_gpt_oss.py:126-130) as one differentiable op:
    forward on the library's router kernel (bf16 tokens, fp32 accumulate),
    backward through the softmax over the k selected logits on
    bs_router_backward (dL/dx, and dL/dW, dL/db when they require grad)."""

    @staticmethod
    def forward(ctx, x: Tensor, weight: Tensor, bias: Tensor, top_k: int):
        xb = x.to(torch.bfloat16).contiguous()
        _, scores, idx = kernels.router(xb, weight, bias, top_k, index_dtype=torch.int32)
        ctx.save_for_backward(xb, weight, scores, idx)
        ctx.x_dtype = x.dtype
        ctx.mark_non_differentiable(idx)
        return scores, idx

    @staticmethod
    def backward(ctx, grad_scores: Tensor, _grad_idx):
        xb, weight, scores, idx = ctx.saved_tensors
        gx, gW, gb = kernels.router_backward(xb, weight, scores, idx, grad_scores,
                                             want_weight_grad=ctx.needs_input_grad[1],
                                             want_bias_grad=ctx.needs_input_grad[2])
        return (gx.to(ctx.x_dtype) if ctx.needs_input_grad[0] else None,
                gW.to(weight.dtype) if gW is not None else None,
                gb.to(weight.dtype) if gb is not None else None, None)


def _packed(experts: int, rows: int, groups: int) -> nn.Parameter:
    return nn.Parameter(torch.empty(experts, rows, groups, 16, dtype=torch.uint8, device="meta"),
                        requires_grad=False)


def _scales(experts: int, rows: int, groups: int) -> nn.Parameter:
    return nn.Parameter(torch.empty(experts, rows, groups, dtype=torch.uint8, device="meta"),
                        requires_grad=False)


class B200MXFP4Experts(nn.Module):
    """Drop-in for ``MXFP4Experts`` / ``GptOssExperts`` running the fused kernels.

    ``forward(hidden_states [T,H], router_indices [T,k], routing_weights [T,k]) -> [T,H]``
    (gptoss.py:137-142).  Parameters (gptoss.py:115-128) are created on ``meta``
    and bound by the caller (``functional_call``, ``load_state_dict(assign=True)``
    or ``.to_empty``).  The down projection's group count is I/32; the reference
    uses H/32 for both (gptoss.py:92), which is the same for gpt-oss (I == H).
    """

    def __init__(self, config, dtype: torch.dtype = torch.bfloat16, algo: int = kernels.ALGO_AUTO) -> None:
        super().__init__()
        self.num_experts = config.num_local_experts
        self.hidden_size = config.hidden_size
        self.expert_dim = config.intermediate_size
        self.alpha = 1.702
        self.limit = getattr(config, "swiglu_limit", 7.0)
        self.algo = algo
        E, H, I = self.num_experts, self.hidden_size, self.expert_dim
        self.gate_up_proj_blocks = _packed(E, 2 * I, H // 32)
        self.gate_up_proj_scales = _scales(E, 2 * I, H // 32)
        self.gate_up_proj_bias = nn.Parameter(torch.empty(E, 2 * I, dtype=dtype, device="meta"),
                                              requires_grad=False)
        self.down_proj_blocks = _packed(E, H, I // 32)
        self.down_proj_scales = _scales(E, H, I // 32)
        self.down_proj_bias = nn.Parameter(torch.empty(E, H, dtype=dtype, device="meta"),
                                           requires_grad=False)

    def forward(self, hidden_states: Tensor, router_indices: Tensor | None = None,
                routing_weights: Tensor | None = None) -> Tensor:
        if router_indices is None or routing_weights is None:
            raise ValueError("B200MXFP4Experts needs router_indices and routing_weights")
        if torch.is_grad_enabled() and (hidden_states.requires_grad or routing_weights.requires_grad):
            return _ExpertsFunction.apply(hidden_states, routing_weights, router_indices, self)
        k = router_indices.shape[-1]
        out, _, _ = kernels.moe_forward(
            hidden_states.to(torch.bfloat16), self.gate_up_proj_blocks, self.gate_up_proj_scales,
            self.gate_up_proj_bias, self.down_proj_blocks, self.down_proj_scales,
            self.down_proj_bias, k, indices=router_indices, scores=routing_weights,
            alpha=self.alpha, limit=self.limit, algo=self.algo)
        return out.to(hidden_states.dtype)


class _Router(nn.Module):
    """Holds ``router.weight`` [E,H] and ``router.bias`` [E] under the HF names."""

    def __init__(self, experts: int, hidden: int, dtype: torch.dtype) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.empty(experts, hidden, dtype=dtype, device="meta"))
        self.bias = nn.Parameter(torch.empty(experts, dtype=dtype, device="meta"))


class B200GptOssMLP(nn.Module):
    """Drop-in for transformers' ``GptOssMLP`` with packed experts.

    ``forward(hidden_states [B,S,H]) -> (out [B,S,H], router_scores [B*S,k])``
    (modeling_gpt_oss.py:140-146): router (fp32 accumulate, top-k, softmax over
    the k), dispatch, gate_up + SwiGLU, down, weighted combine — all on the GPU
    with no host synchronization.  ``router_scores`` has the router's dtype.
    """

    def __init__(self, config, dtype: torch.dtype = torch.bfloat16,
                 router_dtype: torch.dtype = torch.float32, algo: int = kernels.ALGO_AUTO) -> None:
        super().__init__()
        self.top_k = config.num_experts_per_tok
        self.router = _Router(config.num_local_experts, config.hidden_size, router_dtype)
        self.experts = B200MXFP4Experts(config, dtype, algo)

    def forward(self, hidden_states: Tensor):
        B, S, H = hidden_states.shape
        ex = self.experts
        router = self.router
        if torch.is_grad_enabled() and hidden_states.requires_grad:
            # differentiable form: router and experts as two autograd ops over
            # the library's kernels (forward and backward on the GPU); the
            # router's parameters get gradients too when they require them
            flat = hidden_states.reshape(-1, H)
            scores, idx = _RouterFunction.apply(flat, router.weight, router.bias, self.top_k)
            out = _ExpertsFunction.apply(flat, scores, idx, ex)
            return out.reshape(B, S, H), scores.to(router.weight.dtype)
        x = hidden_states.reshape(-1, H).to(torch.bfloat16)
        out, scores, _ = kernels.moe_forward(
            x, ex.gate_up_proj_blocks, ex.gate_up_proj_scales, ex.gate_up_proj_bias,
            ex.down_proj_blocks, ex.down_proj_scales, ex.down_proj_bias, self.top_k,
            router_weight=self.router.weight, router_bias=self.router.bias,
            alpha=ex.alpha, limit=ex.limit, algo=ex.algo)
        return out.reshape(B, S, H).to(hidden_states.dtype), scores.to(self.router.weight.dtype)


class _RMSNorm(nn.Module):
    """Holds ``weight`` [H] under GptOssRMSNorm's name; eps as its ``variance_epsilon``."""

    def __init__(self, hidden: int, eps: float, dtype: torch.dtype) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.empty(hidden, dtype=dtype, device="meta"))
        self.variance_epsilon = eps


class B200GptOssMoEBlock(nn.Module):
    """The MoE half of transformers' ``GptOssDecoderLayer`` fused around the layer:
    ``forward(hidden [B,S,H]) -> hidden + mlp(post_attention_layernorm(hidden))``
    (GptOssDecoderLayer.forward's "Fully Connected" part, modeling_gpt_oss.py),
    with the decoder layer's parameter names (``post_attention_layernorm.weight``,
    ``mlp.router.*``, ``mlp.experts.*``).  On the GPU path the norm is one kernel
    and the residual add happens in the layer's final combine."""

    def __init__(self, config, dtype: torch.dtype = torch.bfloat16, router_dtype: torch.dtype = torch.float32,
                 norm_dtype: torch.dtype = torch.float32, algo: int = kernels.ALGO_AUTO) -> None:
        super().__init__()
        self.post_attention_layernorm = _RMSNorm(config.hidden_size, getattr(config, "rms_norm_eps", 1e-5),
                                                 norm_dtype)
        self.mlp = B200GptOssMLP(config, dtype, router_dtype, algo)

    def forward(self, hidden_states: Tensor) -> Tensor:
        B, S, H = hidden_states.shape
        norm, mlp, ex = self.post_attention_layernorm, self.mlp, self.mlp.experts
        if torch.is_grad_enabled() and hidden_states.requires_grad:
            v = hidden_states.to(torch.float32)
            v = v * torch.rsqrt(v.pow(2).mean(-1, keepdim=True) + norm.variance_epsilon)
            normed = (norm.weight * v).to(hidden_states.dtype)
            out, _ = mlp(normed)
            return hidden_states + out
        out, _, _ = kernels.moe_block_forward(
            hidden_states.reshape(-1, H).to(torch.bfloat16), norm.weight, norm.variance_epsilon,
            ex.gate_up_proj_blocks, ex.gate_up_proj_scales, ex.gate_up_proj_bias, ex.down_proj_blocks,
            ex.down_proj_scales, ex.down_proj_bias, mlp.top_k, mlp.router.weight, mlp.router.bias,
            alpha=ex.alpha, limit=ex.limit, algo=ex.algo)
        return out.reshape(B, S, H).to(hidden_states.dtype)


def install_b200_experts(model: nn.Module, config, dtype=torch.bfloat16) -> int:
    """Swap every ``GptOssExperts`` / ``MXFP4Experts`` for ``B200MXFP4Experts``
    (the counterpart of gptoss.py:180-189)."""
    replaced = 0
    for layer in model.model.layers:
        name = type(layer.mlp.experts).__name__
        if name in ("GptOssExperts", "MXFP4Experts"):
            layer.mlp.experts = B200MXFP4Experts(config, dtype)
            replaced += 1
    return replaced


def install_b200_mlp(model: nn.Module, config, dtype=torch.bfloat16,
                     router_dtype: torch.dtype | None = None) -> int:
    """Swap every ``GptOssMLP`` for ``B200GptOssMLP`` (router + experts fused).
    Parameter names (``mlp.router.*``, ``mlp.experts.*``) are unchanged."""
    replaced = 0
    for layer in model.model.layers:
        if type(layer.mlp).__name__ == "GptOssMLP":
            rd = router_dtype or layer.mlp.router.weight.dtype
            layer.mlp = B200GptOssMLP(config, dtype, rd)
            replaced += 1
    return replaced
