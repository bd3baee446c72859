"""CPU restatement of the gpt-oss MoE layer — test infrastructure only.

Three evaluations of the same layer, all on the CPU with torch tensors:

``router``        transformers ``GptOssTopKRouter.forward``
                  (models/gpt_oss/modeling_gpt_oss.py:126-130): ``F.linear`` in fp32,
                  ``topk`` (sorted descending), softmax over the k selected logits.
``experts_port``  ``block_streamer/gptoss.py:137-177`` (``MXFP4Experts.forward``)
                  with the reference's own rounding points: per hit expert in
                  ascending order, dequant to bf16 (gptoss.py:24-42), bf16 GEMM +
                  bf16 bias (158-165), the clamped interleaved SwiGLU in bf16
                  (130-135), bf16 down GEMM + bias (167-174), scale by the fp32
                  routing weight and round to bf16 (175), ``index_add_`` into a bf16
                  accumulator (176).  This is the CPU baseline ("port").
``experts_fp32``  the same math with every value in fp32 (exact dequant, fp32
                  GEMMs, fp32 SwiGLU, fp32 weighted sum): the accuracy target.

The weight format is the checkpoint's: ``gate_up_proj_blocks`` [E, 2I, G, 16] u8,
``gate_up_proj_scales`` [E, 2I, G] u8, ``gate_up_proj_bias`` [E, 2I],
``down_proj_blocks`` [E, H, G, 16], ``down_proj_scales`` [E, H, G],
``down_proj_bias`` [E, H]  (gptoss.py:115-128; note G = H // 32 is used for the
down projection too, gptoss.py:92, which is only valid when I == H).
"""

from __future__ import annotations

from typing import Mapping

import torch
import torch.nn.functional as F

ALPHA = 1.702   # gptoss.py:90
LIMIT = 7.0     # gptoss.py:91 (swiglu_limit default)

_FP4 = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                     -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], dtype=torch.float64)


def dequant_expert(blocks: torch.Tensor, scales: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """One expert [rows, G, 16] u8 + [rows, G] u8 -> dense [G*32, rows] in ``dtype``.

    Exact product in float64, rounded once to ``dtype`` (products >= 2**128 go to
    +-inf). This equals transformers' LUT + ldexp result bit for bit
    (integrations/mxfp4.py:305-330; pinned by tests/test_oracle.py).  Runs on
    the tensors' device (a test may evaluate the oracle where its inputs are).
    """
    rows, groups, _ = blocks.shape
    b = blocks.to(torch.int64)
    # float32 is exact for every scale <= 254 (2**127 is representable and the
    # product overflows to inf exactly when the reference's does); scale 255
    # needs the wider type because 2**128 itself overflows float32.
    wide = bool((scales == 255).any())
    ft = torch.float64 if wide else torch.float32
    lut = _FP4.to(device=blocks.device, dtype=ft)
    vals = torch.empty(rows, groups, 32, dtype=ft, device=blocks.device)
    vals[..., 0::2] = lut[b & 0x0F]
    vals[..., 1::2] = lut[b >> 4]
    vals = vals * torch.pow(2.0, (scales.to(torch.int64) - 127).unsqueeze(-1).to(ft))
    vals = vals.to(torch.float32).to(dtype)
    return vals.reshape(rows, groups * 32).t().contiguous()


def router(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, top_k: int):
    """Returns (logits [T,E], scores [T,k], indices [T,k] int64), computed like the
    reference router on ``x`` in the router's dtype (modeling_gpt_oss.py:126-130)."""
    logits = F.linear(x.to(weight.dtype), weight, bias)
    top_value, top_index = torch.topk(logits, top_k, dim=-1)
    scores = torch.softmax(top_value, dim=1, dtype=top_value.dtype)
    return logits, scores, top_index


def router_logits_f64(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    """Router logits accumulated in float64 (used to find near-ties)."""
    return x.double() @ weight.double().t() + bias.double()


def near_tie_tokens(logits_f64: torch.Tensor, top_k: int, eps: float = 1e-6,
                    *approx_logits: torch.Tensor) -> torch.Tensor:
    """Bool [T]: tokens whose top-k selection is not decidable.

    A token is a near-tie when the gap between its k-th and (k+1)-th exact
    (fp64) logits, or between two of its selected logits, is at most ``eps``
    widened by the logit errors, on that token, of the fp32 implementations
    being compared (``approx_logits``, each [T, E]): an ordering closer than
    the sum of those errors can legitimately come out either way.
    """
    srt = torch.sort(logits_f64, dim=-1, descending=True).values
    gap_k = srt[:, top_k - 1] - srt[:, top_k] if srt.shape[1] > top_k else torch.full_like(srt[:, 0], 1.0)
    inner = (srt[:, : top_k - 1] - srt[:, 1:top_k]).abs().min(dim=-1).values if top_k > 1 else torch.full_like(srt[:, 0], 1.0)
    band = torch.full_like(gap_k, eps)
    for a in approx_logits:
        band = band + (a.double() - logits_f64).abs().max(dim=-1).values
    return (gap_k <= band) | (inner <= band)


# Stated bound on the library router's logit error (both its tensor-core and
# CUDA-core forms measure below 1.5e-5 at H = 2880); used to widen the tie band
# where a test compares routings without the library's logits.
ROUTER_LOGIT_ERR = 2e-5


def _apply_gate_bf16(gate_up: torch.Tensor, limit: float, alpha: float) -> torch.Tensor:
    """gptoss.py:130-135 in the tensor's own dtype."""
    gate, up = gate_up[..., ::2], gate_up[..., 1::2]
    gate = gate.clamp(max=limit)
    up = up.clamp(min=-limit, max=limit)
    glu = gate * torch.sigmoid(gate * alpha)
    return (up + 1) * glu


def expert_rows(indices: torch.Tensor, expert: int):
    """(top_k_pos, token_idx) for one expert in the reference's order: ``torch.where``
    over the [k, T] one-hot slice (gptoss.py:145-153), i.e. by slot, then token."""
    slot_tok = (indices.t() == expert)
    top_k_pos, token_idx = torch.where(slot_tok)
    return top_k_pos, token_idx


def experts_port(hidden: torch.Tensor, indices: torch.Tensor, weights: torch.Tensor,
                 p: Mapping[str, torch.Tensor], limit: float = LIMIT, alpha: float = ALPHA,
                 experts_subset=None) -> torch.Tensor:
    """Reference-order bf16 evaluation of ``MXFP4Experts.forward`` (gptoss.py:137-177).

    ``experts_subset`` restricts the loop to the given experts (for bounded CPU
    timing samples); the default runs every hit expert.
    """
    dtype = hidden.dtype
    E = p["gate_up_proj_blocks"].shape[0]
    out = torch.zeros_like(hidden)
    hit = sorted(set(indices.reshape(-1).tolist()))
    if experts_subset is not None:
        hit = [e for e in hit if e in set(experts_subset)]
    for e in hit:
        if e == E:
            continue
        top_k_pos, token_idx = expert_rows(indices, e)
        cur = hidden[token_idx]
        w_gu = dequant_expert(p["gate_up_proj_blocks"][e], p["gate_up_proj_scales"][e], dtype)
        gate_up = cur @ w_gu + p["gate_up_proj_bias"][e]
        gated = _apply_gate_bf16(gate_up, limit, alpha)
        w_d = dequant_expert(p["down_proj_blocks"][e], p["down_proj_scales"][e], dtype)
        y = gated @ w_d + p["down_proj_bias"][e]
        y = y * weights[token_idx, top_k_pos, None]
        out.index_add_(0, token_idx, y.to(dtype))
    return out


def experts_fp32(hidden: torch.Tensor, indices: torch.Tensor, weights: torch.Tensor,
                 p: Mapping[str, torch.Tensor], limit: float = LIMIT, alpha: float = ALPHA,
                 return_intermediates: bool = False, experts_subset=None):
    """The reference math with every value in fp32; returns out [T, H] fp32.

    With ``return_intermediates`` also returns a dict keyed by expert with the
    (token_idx, top_k_pos, h [rows, I] fp32, y [rows, H] fp32) of each hit expert.
    ``experts_subset`` restricts the loop to the given experts (``out`` then
    holds only their contributions).  Evaluated on ``hidden``'s device (every
    input must be there); fp32 matmuls must not be run in TF32.
    """
    x = hidden.float()
    T, H = x.shape
    E = p["gate_up_proj_blocks"].shape[0]
    out = torch.zeros(T, H, dtype=torch.float32, device=x.device)
    inter = {}
    hit = sorted(set(indices.reshape(-1).tolist()))
    if experts_subset is not None:
        keep = set(int(e) for e in experts_subset)
        hit = [e for e in hit if e in keep]
    for e in hit:
        if e == E:
            continue
        top_k_pos, token_idx = expert_rows(indices, e)
        cur = x[token_idx]
        w_gu = dequant_expert(p["gate_up_proj_blocks"][e], p["gate_up_proj_scales"][e], torch.float32)
        g = cur @ w_gu + p["gate_up_proj_bias"][e].float()
        gate, up = g[:, ::2].clamp(max=limit), g[:, 1::2].clamp(min=-limit, max=limit)
        h = (up + 1.0) * (gate * torch.sigmoid(gate * alpha))
        w_d = dequant_expert(p["down_proj_blocks"][e], p["down_proj_scales"][e], torch.float32)
        y = h @ w_d + p["down_proj_bias"][e].float()
        out.index_add_(0, token_idx, y * weights[token_idx, top_k_pos, None].float())
        if return_intermediates:
            inter[e] = (token_idx, top_k_pos, h, y)
    if return_intermediates:
        return out, inter
    return out


def mlp_port(hidden: torch.Tensor, router_weight: torch.Tensor, router_bias: torch.Tensor,
             p: Mapping[str, torch.Tensor], top_k: int, **kw):
    """``GptOssMLP.forward`` (modeling_gpt_oss.py:140-146) over [T, H] tokens with
    the bf16 expert port; returns (out, scores, indices)."""
    _, scores, idx = router(hidden, router_weight, router_bias, top_k)
    return experts_port(hidden, idx, scores, p, **kw), scores, idx


def rel_l2(a: torch.Tensor, b: torch.Tensor) -> float:
    a = a.double()
    b = b.double()
    return float((a - b).norm() / b.norm().clamp_min(1e-300))
