"""Seeded synthetic gpt-oss MoE layers and tokens.

No gpt-oss checkpoint exists offline, so every benchmark and parity case runs on
synthetic tensors with the checkpoint's names, shapes and dtypes
(``block_streamer/gptoss.py:115-128`` for the experts,
``transformers/models/gpt_oss/modeling_gpt_oss.py:117-124`` for the router):

* e2m1 codes uniform over all 16 values (uniform random bytes);
* e8m0 scales uniform over an inclusive byte range;
* bf16 biases ~ N(0, 0.02); fp32 router weight ~ N(0, 0.02), bias ~ N(0, sigma_b);
* tokens bf16 ~ N(0, 1).

Each tensor has its own ``torch.Generator`` seeded ``1000 * case + tensor_id`` so
that any single tensor can be regenerated on its own. Generators on different
devices give different streams: parity cases are generated on the CPU and moved.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch


@dataclass(frozen=True)
class LayerShape:
    hidden: int          # H
    intermediate: int    # I
    experts: int         # E
    top_k: int           # k
    scale_lo: int = 124  # inclusive e8m0 range of the expert scales
    scale_hi: int = 130
    router_std: float = 0.02
    router_bias_std: float = 0.01
    swiglu_limit: float = 7.0

    @property
    def groups(self) -> int:
        return self.hidden // 32


# The five cases of the benchmark specification.
CASES = {
    "tiny": LayerShape(256, 256, 8, 2, 124, 130, 0.02, 0.01),
    "gptoss20b": LayerShape(2880, 2880, 32, 4, 120, 128, 0.02, 0.02),
    "gptoss120b": LayerShape(2880, 2880, 128, 4, 124, 130, 0.02, 0.01),
}


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def make_layer(shape: LayerShape, case_id: int, device="cpu") -> dict[str, torch.Tensor]:
    """Router + expert tensors under the reference's parameter names."""
    H, I, E = shape.hidden, shape.intermediate, shape.experts
    G = shape.groups
    s = 1000 * case_id
    dev = torch.device(device)

    def u8(n, shp, lo, hi):
        return torch.randint(lo, hi + 1, shp, generator=_gen(s + n, dev), dtype=torch.uint8, device=dev)

    def normal(n, shp, std, dtype):
        return (torch.randn(shp, generator=_gen(s + n, dev), dtype=torch.float32, device=dev) * std).to(dtype)

    return {
        "router.weight": normal(1, (E, H), shape.router_std, torch.float32),
        "router.bias": normal(2, (E,), shape.router_bias_std, torch.float32),
        "experts.gate_up_proj_blocks": u8(3, (E, 2 * I, G, 16), 0, 255),
        "experts.gate_up_proj_scales": u8(4, (E, 2 * I, G), shape.scale_lo, shape.scale_hi),
        "experts.gate_up_proj_bias": normal(5, (E, 2 * I), 0.02, torch.bfloat16),
        "experts.down_proj_blocks": u8(6, (E, H, I // 32, 16), 0, 255),
        "experts.down_proj_scales": u8(7, (E, H, I // 32), shape.scale_lo, shape.scale_hi),
        "experts.down_proj_bias": normal(8, (E, H), 0.02, torch.bfloat16),
    }


def make_tokens(T: int, H: int, case_id: int, device="cpu", stream: int = 0) -> torch.Tensor:
    """bf16 tokens ~ N(0, 1), [T, H]."""
    g = _gen(1000 * case_id + 100 + stream, torch.device(device))
    return torch.randn((T, H), generator=g, dtype=torch.float32, device=device).to(torch.bfloat16)


def zipf_router_bias(shape: LayerShape, zipf_s: float, case_id: int, logit_scale: float = 1.0) -> torch.Tensor:
    """Router bias that makes expert popularity follow Zipf(s) over a seeded random
    permutation of the experts: bias_e = log(p_rank(e)) * logit_scale, where
    p_r ~ 1 / r**s (the softmax-of-logits view of top-1 selection)."""
    E = shape.experts
    perm = torch.randperm(E, generator=_gen(1000 * case_id + 50, torch.device("cpu")))
    ranks = torch.empty(E, dtype=torch.float64)
    ranks[perm] = torch.arange(1, E + 1, dtype=torch.float64)
    p = ranks.pow(-zipf_s)
    p = p / p.sum()
    return (p.log() * logit_scale).to(torch.float32)


def algorithmic_flops(T: int, shape: LayerShape) -> float:
    """Router 2*H*E per token + 6*H*I per routed (token, expert) pair."""
    return T * (2.0 * shape.hidden * shape.experts + shape.top_k * 6.0 * shape.hidden * shape.intermediate)


def expert_bytes(shape: LayerShape) -> int:
    """Packed bytes of one expert (blocks + scales + bias, both projections)."""
    H, I, G = shape.hidden, shape.intermediate, shape.groups
    gu = 2 * I * G * 16 + 2 * I * G + 2 * I * 2
    Gd = I // 32
    dn = H * Gd * 16 + H * Gd + H * 2
    return gu + dn


def algorithmic_bytes(T: int, shape: LayerShape, distinct_experts: int) -> int:
    """Weights once per distinct expert touched + router weights + tokens in/out (bf16)."""
    router = shape.experts * shape.hidden * 4 + shape.experts * 4
    return distinct_experts * expert_bytes(shape) + router + 2 * T * shape.hidden * 2
