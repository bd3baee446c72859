"""The CTA-pair grouped GEMM (BS_ALGO_TCGEN05_PAIR: tcgen05.mma.cta_group::2,
256 weight rows per MMA split over two CTAs, token rows split in halves)
against the one-CTA kernel (BS_ALGO_TCGEN05).

Both accumulate each output element over K in the same order in fp32 and
apply the same epilogue, so they must agree bit for bit; the one-CTA kernel
is itself checked against the fp32 oracle at these configurations
(tests/test_gpu_parity_configs.py, tests/test_gpu_layer.py).  Cases: the
benchmarked 120b (8192 tokens) and 20b (4096 tokens) layers, a skewed routing
whose hot expert spans three 320-row token chunks, weight rows that are not
a multiple of 256 (the last tile pair half empty), and mxfp4_matmul."""

import pytest
import torch

from blockstreamer_b200 import kernels
from blockstreamer_b200.synthetic import CASES, LayerShape, make_layer, make_tokens

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
NAMES = ("gate_up_proj_blocks", "gate_up_proj_scales", "gate_up_proj_bias", "down_proj_blocks",
         "down_proj_scales", "down_proj_bias")


def both_algos(p, x, idx):
    pe = [p["experts." + n] for n in NAMES]
    d = kernels.dispatch(idx, pe[0].shape[0], x)
    outs = []
    for algo in (kernels.ALGO_TCGEN05, kernels.ALGO_TCGEN05_PAIR):
        h = kernels.moe_gate_up(d.x_perm, d.expert_offsets, *pe[:3], algo=algo)
        y = kernels.moe_down(h, d.expert_offsets, *pe[3:], algo=algo)
        outs.append((h, y))
    torch.cuda.synchronize()
    assert kernels.device_status(clear=True) == 0
    return outs


@pytest.mark.parametrize("key,case_id,T", [("gptoss120b", 4, 8192), ("gptoss20b", 2, 4096)],
                         ids=["120b-prefill-8192", "20b-prefill-4096"])
def test_pair_kernel_equals_one_cta_kernel_at_bench_configs(key, case_id, T):
    shape = CASES[key]
    p = make_layer(shape, case_id, device=DEV)
    x = make_tokens(T, shape.hidden, case_id, device=DEV)
    _, _, idx = kernels.router(x, p["router.weight"], p["router.bias"], shape.top_k, index_dtype=torch.int32)
    (h1, y1), (h2, y2) = both_algos(p, x, idx)
    assert torch.equal(h1, h2)
    assert torch.equal(y1, y2)


def test_pair_kernel_multichunk_and_partial_pairs():
    # H = 384: down has 384 weight rows = 1.5 tile pairs; expert 3 takes 700 rows (3 chunks)
    shape = LayerShape(384, 512, 16, 2)
    T = 700
    p = make_layer(shape, 43, device=DEV)
    x = make_tokens(T, shape.hidden, 43, device=DEV)
    idx = torch.zeros(T, 2, dtype=torch.int32)
    idx[:, 0] = 3
    idx[:, 1] = torch.arange(T, dtype=torch.int32) % 5 + 6
    (h1, y1), (h2, y2) = both_algos(p, x, idx.to(DEV))
    assert torch.equal(h1, h2)
    assert torch.equal(y1, y2)


@pytest.mark.parametrize("m,K,N", [(300, 2880, 5760), (37, 512, 384)])
def test_pair_kernel_mxfp4_matmul(m, K, N):
    g = torch.Generator().manual_seed(m)
    blocks = torch.randint(0, 256, (N, K // 32, 16), dtype=torch.uint8, generator=g).to(DEV)
    scales = torch.randint(120, 132, (N, K // 32), dtype=torch.uint8, generator=g).to(DEV)
    x = torch.randn(m, K, generator=g).to(torch.bfloat16).to(DEV)
    a = kernels.mxfp4_matmul(x, blocks, scales, algo=kernels.ALGO_TCGEN05)
    b = kernels.mxfp4_matmul(x, blocks, scales, algo=kernels.ALGO_TCGEN05_PAIR)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    assert kernels.device_status(clear=True) == 0
