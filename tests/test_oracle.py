"""Pin the CPU oracle to the reference's own outputs (golden fixtures).

The fixtures were produced by ``tests/golden/make_golden.py`` running the
reference (``block_streamer.gptoss`` + transformers' gpt-oss router) on seeded
inputs; these tests need no GPU and no reference install.
"""

import hashlib
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from blockstreamer_b200.synthetic import CASES, make_layer, make_tokens
from oracle import mxfp4
from oracle import moe

LAYER_CASES = [("tiny", "tiny"), ("gptoss20b_t4", "gptoss20b"), ("gptoss120b_t3", "gptoss120b")]


def _sha(t):
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def _load(name):
    return np.load(os.path.join(GOLDEN, name))


def test_dequant_sweep_bit_exact():
    """All 256 byte values x all 256 e8m0 scales, against dequantize_expert."""
    golden = _load("dequant_sweep.npz")["bits"]
    rows, groups = 256, 16
    b = np.arange(256, dtype=np.uint8).reshape(groups, 16)
    blocks = np.broadcast_to(b, (1, rows, groups, 16)).copy()
    scales = np.broadcast_to(np.arange(256, dtype=np.uint8)[:, None], (1, rows, groups)).copy()
    bits = mxfp4.dequant_bf16_bits(blocks, scales)[0]
    assert bits.shape == golden.shape == (512, 256)
    assert np.array_equal(bits, golden)
    # torch form used by the expert port agrees too
    t = moe.dequant_expert(torch.from_numpy(blocks[0]), torch.from_numpy(scales[0]), torch.bfloat16)
    assert np.array_equal(t.view(torch.int16).numpy().astype(np.uint16), golden)


def test_dequant_edge_values():
    # 0.5 * 2**-127 is a bf16 subnormal; 6 * 2**127 overflows to inf; 0 * 2**128 stays 0
    assert mxfp4.e2m1_bf16_bits(1, 0) == 0x0020
    assert mxfp4.e2m1_bf16_bits(7, 254) == 0x7F80
    assert mxfp4.e2m1_bf16_bits(15, 254) == 0xFF80
    assert mxfp4.e2m1_bf16_bits(0, 255) == 0x0000
    assert mxfp4.e2m1_bf16_bits(8, 127) == 0x8000   # -0.0 keeps its sign
    assert mxfp4.e2m1_bf16_bits(2, 127) == 0x3F80


def test_dequant_orientation_matches_reference_test():
    """Mirrors the reference's own CPU test (tests/test_offload.py:405-414):
    [1, rows, groups, 16] -> [groups * 32, rows]."""
    g = torch.Generator().manual_seed(0)
    blocks = torch.randint(0, 255, (1, 64, 4, 16), dtype=torch.uint8, generator=g)
    scales = torch.randint(120, 134, (1, 64, 4), dtype=torch.uint8, generator=g)
    out = mxfp4.dequant_f32(blocks.numpy(), scales.numpy())
    assert out.shape == (1, 128, 64)


@pytest.mark.parametrize("name,key", LAYER_CASES)
def test_inputs_regenerate_identically(name, key):
    gold = _load(f"layer_{name}.npz")
    cid, T = int(gold["case"][0]), int(gold["tokens"][0])
    shape = CASES[key]
    p = make_layer(shape, cid)
    x = make_tokens(T, shape.hidden, cid)
    assert _sha(x) == str(gold["sha_x"][0])
    for k, v in p.items():
        assert _sha(v) == str(gold["sha_" + k.replace(".", "_")][0]), k


@pytest.mark.parametrize("name,key", LAYER_CASES)
def test_router_matches_reference(name, key):
    gold = _load(f"layer_{name}.npz")
    cid, T = int(gold["case"][0]), int(gold["tokens"][0])
    shape = CASES[key]
    p = make_layer(shape, cid)
    x = make_tokens(T, shape.hidden, cid)
    logits, scores, idx = moe.router(x.float(), p["router.weight"], p["router.bias"], shape.top_k)
    assert np.array_equal(logits.numpy(), gold["logits"])
    assert np.array_equal(idx.numpy(), gold["indices"])
    assert np.array_equal(scores.numpy(), gold["scores"])


@pytest.mark.parametrize("name,key", LAYER_CASES)
def test_expert_port_bit_exact_vs_reference(name, key):
    """The bf16 port reproduces MXFP4Experts.forward bit for bit."""
    gold = _load(f"layer_{name}.npz")
    cid, T = int(gold["case"][0]), int(gold["tokens"][0])
    shape = CASES[key]
    p = {k.split(".", 1)[1]: v for k, v in make_layer(shape, cid).items() if k.startswith("experts.")}
    x = make_tokens(T, shape.hidden, cid)
    idx = torch.from_numpy(gold["indices"])
    w = torch.from_numpy(gold["scores"])
    out = moe.experts_port(x, idx, w, p)
    assert np.array_equal(out.view(torch.int16).numpy().astype(np.uint16), gold["out_bits"])


@pytest.mark.parametrize("name,key", LAYER_CASES)
def test_fp32_oracle_calibration(name, key):
    """The reference bf16 output sits within the layer tolerance of the fp32
    evaluation (this is the calibration line for the CUDA path's own error)."""
    gold = _load(f"layer_{name}.npz")
    cid, T = int(gold["case"][0]), int(gold["tokens"][0])
    shape = CASES[key]
    p = {k.split(".", 1)[1]: v for k, v in make_layer(shape, cid).items() if k.startswith("experts.")}
    x = make_tokens(T, shape.hidden, cid)
    idx = torch.from_numpy(gold["indices"])
    w = torch.from_numpy(gold["scores"])
    ref = torch.from_numpy(gold["out_bits"].astype(np.int16)).view(torch.bfloat16).float()
    f32 = moe.experts_fp32(x, idx, w, p)
    assert moe.rel_l2(ref, f32) < 5e-3
