"""GPU parity of the individual kernels against the CPU oracle and the
reference's golden fixtures (all calls go through the C ABI)."""

import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from blockstreamer_b200 import kernels
from blockstreamer_b200.synthetic import CASES, make_layer, make_tokens
from oracle import moe as omoe
from oracle import mxfp4 as omx

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def bits(t):
    return t.contiguous().view(torch.int16).cpu().numpy().astype(np.uint16)


# ------------------------------------------------------------------ dequant

def test_dequant_sweep_bit_exact_against_reference():
    golden = np.load(os.path.join(GOLDEN, "dequant_sweep.npz"))["bits"]
    b = np.arange(256, dtype=np.uint8).reshape(16, 16)
    blocks = torch.from_numpy(np.broadcast_to(b, (1, 256, 16, 16)).copy()).to(DEV)
    scales = torch.from_numpy(np.broadcast_to(np.arange(256, dtype=np.uint8)[:, None], (1, 256, 16)).copy()).to(DEV)
    out = kernels.dequant_mxfp4(blocks, scales, transpose=True)
    assert np.array_equal(bits(out[0]), golden)
    nat = kernels.dequant_mxfp4(blocks, scales, transpose=False)
    assert np.array_equal(bits(nat[0]).T, golden)


@pytest.mark.parametrize("E,R,G,lo,hi", [(2, 64, 4, 120, 133), (3, 100, 90, 0, 255), (1, 5760, 90, 124, 130)])
def test_dequant_random_experts_bit_exact(E, R, G, lo, hi):
    g = torch.Generator().manual_seed(E * 1000 + R)
    blocks = torch.randint(0, 256, (E, R, G, 16), dtype=torch.uint8, generator=g)
    scales = torch.randint(lo, hi + 1, (E, R, G), dtype=torch.uint8, generator=g)
    want = omx.dequant_bf16_bits(blocks.numpy(), scales.numpy())
    got = kernels.dequant_mxfp4(blocks.to(DEV), scales.to(DEV))
    assert np.array_equal(bits(got), want)


def test_dequantize_expert_orientation_like_reference_test():
    from blockstreamer_b200 import dequantize_expert
    g = torch.Generator().manual_seed(0)
    blocks = torch.randint(0, 255, (1, 64, 4, 16), dtype=torch.uint8, generator=g).to(DEV)
    scales = torch.randint(120, 134, (1, 64, 4), dtype=torch.uint8, generator=g).to(DEV)
    out = dequantize_expert(blocks, scales, torch.float32)
    assert out.shape == (128, 64)
    want = omx.dequant_f32(blocks.cpu().numpy(), scales.cpu().numpy())[0]
    assert np.array_equal(out.cpu().numpy(), want)


# ------------------------------------------------------------------ router

LAYER_CASES = [("tiny", "tiny"), ("gptoss20b_t4", "gptoss20b"), ("gptoss120b_t3", "gptoss120b")]


@pytest.mark.parametrize("name,key", LAYER_CASES)
@pytest.mark.parametrize("want_logits", [True, False])
def test_router_matches_reference_golden(name, key, want_logits):
    gold = np.load(os.path.join(GOLDEN, f"layer_{name}.npz"))
    cid, T = int(gold["case"][0]), int(gold["tokens"][0])
    shape = CASES[key]
    p = make_layer(shape, cid)
    x = make_tokens(T, shape.hidden, cid)
    logits, scores, idx = kernels.router(x.to(DEV), p["router.weight"].to(DEV), p["router.bias"].to(DEV),
                                         shape.top_k, return_logits=True)
    f64 = omoe.router_logits_f64(x, p["router.weight"], p["router.bias"])
    ties = omoe.near_tie_tokens(f64, shape.top_k, 1e-6, torch.from_numpy(gold["logits"]), logits.cpu())
    keep = ~ties.numpy()
    assert (logits.cpu().double() - f64).abs().max() <= omoe.ROUTER_LOGIT_ERR
    assert np.array_equal(idx.cpu().numpy()[keep], gold["indices"][keep])
    np.testing.assert_allclose(scores.cpu().numpy()[keep], gold["scores"][keep], rtol=0, atol=1e-5)
    if want_logits:
        np.testing.assert_allclose(logits.cpu().numpy(), gold["logits"], rtol=1e-5, atol=2e-5)


@pytest.mark.parametrize("T", [1, 5, 8, 33, 700, 8192])
@pytest.mark.parametrize("E,k", [(128, 4), (32, 4), (8, 2)])
@pytest.mark.parametrize("use_ws", [True, False], ids=["ws", "nows"])
def test_router_against_oracle(T, E, k, use_ws):
    """With a workspace and T > 64 the tensor-core form runs (split fp32 weight);
    without, the fp32 CUDA-core forms.  Both must match the reference router."""
    H = 2880
    g = torch.Generator().manual_seed(T * 7 + E)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    W = torch.randn(E, H, generator=g) * 0.02
    b = torch.randn(E, generator=g) * 0.01
    lg_ref, s_ref, i_ref = omoe.router(x.float(), W, b, k)
    f64 = omoe.router_logits_f64(x, W, b)
    lg, s, i = kernels.router(x.to(DEV), W.to(DEV), b.to(DEV), k, return_logits=True,
                              use_workspace=use_ws)
    err = (lg.cpu().double() - f64).abs().max().item()
    print(f"router T={T} E={E} ws={use_ws}: max logit error {err:.2e}")
    assert err <= omoe.ROUTER_LOGIT_ERR
    keep = ~omoe.near_tie_tokens(f64, k, 1e-6, lg_ref, lg.cpu()).numpy()
    assert keep.sum() >= 0.99 * T
    assert np.array_equal(i.cpu().numpy()[keep], i_ref.numpy()[keep])
    np.testing.assert_allclose(s.cpu().numpy()[keep], s_ref.numpy()[keep], rtol=0, atol=1e-5)
    # without the logits output (at small T a different CUDA-core kernel) the routing agrees
    _, s2, i2 = kernels.router(x.to(DEV), W.to(DEV), b.to(DEV), k, use_workspace=use_ws)
    assert np.array_equal(i2.cpu().numpy()[keep], i_ref.numpy()[keep])
    np.testing.assert_allclose(s2.cpu().numpy()[keep], s_ref.numpy()[keep], rtol=0, atol=1e-5)


@pytest.mark.parametrize("T", [64, 300])
def test_router_bf16_weights_round_logits_like_reference(T):
    """A bf16 router (the real checkpoint's dtype) computes logits in bf16."""
    H, E, k = 2880, 32, 4
    g = torch.Generator().manual_seed(5)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    W = (torch.randn(E, H, generator=g) * 0.02).to(torch.bfloat16)
    b = (torch.randn(E, generator=g) * 0.01).to(torch.bfloat16)
    logits, s, i = kernels.router(x.to(DEV), W.to(DEV), b.to(DEV), k, return_logits=True)
    lg = logits.cpu()
    assert torch.equal(lg, lg.to(torch.bfloat16).float())   # logits are bf16 values
    ref = (x.double() @ W.double().t() + b.double()).float()
    assert (lg - ref).abs().max() <= ref.abs().max() * 2 ** -7


# ------------------------------------------------------------------ dispatch / combine

@pytest.mark.parametrize("T,E,k", [(1, 128, 4), (64, 8, 2), (300, 32, 4), (2049, 128, 4)])
@pytest.mark.parametrize("idx_dtype", [torch.int32, torch.int64])
def test_dispatch_is_a_stable_grouping(T, E, k, idx_dtype):
    g = torch.Generator().manual_seed(T + E)
    idx = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).to(idx_dtype)
    H = 256
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    d = kernels.dispatch(idx.to(DEV), E, x.to(DEV))
    off = d.expert_offsets.cpu().long()
    cnt = torch.bincount(idx.reshape(-1).long(), minlength=E)
    assert off[0] == 0 and torch.equal(off[1:] - off[:-1], cnt) and off[-1] == T * k
    ros = d.row_of_slot.cpu().long()
    assert torch.equal(torch.sort(ros).values, torch.arange(T * k))
    tor = d.token_of_row.cpu().long()
    slots = torch.arange(T * k)
    assert torch.equal(tor[ros], slots // k)
    # rows of each expert keep (token, slot) order
    for e in range(E):
        rows = torch.arange(off[e], off[e + 1])
        slot_of_row = torch.empty(T * k, dtype=torch.long)
        slot_of_row[ros] = slots
        s = slot_of_row[rows]
        assert torch.all(s[1:] > s[:-1])
        assert torch.all(idx.reshape(-1)[s].long() == e)
    assert torch.equal(d.x_perm.cpu(), x[tor])


def test_dispatch_flags_out_of_range_indices():
    idx = torch.tensor([[0, 1], [2, 9]], dtype=torch.int32, device=DEV)
    kernels.device_status(clear=True)
    d = kernels.dispatch(idx, 4)
    assert kernels.device_status(clear=True) == 1  # BS_ERR_INVALID_ARGUMENT recorded
    assert d.row_of_slot.cpu().tolist()[3] == -1


@pytest.mark.parametrize("T,k,H", [(1, 4, 2880), (37, 2, 256), (1000, 4, 2880)])
def test_combine_against_fp32(T, k, H):
    g = torch.Generator().manual_seed(T)
    y = torch.randn(T * k, H, generator=g).to(torch.bfloat16)
    ros = torch.randperm(T * k, generator=g).to(torch.int32)
    w = torch.rand(T, k, generator=g)
    out = kernels.combine(y.to(DEV), ros.to(DEV), w.to(DEV), T).cpu()
    ref = (y.float()[ros.long()].reshape(T, k, H) * w[..., None]).sum(1)
    # one bf16 rounding of an fp32 sum
    assert torch.equal(out, ref.to(torch.bfloat16)) or (out.float() - ref).abs().max() <= ref.abs().max() * 2 ** -8
