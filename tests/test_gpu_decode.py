"""GPU parity of the decode path (bs_moe_forward with BS_ALGO_MX, T <= 64):
router + dispatch in one launch, expert projections on tcgen05 block-scaled
MMAs (kind::mxf4) over the stored e2m1 codes, activations as four e2m1 terms.

Same bars as the other layer tests: routing exact away from near-ties with
weights within 1e-5, layer output rel-L2 <= 5e-3 and max-abs <= 2e-2 * max|y|
against the fp32 evaluation of the reference math.  The four-term split keeps
dot products within ~1e-4 relative, so the expected error is that of the bf16
output rounding; the tests also hold it to 2x the reference's own bf16 error
on the golden cases.
"""

import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from blockstreamer_b200 import kernels
from blockstreamer_b200.synthetic import CASES, LayerShape, make_layer, make_tokens
from oracle import moe as omoe

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
MX = kernels.ALGO_MX
LAYER_CASES = [("tiny", "tiny"), ("gptoss20b_t4", "gptoss20b"), ("gptoss120b_t3", "gptoss120b")]


def experts_of(p):
    return {k.split(".", 1)[1]: v for k, v in p.items() if k.startswith("experts.")}


def forward(x, pe, k, **kw):
    g = {n: t.to(DEV) for n, t in pe.items()}
    kw = {n: (v.to(DEV) if isinstance(v, torch.Tensor) else v) for n, v in kw.items()}
    out, sc, idx = kernels.moe_forward(x.to(DEV), g["gate_up_proj_blocks"], g["gate_up_proj_scales"],
                                       g["gate_up_proj_bias"], g["down_proj_blocks"],
                                       g["down_proj_scales"], g["down_proj_bias"], k, algo=MX, **kw)
    torch.cuda.synchronize()
    return out.cpu(), sc.cpu(), idx.cpu()


def check_close(out, ref_f32, label):
    rel = omoe.rel_l2(out.float(), ref_f32)
    mx = (out.float() - ref_f32).abs().max().item()
    scale = ref_f32.abs().max().item()
    print(f"{label}: rel_l2={rel:.3e} max_abs={mx:.3e} max_abs/max|y|={mx / scale:.3e}")
    assert rel <= 5e-3, label
    assert mx <= 2e-2 * scale, label
    return rel


@pytest.mark.parametrize("name,key", LAYER_CASES)
def test_decode_experts_vs_reference_golden(name, key):
    gold = np.load(os.path.join(GOLDEN, f"layer_{name}.npz"))
    cid, T = int(gold["case"][0]), int(gold["tokens"][0])
    shape = CASES[key]
    pe = experts_of(make_layer(shape, cid))
    x = make_tokens(T, shape.hidden, cid)
    idx = torch.from_numpy(gold["indices"])
    w = torch.from_numpy(gold["scores"])
    out, _, _ = forward(x, pe, shape.top_k, indices=idx, scores=w)
    f32 = omoe.experts_fp32(x, idx, w, pe)
    rel = check_close(out, f32, f"decode {name} vs fp32")
    ref = torch.from_numpy(gold["out_bits"].astype(np.int16)).view(torch.bfloat16).float()
    assert rel <= max(2 * omoe.rel_l2(ref, f32), 1e-3)


@pytest.mark.parametrize("name,key", LAYER_CASES)
def test_decode_full_mlp_vs_oracle(name, key):
    gold = np.load(os.path.join(GOLDEN, f"layer_{name}.npz"))
    cid, T = int(gold["case"][0]), int(gold["tokens"][0])
    shape = CASES[key]
    p = make_layer(shape, cid)
    x = make_tokens(T, shape.hidden, cid)
    out, sc, idx = forward(x, experts_of(p), shape.top_k, router_weight=p["router.weight"].to(DEV),
                           router_bias=p["router.bias"].to(DEV))
    f64 = omoe.router_logits_f64(x, p["router.weight"], p["router.bias"])
    ties = omoe.near_tie_tokens(f64, shape.top_k, 1e-6 + omoe.ROUTER_LOGIT_ERR,
                                torch.from_numpy(gold["logits"]))
    keep = ~ties
    gi, gs = torch.from_numpy(gold["indices"]), torch.from_numpy(gold["scores"])
    assert torch.equal(idx.long()[keep], gi[keep])
    assert torch.allclose(sc[keep], gs[keep], atol=1e-5, rtol=0)
    f32 = omoe.experts_fp32(x, gi, gs, experts_of(p))
    check_close(out[keep], f32[keep], f"decode mlp {name}")


@pytest.mark.parametrize("T", [1, 2, 8, 33, 64])
@pytest.mark.parametrize("H,I,E,k", [(512, 512, 32, 4), (320, 448, 8, 2)])
def test_decode_random_routing_vs_fp32(T, H, I, E, k):
    """K not a multiple of 256 (320, 448) leaves a partial last K stage and
    H = 320 a half-filled last row tile of the down projection; T=64 with E=8
    gives experts with up to 64 tokens (N = 4 terms x 64 = 256 B rows)."""
    shape = LayerShape(H, I, E, k, 120, 128)
    pe = experts_of(make_layer(shape, 60 + T))
    x = make_tokens(T, H, 60 + T)
    g = torch.Generator().manual_seed(T + H)
    idx = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)])
    w = torch.softmax(torch.randn(T, k, generator=g), -1)
    out, _, _ = forward(x, pe, k, indices=idx, scores=w)
    check_close(out, omoe.experts_fp32(x, idx, w, pe), f"decode T={T} H={H} I={I} E={E}")


def test_decode_one_hot_expert():
    """All 64 tokens on expert 5 (slot 0), the rest spread: N reaches 128."""
    T, E, k = 64, 16, 2
    shape = LayerShape(256, 256, E, k, 124, 130)
    pe = experts_of(make_layer(shape, 91))
    x = make_tokens(T, shape.hidden, 91)
    idx = torch.zeros(T, k, dtype=torch.long)
    idx[:, 0] = 5
    idx[:, 1] = torch.arange(T) % 4 + 8
    w = torch.softmax(torch.randn(T, k, generator=torch.Generator().manual_seed(2)), -1)
    out, _, _ = forward(x, pe, k, indices=idx, scores=w)
    check_close(out, omoe.experts_fp32(x, idx, w, pe), "decode one hot expert")


def test_decode_activation_range():
    """Activations spanning 2^-20..2^20 within a token: per-32 block scales keep them."""
    T, E, k = 4, 8, 2
    shape = LayerShape(256, 256, E, k, 124, 130)
    pe = experts_of(make_layer(shape, 93))
    g = torch.Generator().manual_seed(3)
    mag = torch.pow(2.0, torch.randint(-20, 21, (T, shape.hidden), generator=g).float())
    x = (torch.randn(T, shape.hidden, generator=g) * mag).to(torch.bfloat16)
    idx = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)])
    w = torch.softmax(torch.randn(T, k, generator=g), -1)
    out, _, _ = forward(x, pe, k, indices=idx, scores=w)
    check_close(out, omoe.experts_fp32(x, idx, w, pe), "decode wide-range activations")


def test_decode_matches_across_calls_and_graph():
    """Deterministic: two eager calls and a CUDA-graph replay give identical bits."""
    shape = CASES["gptoss20b"]
    p = make_layer(shape, 5)
    g = {n: t.to(DEV) for n, t in p.items()}
    x = make_tokens(8, shape.hidden, 5).to(DEV)
    args = (x, g["experts.gate_up_proj_blocks"], g["experts.gate_up_proj_scales"],
            g["experts.gate_up_proj_bias"], g["experts.down_proj_blocks"],
            g["experts.down_proj_scales"], g["experts.down_proj_bias"], shape.top_k)
    kw = dict(router_weight=g["router.weight"], router_bias=g["router.bias"], algo=MX)
    a = kernels.moe_forward(*args, **kw)[0].clone()
    b = kernels.moe_forward(*args, **kw)[0].clone()
    assert torch.equal(a, b)
    ws = torch.empty(1 << 24, dtype=torch.uint8, device=DEV)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        kernels.moe_forward(*args, workspace=ws, **kw)   # warm (attribute setup) before capture
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        c = kernels.moe_forward(*args, workspace=ws, **kw)[0]
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(a, c)
    assert kernels.device_status(clear=True) == 0


def test_bs_moe_decode_entry_point_matches_forward():
    """bs_moe_decode (the decode-shape C entry point) gives the same bits as
    bs_moe_forward's AUTO choice (the block-scaled path at T <= 64), and
    rejects more than 64 tokens."""
    import ctypes
    from blockstreamer_b200 import _lib
    shape = LayerShape(512, 512, 32, 4)
    p = make_layer(shape, 12, device=DEV)
    pe = [p[n] for n in ("experts.gate_up_proj_blocks", "experts.gate_up_proj_scales",
                         "experts.gate_up_proj_bias", "experts.down_proj_blocks",
                         "experts.down_proj_scales", "experts.down_proj_bias")]
    vp = lambda t: ctypes.c_void_p(t.data_ptr())
    lib = _lib.load()
    for T in (1, 8, 20):
        x = make_tokens(T, shape.hidden, 12, device=DEV)
        ref, sc_ref, idx_ref = kernels.moe_forward(x, *pe, shape.top_k, router_weight=p["router.weight"],
                                                   router_bias=p["router.bias"], algo=kernels.ALGO_AUTO)
        ws = torch.empty(lib.bs_moe_workspace_bytes(T, shape.hidden, shape.intermediate, shape.experts,
                                                    shape.top_k), dtype=torch.uint8, device=DEV)
        out = torch.empty_like(x)
        sc = torch.empty(T, shape.top_k, dtype=torch.float32, device=DEV)
        idx = torch.empty(T, shape.top_k, dtype=torch.int32, device=DEV)
        _lib.call("bs_moe_decode", vp(x), T, shape.hidden, shape.intermediate, shape.experts, shape.top_k,
                  vp(p["router.weight"]), vp(p["router.bias"]), _lib.BS_F32, vp(sc), vp(idx),
                  *[vp(t) for t in pe], _lib.BS_BF16, 1.702, 7.0, vp(out), vp(ws), ws.numel(),
                  ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        torch.cuda.synchronize()
        assert torch.equal(out, ref) and torch.equal(idx, idx_ref) and torch.equal(sc, sc_ref)
    big = torch.empty(65, shape.hidden, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(ValueError):
        _lib.call("bs_moe_decode", vp(big), 65, shape.hidden, shape.intermediate, shape.experts, shape.top_k,
                  None, None, _lib.BS_F32, vp(sc), vp(idx), *[vp(t) for t in pe], _lib.BS_BF16, 1.702, 7.0,
                  vp(big), vp(ws), ws.numel(), None)
