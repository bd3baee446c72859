"""GPU parity of the whole MoE layer (router, dispatch, expert projections,
combine) against the reference's golden outputs and the fp32 oracle.

Tolerances (from the benchmark specification):
  * routing: indices equal and weights within 1e-5 away from near-ties
    (tokens whose k-th/(k+1)-th exact logits are within 1e-6 are excluded, the
    band widened by the compared implementations' own logit errors on that
    token — the reference's CPU fp32 GEMM is itself ~2.5e-6 from exact);
  * layer output: relative L2 <= 5e-3 against the fp32 evaluation of the
    reference math.  The absolute bound 2e-2 is unattainable for ANY bf16
    output at these magnitudes (outputs reach ~6e4, where one bf16 ulp is 256;
    the reference's own bf16 path misses it by the same margin), so the max
    absolute error is asserted relative to max|y|: <= 2e-2 * max|y|.
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
ALGOS = [kernels.ALGO_GEMV, kernels.ALGO_TCGEN05]
LAYER_CASES = [("tiny", "tiny"), ("gptoss20b_t4", "gptoss20b"), ("gptoss120b_t3", "gptoss120b")]


def experts_of(p):
    return {k.split(".", 1)[1]: v for k, v in p.items() if k.startswith("experts.")}


def run_experts(x, idx, w, pe, algo, k):
    g = {n: t.to(DEV) for n, t in pe.items()}
    out, _, _ = kernels.moe_forward(x.to(DEV), g["gate_up_proj_blocks"], g["gate_up_proj_scales"],
                                    g["gate_up_proj_bias"], g["down_proj_blocks"], g["down_proj_scales"],
                                    g["down_proj_bias"], k, indices=idx.to(DEV), scores=w.to(DEV),
                                    algo=algo)
    return out.cpu()


def check_close(out, ref_f32, label):
    rel = omoe.rel_l2(out.float(), ref_f32)
    mx = (out.float() - ref_f32).abs().max().item()
    scale = ref_f32.abs().max().item()
    print(f"{label}: rel_l2={rel:.3e} max_abs={mx:.3e} max_abs/max|y|={mx / scale:.3e}")
    assert rel <= 5e-3, label
    assert mx <= 2e-2 * scale, label


@pytest.mark.parametrize("algo", ALGOS, ids=["gemv", "tcgen05"])
@pytest.mark.parametrize("name,key", LAYER_CASES)
def test_experts_vs_reference_golden(name, key, algo):
    gold = np.load(os.path.join(GOLDEN, f"layer_{name}.npz"))
    cid, T = int(gold["case"][0]), int(gold["tokens"][0])
    shape = CASES[key]
    pe = experts_of(make_layer(shape, cid))
    x = make_tokens(T, shape.hidden, cid)
    idx = torch.from_numpy(gold["indices"])
    w = torch.from_numpy(gold["scores"])
    out = run_experts(x, idx, w, pe, algo, shape.top_k)
    f32 = omoe.experts_fp32(x, idx, w, pe)
    check_close(out, f32, f"{name} algo={algo} vs fp32")
    ref = torch.from_numpy(gold["out_bits"].astype(np.int16)).view(torch.bfloat16).float()
    # the reference's own bf16 error is the calibration line; ours must not be worse than 2x it
    assert omoe.rel_l2(out.float(), f32) <= max(2 * omoe.rel_l2(ref, f32), 1e-3)


@pytest.mark.parametrize("algo", ALGOS, ids=["gemv", "tcgen05"])
@pytest.mark.parametrize("T,E,k", [(1, 32, 4), (19, 8, 2), (130, 16, 4), (600, 8, 4)])
def test_experts_random_routing_vs_fp32(T, E, k, algo):
    shape = LayerShape(512, 512, E, k, 120, 128)
    pe = experts_of(make_layer(shape, 40 + T))
    x = make_tokens(T, shape.hidden, 40 + T)
    g = torch.Generator().manual_seed(T)
    idx = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)])
    w = torch.softmax(torch.randn(T, k, generator=g), -1)
    out = run_experts(x, idx, w, pe, algo, k)
    check_close(out, omoe.experts_fp32(x, idx, w, pe), f"T={T} E={E} algo={algo}")


@pytest.mark.parametrize("algo", ALGOS, ids=["gemv", "tcgen05"])
def test_experts_skewed_routing(algo):
    """One expert takes most tokens (the Zipf case's hot expert) and several take none."""
    T, E, k = 700, 16, 2
    shape = LayerShape(256, 256, E, k, 124, 130)
    pe = experts_of(make_layer(shape, 77))
    x = make_tokens(T, shape.hidden, 77)
    idx = torch.zeros(T, k, dtype=torch.long)
    idx[:, 0] = 3
    idx[:, 1] = torch.arange(T) % 3 + 4   # experts 4..6; the rest get nothing
    w = torch.softmax(torch.randn(T, k, generator=torch.Generator().manual_seed(1)), -1)
    out = run_experts(x, idx, w, pe, algo, k)
    check_close(out, omoe.experts_fp32(x, idx, w, pe), f"skewed algo={algo}")


@pytest.mark.parametrize("algo", ALGOS, ids=["gemv", "tcgen05"])
@pytest.mark.parametrize("name,key", LAYER_CASES)
def test_full_mlp_vs_oracle(name, key, algo):
    gold = np.load(os.path.join(GOLDEN, f"layer_{name}.npz"))
    cid, T = int(gold["case"][0]), int(gold["tokens"][0])
    shape = CASES[key]
    p = make_layer(shape, cid)
    x = make_tokens(T, shape.hidden, cid)
    g = {n: t.to(DEV) for n, t in p.items()}
    out, sc, idx = kernels.moe_forward(
        x.to(DEV), g["experts.gate_up_proj_blocks"], g["experts.gate_up_proj_scales"],
        g["experts.gate_up_proj_bias"], g["experts.down_proj_blocks"], g["experts.down_proj_scales"],
        g["experts.down_proj_bias"], shape.top_k, router_weight=g["router.weight"],
        router_bias=g["router.bias"], algo=algo)
    f64 = omoe.router_logits_f64(x, p["router.weight"], p["router.bias"])
    ties = omoe.near_tie_tokens(f64, shape.top_k, 1e-6 + omoe.ROUTER_LOGIT_ERR,
                                torch.from_numpy(gold["logits"]))
    keep = ~ties
    assert torch.equal(idx.cpu().long()[keep], torch.from_numpy(gold["indices"])[keep])
    pe = experts_of(p)
    f32 = omoe.experts_fp32(x, torch.from_numpy(gold["indices"]), torch.from_numpy(gold["scores"]), pe)
    check_close(out.cpu()[keep], f32[keep], f"mlp {name} algo={algo}")


@pytest.mark.parametrize("algo", ALGOS, ids=["gemv", "tcgen05"])
@pytest.mark.parametrize("m,K,N", [(8, 128, 64), (3, 2880, 5760), (300, 512, 256)])
def test_mxfp4_matmul_matches_dense(m, K, N, algo):
    """Mirrors tests/test_offload.py:369-388: x @ dequantize_expert(...)."""
    from blockstreamer_b200 import dequantize_expert
    g = torch.Generator().manual_seed(m * K)
    blocks = torch.randint(0, 255, (1, N, K // 32, 16), dtype=torch.uint8, generator=g).to(DEV)
    scales = torch.randint(120, 134, (1, N, K // 32), dtype=torch.uint8, generator=g).to(DEV)
    x = torch.randn(m, K, generator=g).to(torch.bfloat16).to(DEV)
    w = dequantize_expert(blocks, scales, torch.float32)
    ref = x.float() @ w
    out = kernels.mxfp4_matmul(x, blocks[0], scales[0], algo=algo).float()
    rel = omoe.rel_l2(out.cpu(), ref.cpu())
    assert rel < 4e-3, rel


def test_mxfp4_matmul_autograd_and_memory():
    """Gradient equals grad @ W^T (here to bf16 rounding: the transposed GEMM
    accumulates in fp32 from the packed codes) and no dense weight survives
    into backward (tests/test_offload.py:390-402)."""
    from blockstreamer_b200 import dequantize_expert, mxfp4_matmul
    torch.manual_seed(0)
    blocks = torch.randint(0, 255, (1, 64, 4, 16), dtype=torch.uint8, device=DEV)
    scales = torch.randint(120, 134, (1, 64, 4), dtype=torch.uint8, device=DEV)
    weight = dequantize_expert(blocks, scales, torch.bfloat16)
    x = torch.randn(8, 128, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    out = mxfp4_matmul(x, blocks, scales)
    grad = torch.randn_like(out)
    out.backward(grad)
    ref = grad.float() @ weight.float().t()
    assert omoe.rel_l2(x.grad.float().cpu(), ref.cpu()) <= 4e-3
    torch.cuda.reset_peak_memory_stats()
    base = torch.cuda.memory_allocated()
    chained = [mxfp4_matmul(x, blocks, scales) for _ in range(64)]
    peak = torch.cuda.max_memory_allocated() - base
    sum(y.float().sum() for y in chained).backward()
    assert peak < weight.numel() * weight.element_size() * 16


def test_drop_in_modules_bind_state_like_functional_call():
    """B200GptOssMLP / B200MXFP4Experts driven through torch.func.functional_call
    with a state dict keyed by the checkpoint names (what StreamedModel does)."""
    from torch.func import functional_call
    import types
    from blockstreamer_b200 import B200GptOssMLP
    shape = CASES["tiny"]
    cfg = types.SimpleNamespace(hidden_size=shape.hidden, intermediate_size=shape.intermediate,
                                num_local_experts=shape.experts, num_experts_per_tok=shape.top_k,
                                swiglu_limit=7.0)
    mlp = B200GptOssMLP(cfg)
    p = make_layer(shape, 1)
    state = {n: t.to(DEV) for n, t in p.items()}
    x = make_tokens(64, shape.hidden, 1).to(DEV).reshape(2, 32, shape.hidden)
    versions = {n: t._version for n, t in state.items()}
    out, scores = functional_call(mlp, state, (x,), strict=True)
    assert out.shape == x.shape and scores.shape == (64, shape.top_k)
    assert all(state[n]._version == v for n, v in versions.items())   # no mutation
    gold = np.load(os.path.join(GOLDEN, "layer_tiny.npz"))
    f32 = omoe.experts_fp32(x.reshape(64, -1).cpu(), torch.from_numpy(gold["indices"]),
                            torch.from_numpy(gold["scores"]), experts_of(p))
    check_close(out.reshape(64, -1).cpu(), f32, "functional_call mlp")


def test_no_device_errors_recorded():
    assert kernels.device_status(clear=True) == 0


def test_reference_streamed_model_streams_the_b200_mlp():
    """The reference's own StreamedModel (installed under baseline/_ref)
    streams B200GptOssMLP blocks from pinned host memory through its prefetch
    ring (prefetch_ahead=1) and binds their state with functional_call: the
    output equals running the same blocks resident on the GPU."""
    import copy
    import sys
    import types

    ref_dir = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")
    if not os.path.exists(os.path.join(ref_dir, "streamer.py")):
        pytest.skip("reference package not installed under baseline/_ref")
    if ref_dir not in sys.path:
        sys.path.insert(0, ref_dir)
    from streamer import StreamedModel
    from blockstreamer_b200 import B200GptOssMLP

    shape = LayerShape(512, 512, 16, 4)
    cfg = types.SimpleNamespace(hidden_size=shape.hidden, intermediate_size=shape.intermediate,
                                num_local_experts=shape.experts, num_experts_per_tok=shape.top_k,
                                swiglu_limit=7.0)
    blocks = []
    for layer in range(3):
        mlp = B200GptOssMLP(cfg)
        mlp.load_state_dict(make_layer(shape, 20 + layer), strict=True, assign=True)
        blocks.append(mlp)
    resident = [copy.deepcopy(b).to(DEV) for b in blocks]
    x = make_tokens(96, shape.hidden, 20).to(DEV).reshape(3, 32, shape.hidden)
    h = x
    for b in resident:
        h, scores_direct = b(h)
    model = StreamedModel(blocks, device=DEV, prefetch_ahead=1, dtype=None)
    out, scores = model(x)
    torch.cuda.synchronize()
    assert torch.equal(out, h)
    assert torch.equal(scores, scores_direct)
    assert model.stats()["transfer_bytes"] > 0


def test_experts_and_mlp_backward_match_fp32_autograd():
    """Gradients through the drop-in modules (the reference trains through the
    experts: gptoss.py:45-75, 137-177): dL/dx and dL/d routing weights of
    B200MXFP4Experts, and dL/dx of B200GptOssMLP (router included), against
    autograd through the fp32 restatement of the reference math."""
    import types
    from blockstreamer_b200 import B200GptOssMLP, B200MXFP4Experts

    shape = CASES["tiny"]
    cfg = types.SimpleNamespace(hidden_size=shape.hidden, intermediate_size=shape.intermediate,
                                num_local_experts=shape.experts, num_experts_per_tok=shape.top_k,
                                swiglu_limit=7.0)
    p = make_layer(shape, 3)
    x = make_tokens(64, shape.hidden, 3)
    pe = experts_of(p)
    _, s_ref, i_ref = omoe.router(x.float(), p["router.weight"], p["router.bias"], shape.top_k)
    g = torch.randn(64, shape.hidden, generator=torch.Generator().manual_seed(5))

    ex = B200MXFP4Experts(cfg)
    ex.load_state_dict({n: t.to(DEV) for n, t in pe.items()}, strict=True, assign=True)
    xg = x.to(DEV).float().requires_grad_()
    wg = s_ref.to(DEV).requires_grad_()
    out = ex(xg, i_ref.to(DEV), wg)
    out.backward(g.to(DEV))
    xc = x.float().requires_grad_()
    wc = s_ref.clone().requires_grad_()
    ref = omoe.experts_fp32(xc, i_ref, wc, pe)
    ref.backward(g)
    r_out, r_dx, r_dw = (omoe.rel_l2(out.detach().cpu(), ref.detach()), omoe.rel_l2(xg.grad.cpu(), xc.grad),
                         omoe.rel_l2(wg.grad.cpu(), wc.grad))
    print(f"experts: out {r_out:.2e} dx {r_dx:.2e} dw {r_dw:.2e}")
    assert r_out <= 5e-3 and r_dx <= 1e-2 and r_dw <= 1e-2

    mlp = B200GptOssMLP(cfg)
    mlp.load_state_dict({n: t.to(DEV) for n, t in p.items()}, strict=True, assign=True)
    xm = x.to(DEV).float().reshape(2, 32, shape.hidden).requires_grad_()
    om, _ = mlp(xm)
    om.reshape(64, -1).backward(g.to(DEV))
    xr = x.float().requires_grad_()
    logits = torch.nn.functional.linear(xr, p["router.weight"], p["router.bias"])
    top_v, top_i = torch.topk(logits, shape.top_k, dim=-1)
    ref_m = omoe.experts_fp32(xr, top_i, torch.softmax(top_v, dim=1), pe)
    ref_m.backward(g)
    keep = ~omoe.near_tie_tokens(omoe.router_logits_f64(x, p["router.weight"], p["router.bias"]),
                                 shape.top_k, 1e-6 + omoe.ROUTER_LOGIT_ERR, logits.detach())
    r_mo = omoe.rel_l2(om.detach().reshape(64, -1).cpu()[keep], ref_m.detach()[keep])
    r_mdx = omoe.rel_l2(xm.grad.reshape(64, -1).cpu()[keep], xr.grad[keep])
    print(f"mlp: out {r_mo:.2e} dx {r_mdx:.2e}")
    assert r_mo <= 5e-3 and r_mdx <= 1e-2


def test_reference_disk_shards_stream_the_b200_mlp(tmp_path):
    """The reference's on-disk shard format (block_streamer/shards.py:
    convert_modules writes one flat file per block plus manifest.json) and its
    DiskBufferPool (StreamedModel(manifest=...)) feed B200GptOssMLP blocks
    built on ``meta``: the output equals the same blocks resident on the GPU."""
    import sys
    import types

    ref_dir = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")
    if not os.path.exists(os.path.join(ref_dir, "streamer.py")):
        pytest.skip("reference package not installed under baseline/_ref")
    if ref_dir not in sys.path:
        sys.path.insert(0, ref_dir)
    from streamer import StreamedModel
    from block_streamer.shards import convert_modules
    from blockstreamer_b200 import B200GptOssMLP

    shape = LayerShape(512, 512, 16, 4)
    cfg = types.SimpleNamespace(hidden_size=shape.hidden, intermediate_size=shape.intermediate,
                                num_local_experts=shape.experts, num_experts_per_tok=shape.top_k,
                                swiglu_limit=7.0)
    states = [make_layer(shape, 30 + layer) for layer in range(3)]
    manifest = convert_modules(((i, st) for i, st in enumerate(states)), tmp_path)
    h = make_tokens(96, shape.hidden, 30).to(DEV).reshape(3, 32, shape.hidden)
    x = h.clone()
    for st in states:
        b = B200GptOssMLP(cfg)
        b.load_state_dict({n: t.to(DEV) for n, t in st.items()}, strict=True, assign=True)
        h, scores_direct = b(h)
    model = StreamedModel([B200GptOssMLP(cfg) for _ in states], device=DEV, prefetch_ahead=1, dtype=None,
                          manifest=manifest)
    out, scores = model(x)
    torch.cuda.synchronize()
    assert torch.equal(out, h)
    assert torch.equal(scores, scores_direct)
    model.close()


@pytest.mark.parametrize("algo", [kernels.ALGO_AUTO, kernels.ALGO_TCGEN05, kernels.ALGO_GEMV])
def test_moe_block_norm_and_residual_vs_reference_math(algo):
    """B200GptOssMoEBlock = x + mlp(post_attention_layernorm(x)) (the MoE half of
    GptOssDecoderLayer.forward): RMSNorm kernel against GptOssRMSNorm's torch
    math (within one bf16 ulp), and the block against the fp32 reference math
    on the normalized rows plus the residual (rel-L2 <= 5e-3, routing exact
    away from near-ties)."""
    import types
    from blockstreamer_b200 import B200GptOssMoEBlock

    shape = CASES["tiny"]
    T = 64
    cfg = types.SimpleNamespace(hidden_size=shape.hidden, intermediate_size=shape.intermediate,
                                num_local_experts=shape.experts, num_experts_per_tok=shape.top_k,
                                swiglu_limit=7.0, rms_norm_eps=1e-5)
    p = make_layer(shape, 6)
    g = torch.Generator().manual_seed(6)
    nw = (1.0 + 0.1 * torch.randn(shape.hidden, generator=g)).float()
    x = make_tokens(T, shape.hidden, 6)
    # GptOssRMSNorm.forward's math
    v = x.float()
    xn = (nw * (v * torch.rsqrt(v.pow(2).mean(-1, keepdim=True) + 1e-5))).to(torch.bfloat16)
    got_n = kernels.rmsnorm(x.to(DEV), nw.to(DEV), 1e-5).cpu()
    ulp = (xn.float().abs() * 2.0 ** -7).clamp_min(1e-30)
    assert bool(((got_n.float() - xn.float()).abs() <= ulp).all())

    blk = B200GptOssMoEBlock(cfg, algo=algo)
    state = {"post_attention_layernorm.weight": nw}
    state.update({"mlp." + n: t for n, t in p.items()})
    blk.load_state_dict({n: t.to(DEV) for n, t in state.items()}, strict=True, assign=True)
    out = blk(x.to(DEV).reshape(1, T, -1)).reshape(T, -1).cpu()
    lg, s_ref, i_ref = omoe.router(xn.float(), p["router.weight"], p["router.bias"], shape.top_k)
    ref = x.float() + omoe.experts_fp32(xn, i_ref, s_ref, experts_of(p))
    keep = ~omoe.near_tie_tokens(omoe.router_logits_f64(xn, p["router.weight"], p["router.bias"]),
                                 shape.top_k, 1e-6 + omoe.ROUTER_LOGIT_ERR, lg)
    rel = omoe.rel_l2(out.float()[keep], ref[keep])
    print(f"algo {algo}: block rel_l2 {rel:.2e} ({int(keep.sum())} of {T} tokens)")
    assert rel <= 5e-3
