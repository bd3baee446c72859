"""Parity at the benchmarked configurations, on the exact inputs bench.py times.

* gpt-oss-120b prefill, 8192 tokens, 128 experts (the default bench workload,
  BASELINE config 4 at one GPU: 203-305 rows per expert, so every expert runs
  the 320-row tile with its second 128 x 64 MMA or a two-chunk split);
* gpt-oss-20b prefill, 4096 tokens, 32 experts (config 2: ~512 rows per
  expert, several token chunks per expert);
* gpt-oss-120b decode, 1 / 8 / 64 tokens (config 3: the block-scaled decode
  path at all three, with gathered activation rows above 16 tokens, and the
  single-launch kernel at 1 and 8 tokens).

Each test runs the layer through the C ABI (``bs_moe_forward``, router
included) and checks, following block_streamer/gptoss.py:137-177 and
transformers modeling_gpt_oss.py:126-130:
  * routing: indices equal and weights within 1e-5 on every token away from
    near-ties (k-th/(k+1)-th exact logits within 1e-6, widened by the logit
    error of the compared implementations), against the CPU oracle router;
  * layer output: relative L2 <= 5e-3 and max-abs <= 2e-2 * max|y| against
    the fp32 oracle (evaluated on the GPU's copy of the inputs so that all
    experts fit in the test's time; matmuls in true fp32, TF32 off);
  * prefill, in addition: gate_up (h) and down (y) rows of six experts,
    including the one with the fewest and the one with the most rows, against
    the fp32 oracle on the CPU; the combine against an exact (fp64)
    recombination of the kernel's own y rows, within the fp32-sum and one-bf16-
    rounding error bound; and bs_moe_forward equal, bit for bit, to the same
    kernels called stage by stage.
"""

import pytest
import torch

from blockstreamer_b200 import kernels
from blockstreamer_b200.synthetic import CASES, make_layer, make_tokens
from oracle import moe as omoe

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
EXPERT_KEYS = ("gate_up_proj_blocks", "gate_up_proj_scales", "gate_up_proj_bias",
               "down_proj_blocks", "down_proj_scales", "down_proj_bias")


@pytest.fixture(autouse=True)
def _true_fp32():
    prev = (torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = prev


def experts_of(p):
    return {k.split(".", 1)[1]: v for k, v in p.items() if k.startswith("experts.")}


def check_routing(x, p, k, sc, idx):
    """Indices exact and weights within 1e-5 away from near-ties (CPU oracle router)."""
    xc, W, b = x.cpu(), p["router.weight"].cpu(), p["router.bias"].cpu()
    lg_ref, s_ref, i_ref = omoe.router(xc.float(), W, b, k)
    f64 = omoe.router_logits_f64(xc, W, b)
    ties = omoe.near_tie_tokens(f64, k, 1e-6 + omoe.ROUTER_LOGIT_ERR, lg_ref)
    keep = ~ties
    T = xc.shape[0]
    print(f"routing: {int(ties.sum())} of {T} tokens excluded as near-ties")
    assert int(keep.sum()) >= 0.99 * T
    assert torch.equal(idx.cpu().long()[keep], i_ref[keep])
    assert float((sc.cpu()[keep] - s_ref[keep]).abs().max()) <= 1e-5


def check_close(out, ref, label):
    rel = omoe.rel_l2(out.float(), ref.float())
    mx = float((out.float() - ref.float()).abs().max())
    scale = float(ref.float().abs().max())
    print(f"{label}: rel_l2={rel:.3e} max_abs={mx:.3e} max_abs/max|y|={mx / scale:.3e}")
    assert rel <= 5e-3, label
    assert mx <= 2e-2 * scale, label


def layer_args(p):
    return [p["experts." + n] for n in EXPERT_KEYS]


@pytest.mark.parametrize("key,case_id,T", [("gptoss120b", 4, 8192), ("gptoss20b", 2, 4096)],
                         ids=["120b-prefill-8192", "20b-prefill-4096"])
def test_prefill_parity_at_bench_config(key, case_id, T):
    shape = CASES[key]
    k, E = shape.top_k, shape.experts
    p = make_layer(shape, case_id, device=DEV)        # bench.py's inputs
    x = make_tokens(T, shape.hidden, case_id, device=DEV)
    args = layer_args(p)
    out, sc, idx = kernels.moe_forward(x, *args, k, router_weight=p["router.weight"],
                                       router_bias=p["router.bias"], algo=kernels.ALGO_AUTO)
    out_tc, _, _ = kernels.moe_forward(x, *args, k, router_weight=p["router.weight"],
                                       router_bias=p["router.bias"], algo=kernels.ALGO_TCGEN05)
    torch.cuda.synchronize()
    assert torch.equal(out, out_tc)                    # AUTO takes the tcgen05 path here
    check_routing(x, p, k, sc, idx)

    # the same kernels stage by stage through the C ABI: identical bits
    d = kernels.dispatch(idx, E, x)
    h = kernels.moe_gate_up(d.x_perm, d.expert_offsets, *args[:3])
    y = kernels.moe_down(h, d.expert_offsets, *args[3:])
    out_st = kernels.combine(y, d.row_of_slot, sc, T)
    torch.cuda.synchronize()
    assert torch.equal(out_st, out)
    counts = (d.expert_offsets[1:] - d.expert_offsets[:-1]).cpu()
    print(f"rows per expert: min {int(counts.min())} max {int(counts.max())}")

    # six experts' h and y rows against the CPU fp32 oracle
    g = torch.Generator().manual_seed(T)
    lo, hi = int(counts.argmin()), int(counts.argmax())
    others = [int(e) for e in torch.randperm(E, generator=g) if int(e) not in (lo, hi)][:4]
    chosen = [lo, hi] + others
    pe_cpu = {n: t.cpu() for n, t in experts_of(p).items()}
    idx_c, sc_c = idx.cpu().long(), sc.cpu()
    _, inter = omoe.experts_fp32(x.cpu(), idx_c, sc_c, pe_cpu, return_intermediates=True,
                                 experts_subset=chosen)
    ros = d.row_of_slot.cpu().long()
    h_c, y_c = h.cpu(), y.cpu()
    for e in chosen:
        tok, slot, h_ref, y_ref = inter[e]
        rows = ros[tok * k + slot]                      # the oracle's row order -> ours
        check_close(h_c[rows], h_ref, f"{key} expert {e} ({len(rows)} rows) h")
        check_close(y_c[rows], y_ref, f"{key} expert {e} ({len(rows)} rows) y")

    # combine: the kernel's own y rows summed exactly (fp64); the kernel's fp32
    # sum of k terms is within k * 2^-24 * sum|w y| of it, and its one bf16
    # rounding within 2^-8 of the value
    yk = y.double()[d.row_of_slot.long()].view(T, k, -1) * sc.double().unsqueeze(-1)
    ref_c = yk.sum(1)
    tol = ref_c.abs() * 2.0 ** -8 + k * 2.0 ** -23 * yk.abs().sum(1) + 1e-30
    assert bool(((out.double() - ref_c).abs() <= tol).all())

    # the whole layer against the fp32 oracle on the GPU's copy of the inputs
    ref = omoe.experts_fp32(x, idx.long(), sc, experts_of(p))
    check_close(out, ref, f"{key} T={T} layer")
    assert kernels.device_status(clear=True) == 0


@pytest.mark.parametrize("T", [1, 8, 64])
def test_decode_parity_at_bench_config(T):
    shape = CASES["gptoss120b"]
    k = shape.top_k
    p = make_layer(shape, 3, device=DEV)                # bench.py's decode inputs
    x = make_tokens(T, shape.hidden, 3, device=DEV)
    args = layer_args(p)
    out, sc, idx = kernels.moe_forward(x, *args, k, router_weight=p["router.weight"],
                                       router_bias=p["router.bias"], algo=kernels.ALGO_AUTO)
    # AUTO takes the block-scaled decode path at T <= 64
    out_a, sc_a, idx_a = kernels.moe_forward(x, *args, k, router_weight=p["router.weight"],
                                             router_bias=p["router.bias"], algo=kernels.ALGO_MX)
    torch.cuda.synchronize()
    assert torch.equal(out, out_a) and torch.equal(idx, idx_a)
    check_routing(x, p, k, sc, idx)
    print(f"T={T}: {int(torch.unique(idx).numel())} distinct experts")
    ref = omoe.experts_fp32(x, idx.long(), sc, experts_of(p))
    check_close(out, ref, f"120b decode T={T} layer")
    if T <= 8:   # the single-launch kernel (on request) on the same inputs
        out_f, _, idx_f = kernels.moe_forward(x, *args, k, router_weight=p["router.weight"],
                                              router_bias=p["router.bias"], algo=kernels.ALGO_FUSED)
        assert torch.equal(idx_f, idx)
        check_close(out_f, ref, f"120b decode T={T} single-launch kernel")
    # against the prefill kernels (tcgen05 grouped GEMM) on the same routing
    out_tc, _, _ = kernels.moe_forward(x, *args, k, indices=idx, scores=sc, algo=kernels.ALGO_TCGEN05)
    check_close(out_tc, ref, f"120b T={T} tcgen05 path")
    assert kernels.device_status(clear=True) == 0
