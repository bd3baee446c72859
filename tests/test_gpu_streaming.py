"""The expert-granular streamer (blockstreamer_b200.streaming) against the
same layers with every weight resident.

Its GEMMs run per staged id range instead of once over all experts, but every
expert's rows go through the same tiles either way, so the stack's output must
equal, bit for bit, the resident layers chained through ``bs_moe_forward``.
Checked with Zipf routing (some experts unused: their slots keep the previous
layer's weights and must never be read), all-expert staging, one and several
ranges, and that exactly the hit experts' bytes were staged."""

import pytest
import torch

from blockstreamer_b200 import kernels
from blockstreamer_b200.streaming import EXPERT_TENSORS, StreamedMoEStack
from blockstreamer_b200.synthetic import LayerShape, make_layer, make_tokens, zipf_router_bias

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def resident_stack(states, x, k):
    for s in states:
        p = {n: t.to(DEV) for n, t in s.items()}
        x, _, _ = kernels.moe_forward(x, *[p["experts." + n] for n in EXPERT_TENSORS], k,
                                      router_weight=p["router.weight"], router_bias=p["router.bias"])
    return x


@pytest.mark.parametrize("hit_only,groups", [(True, 3), (True, 1), (False, 4)])
def test_streamed_stack_equals_resident_layers(hit_only, groups):
    shape = LayerShape(512, 512, 32, 4)
    T, layers = 300, 3
    states = []
    for li in range(layers):
        p = make_layer(shape, 60 + li)
        p["router.bias"] = zipf_router_bias(shape, 1.6, 60 + li) * 4.0   # leaves experts unused
        states.append(p)
    x = make_tokens(T, shape.hidden, 61, device=DEV)
    stack = StreamedMoEStack(states, shape.top_k, DEV, groups=groups, hit_only=hit_only)
    for _ in range(2):          # a second pass reuses both slots with stale weights in them
        out = stack(x)
    torch.cuda.synchronize()
    ref = resident_stack(states, x, shape.top_k)
    assert torch.equal(out, ref)
    per_expert = stack.layers[0].bytes_per_expert
    staged = stack.stats.experts_staged[-layers:]
    assert stack.stats.bytes_staged[-layers:] == [n * per_expert for n in staged]
    if hit_only:
        assert min(staged) < shape.experts          # the Zipf bias left experts unused
    else:
        assert staged == [shape.experts] * layers
    assert kernels.device_status(clear=True) == 0
