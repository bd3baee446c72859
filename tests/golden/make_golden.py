"""Generate the golden fixtures in this directory by running the REFERENCE itself.

Run in a container where the reference is importable (it is not shipped here):

    python tests/golden/make_golden.py /path/to/BlockStreamer

The reference path is ``block_streamer.gptoss`` (``dequantize_expert``,
``MXFP4Experts``) plus transformers' ``GptOssTopKRouter`` — the same objects
``GptOssMLP.forward`` calls (transformers models/gpt_oss/modeling_gpt_oss.py:140-146).
The router is fed ``x.float()`` because the benchmark's router weights are fp32.

Fixtures written (small; inputs are regenerated from their seeds with
``blockstreamer_b200.synthetic`` and checked against the stored SHA-256):

* ``dequant_sweep.npz``  bf16 bits of every byte value (both nibbles) under
  every e8m0 scale 0..255, through ``dequantize_expert`` -> [512, 256].
* ``layer_<case>.npz``   router logits/scores/indices and the experts output of
  the reference for one seeded case, plus input checksums.
"""

from __future__ import annotations

import hashlib
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from blockstreamer_b200.synthetic import CASES, make_layer, make_tokens  # noqa: E402

# (name, case shape key, case id, tokens)
LAYER_CASES = [
    ("tiny", "tiny", 1, 64),
    ("gptoss20b_t4", "gptoss20b", 2, 4),
    ("gptoss120b_t3", "gptoss120b", 3, 3),
]


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def bits16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().astype(np.uint16)


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    from block_streamer.gptoss import MXFP4Experts, dequantize_expert
    from transformers.models.gpt_oss.configuration_gpt_oss import GptOssConfig
    from transformers.models.gpt_oss.modeling_gpt_oss import GptOssTopKRouter

    # 1. dequant sweep: row r uses scale r; its 16 groups hold bytes 0..255.
    rows, groups = 256, 16
    b = np.arange(256, dtype=np.uint8).reshape(groups, 16)
    blocks = torch.from_numpy(np.broadcast_to(b, (1, rows, groups, 16)).copy())
    scales = torch.from_numpy(np.broadcast_to(np.arange(256, dtype=np.uint8)[:, None], (1, rows, groups)).copy())
    dense = dequantize_expert(blocks, scales, torch.bfloat16)
    assert dense.shape == (groups * 32, rows)
    np.savez_compressed(os.path.join(HERE, "dequant_sweep.npz"), bits=bits16(dense))

    # 2. layer cases
    for name, key, cid, T in LAYER_CASES:
        shape = CASES[key]
        p = make_layer(shape, cid)
        x = make_tokens(T, shape.hidden, cid)
        cfg = GptOssConfig(hidden_size=shape.hidden, intermediate_size=shape.intermediate,
                           num_local_experts=shape.experts, num_experts_per_tok=shape.top_k,
                           swiglu_limit=shape.swiglu_limit)
        router = GptOssTopKRouter(cfg)
        router.weight.data = p["router.weight"].clone()
        router.bias.data = p["router.bias"].clone()
        experts = MXFP4Experts(cfg, torch.bfloat16)
        for n in ("gate_up_proj_blocks", "gate_up_proj_scales", "gate_up_proj_bias",
                  "down_proj_blocks", "down_proj_scales", "down_proj_bias"):
            setattr(experts, n, torch.nn.Parameter(p["experts." + n].clone(), requires_grad=False))
        with torch.no_grad():
            logits, scores, idx = router(x.float())
            out = experts(x, idx, scores)
        np.savez_compressed(
            os.path.join(HERE, f"layer_{name}.npz"),
            case=np.array([cid]), tokens=np.array([T]),
            logits=logits.numpy(), scores=scores.numpy(), indices=idx.numpy(),
            out_bits=bits16(out),
            sha_x=np.array([sha(x)]),
            **{"sha_" + k.replace(".", "_"): np.array([sha(v)]) for k, v in p.items()},
        )
        print(name, "T", T, "hit experts", len(set(idx.reshape(-1).tolist())))


if __name__ == "__main__":
    # the reference checkout (or its installed copy, baseline/_ref) as the argument
    main(sys.argv[1] if len(sys.argv) > 1 else os.path.join(os.path.dirname(os.path.dirname(HERE)),
                                                           "baseline", "_ref"))
