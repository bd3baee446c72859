"""Bit-exact MXFP4 dequantization on the CPU (numpy) — test infrastructure.

Restates the algorithm of ``transformers.integrations.mxfp4._convert_moe_packed_tensors``
(transformers 5.5.0, integrations/mxfp4.py:279-330), which the reference reaches
through ``block_streamer/gptoss.py:24-42`` (``dequantize_expert``):

* each packed byte holds two e2m1 codes: the LOW nibble is the even element,
  the HIGH nibble the odd one (mxfp4.py:311-319);
* a code indexes the 16-entry table ``FP4_VALUES`` (mxfp4.py:29-46):
  +-{0, 0.5, 1, 1.5, 2, 3, 4, 6}, codes 8..15 negative (8 is -0.0);
* the e8m0 scale byte ``s`` multiplies the 32 elements of its block by
  ``2**(s - 127)`` via ``torch.ldexp`` (mxfp4.py:295, 322);
* the result [.., rows, G*32] is transposed to [.., G*32, rows] (mxfp4.py:328-330).

Measured against the reference over all 256 bytes x 256 scales: the value is
the exact product rounded once to the output dtype, products >= 2**128 become
+-inf, subnormal products survive, and no NaN is ever produced.
"""

from __future__ import annotations

import numpy as np

FP4_VALUES = np.array(
    [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
     -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0],
    dtype=np.float64,
)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round float32 values to bf16 (round-to-nearest-even); returns uint16 bits."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    lsb = (u >> 16) & 1
    out = ((u + 0x7FFF + lsb) >> 16).astype(np.uint16)
    out[nan] = 0x7FC0
    return out


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def _values_f64(blocks: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """Exact dequantized values in float64, natural orientation [..., G*32]."""
    blocks = np.asarray(blocks, dtype=np.uint8)
    scales = np.asarray(scales, dtype=np.uint8)
    if blocks.shape[:-1] != scales.shape or blocks.shape[-1] != 16:
        raise ValueError(
            f"blocks {blocks.shape} must be scales {scales.shape} + (16,)")
    lo = FP4_VALUES[blocks & 0x0F]
    hi = FP4_VALUES[blocks >> 4]
    vals = np.empty(blocks.shape[:-1] + (32,), dtype=np.float64)
    vals[..., 0::2] = lo
    vals[..., 1::2] = hi
    exp = scales.astype(np.int64) - 127
    with np.errstate(over="ignore"):
        vals = np.ldexp(vals, exp[..., None])
    return vals.reshape(blocks.shape[:-2] + (blocks.shape[-2] * 32,))


def dequant_f32(blocks: np.ndarray, scales: np.ndarray, transpose: bool = True) -> np.ndarray:
    """Dequantize [E, rows, G, 16] blocks + [E, rows, G] scales to float32.

    With ``transpose`` (the reference's orientation) the result is
    [E, G*32, rows]; otherwise [E, rows, G*32].
    """
    with np.errstate(over="ignore"):
        vals = _values_f64(blocks, scales).astype(np.float32)
    if transpose:
        vals = np.ascontiguousarray(np.swapaxes(vals, -1, -2))
    return vals


def dequant_bf16_bits(blocks: np.ndarray, scales: np.ndarray, transpose: bool = True) -> np.ndarray:
    """Dequantize to bf16 and return the uint16 bit patterns (see ``dequant_f32``)."""
    return f32_to_bf16_bits(dequant_f32(blocks, scales, transpose))


def e2m1_bf16_bits(code: int, scale: int) -> int:
    """Scalar form, for spot checks: bf16 bits of FP4_VALUES[code] * 2**(scale-127)."""
    v = np.float32(np.ldexp(FP4_VALUES[code], scale - 127)) if abs(
        np.ldexp(FP4_VALUES[code], scale - 127)) < 2.0 ** 128 else np.float32(
        np.copysign(np.inf, FP4_VALUES[code]))
    return int(f32_to_bf16_bits(np.array([v], dtype=np.float32))[0])
