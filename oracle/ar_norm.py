"""The layer-input step after the TP all-reduce: sum of the ranks' partial
hidden states + residual, RMSNorm, MXFP4 quantisation.

TEST INFRASTRUCTURE ONLY (the oracle): imported by tests, never by the
product package.

Restates the fused one-shot all-reduce + residual + RMSNorm of
patches/aiter-1stage-nloop-ar-rmsnorm.patch:12-253 (``allreduce_fusion_
kernel_1stage_nloop``: the ranks' rows summed in float32, the residual added,
the new residual written, the sum of squares reduced for the norm) followed by
the quant-only step the reference checks it against
(tests/test_ar_fusion_correctness.py:115-151):

    combined = bf16(sum_r x_r + residual)          (the new residual)
    normed   = bf16(combined * rsqrt(mean(combined^2) + eps))
    out      = bf16(normed * weight)
    nibbles, scales = MXFP4(out)                   (e2m1 + e8m0 per 32)

The MXFP4 scales are emitted unshuffled ([rows, hidden / 32]); aiter's CK
scale-shuffle layout is not restated.

Every float32 operation is done in the order the CUDA kernel does it, so the
results are bit-exact: per row, thread g (0 .. hidden/32 - 1) owns elements
32 g .. 32 g + 31; it sums its 32 squares in element order; a warp of 32
threads combines them with a butterfly (lane l adds lane l ^ 16, then ^ 8,
^ 4, ^ 2, ^ 1; lane 0's value is kept); the warps' values are added in warp
order; var = total / hidden; r = 1 / sqrt(var + eps), each step rounded.
"""
from __future__ import annotations

import numpy as np

from . import mxfp4

F32 = np.float32


def _butterfly_lane0(s: np.ndarray) -> np.ndarray:
    """[rows, 32] float32 -> lane 0's butterfly sum [rows]."""
    v = s.astype(F32).copy()
    lanes = np.arange(32)
    for off in (16, 8, 4, 2, 1):
        v = (v + v[:, lanes ^ off]).astype(F32)
    return v[:, 0]


def ar_rmsnorm_mxfp4(inputs_bits, residual_bits, weight_bits, eps: float, legacy_rule: bool = False):
    """inputs_bits: list of bf16 bits [rows, hidden] (rank order); residual
    and weight bf16 bits.  Returns (residual_out bits, out bits, nibbles
    [rows, hidden/2], scales [rows, hidden/32])."""
    acc = mxfp4.bf16_bits_to_f32(inputs_bits[0]).astype(F32)
    for x in inputs_bits[1:]:
        acc = (acc + mxfp4.bf16_bits_to_f32(x)).astype(F32)
    acc = (acc + mxfp4.bf16_bits_to_f32(residual_bits)).astype(F32)
    comb_bits = mxfp4.f32_to_bf16_bits(acc)
    c = mxfp4.bf16_bits_to_f32(comb_bits)
    rows, hidden = c.shape
    groups = hidden // 32
    sq = (c * c).astype(F32).reshape(rows, groups, 32)
    s = np.zeros((rows, groups), F32)
    for i in range(32):
        s = (s + sq[:, :, i]).astype(F32)
    nwarps = (groups + 31) // 32
    s = np.concatenate([s, np.zeros((rows, nwarps * 32 - groups), F32)], axis=1).reshape(rows, nwarps, 32)
    total = np.zeros(rows, F32)
    for w in range(nwarps):
        total = (total + _butterfly_lane0(s[:, w])).astype(F32)
    var = (total / F32(hidden)).astype(F32)
    r = (F32(1.0) / np.sqrt((var + F32(eps)).astype(F32))).astype(F32)
    normed = mxfp4.bf16_bits_to_f32(mxfp4.f32_to_bf16_bits((c * r[:, None]).astype(F32)))
    out_bits = mxfp4.f32_to_bf16_bits((normed * mxfp4.bf16_bits_to_f32(weight_bits)[None, :]).astype(F32))
    quant = mxfp4.quantize_legacy if legacy_rule else mxfp4.quantize_inline
    nib, sc = quant(out_bits)
    return comb_bits, out_bits, nib, sc
