"""The decode step after attention: V up-projection by W_UV, then o_proj.

TEST INFRASTRUCTURE ONLY (the oracle): imported by tests, never by the
product package.

Restates ``MLAAttention._v_up_proj_and_o_proj(x, heads_first=True)``
(patches/atom-optimizations.patch:131-143, called on the decode's
heads-first output at :297-302) as the reference's own test states it
(tests/test_mla_heads_first_e2e.py:50-59, ``forward_heads_first``):

* ``x = bmm(o.float(), W_V.float()).to(bf16)``: o [N, B, 512] heads-first,
  W_V [N, 512, 128], one rounding to bf16 of the float32 product;
* ``x`` transposed to [B, N * 128] (head-major columns);
* ``out = mm(x, o_proj_weight.T)`` in bf16: o_proj_weight [hidden, N * 128],
  float32 accumulation, one rounding to bf16.

The products are accumulated here in float64 and rounded to float32, then to
bf16; a float32 accumulation in another order can land one bf16 step away
near a rounding boundary, so comparisons use a tolerance.
"""
from __future__ import annotations

import numpy as np

from . import mxfp4


def v_up_o_proj(o_bits: np.ndarray, w_uv_bits: np.ndarray, w_o_bits: np.ndarray):
    """o_bits bf16 bits [N, B, 512], w_uv_bits [N, 512, 128], w_o_bits
    [hidden, N * 128] -> (x bits [B, N * 128], out bits [B, hidden])."""
    o = mxfp4.bf16_bits_to_f32(o_bits).astype(np.float64)
    w_uv = mxfp4.bf16_bits_to_f32(w_uv_bits).astype(np.float64)
    w_o = mxfp4.bf16_bits_to_f32(w_o_bits).astype(np.float64)
    n, b, _ = o.shape
    x = np.einsum("nbl,nlv->bnv", o, w_uv).astype(np.float32)          # [B, N, 128]
    x_bits = mxfp4.f32_to_bf16_bits(x.reshape(b, n * w_uv.shape[2]))
    xb = mxfp4.bf16_bits_to_f32(x_bits).astype(np.float64)
    out = (xb @ w_o.T).astype(np.float32)
    return x_bits, mxfp4.f32_to_bf16_bits(out)
