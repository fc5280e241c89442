"""MXFP4 (OCP microscaling, e2m1 elements + e8m0 block scale) in numpy.

TEST INFRASTRUCTURE ONLY (the oracle): imported by tests, smoke() and the
bench CPU baseline, never by the product package.

Everything here is integer / float32 arithmetic in numpy that restates the
reference bit for bit:

* :func:`quantize_inline` -- ``_mxfp4_quant_inline``
  (archive/mla-mxfp4-dead-end/mla_decode_mxfp4_v5.py:18-75), the rule the
  decode path's KV-append quantiser follows by default.
* :func:`quantize_legacy` -- ``_quantize_mxfp4_torch``
  (archive/mla-mxfp4-dead-end/mla_decode_mxfp4_v5.py:421-438), the host torch
  rule the archive tests used to build their caches.  Its scale choice
  (``floor(log2(amax)) + 2``) only ever uses the e2m1 codes 0 and 0.5; it is
  reproduced byte for byte because it is the reference's behaviour, not
  because it is a good quantiser.
* :func:`dequantize` -- ``_dequant_mxfp4_torch``
  (archive/mla-mxfp4-dead-end/mla_decode_mxfp4_v5.py:381-400).

bf16 tensors are carried as ``uint16`` bit patterns (numpy has no bf16).
"""
from __future__ import annotations

import numpy as np

GROUP = 32  # elements per e8m0 scale (v5.py:15 SCALE_GROUP_SIZE)

# e2m1 magnitude table, v5.py:83-96 and v5.py:382 / :422.
E2M1_VALUES = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float32)


# --------------------------------------------------------------------------
# bf16 helpers
# --------------------------------------------------------------------------
def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """uint16 bf16 bit patterns -> float32 (exact)."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns, round-to-nearest-even (torch's ``.to(bfloat16)``)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    out = rounded.astype(np.uint16)
    out[nan] = 0x7FC0
    return out


def _as_f32(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x)
    if x.dtype == np.uint16:
        return bf16_bits_to_f32(x)
    return x.astype(np.float32)


def _pack_pairs(codes: np.ndarray) -> np.ndarray:
    """[..., D] uint8 4-bit codes -> [..., D/2] bytes; element 2j in the low
    nibble, element 2j+1 in the high nibble (v5.py:71-73, :435-437)."""
    return (codes[..., 0::2] | (codes[..., 1::2] << 4)).astype(np.uint8)


# --------------------------------------------------------------------------
# Inline (device) rule -- v5.py:18-75
# --------------------------------------------------------------------------
def scale_exponent_inline(amax: np.ndarray) -> np.ndarray:
    """Unbiased e8m0 exponent chosen by the in-kernel rule.

    v5.py:36-40: round amax up at mantissa 0b11 (``+0x200000`` then clear the
    mantissa), ``floor(log2(.)) - 2``, clamp to [-127, 127].  The rounded
    amax is an exact power of two (or 0 / inf), so ``floor(log2())`` is read
    off the exponent field instead of calling a libm ``log2``.
    """
    bits = np.ascontiguousarray(amax, dtype=np.float32).view(np.int32).astype(np.int64)
    bits = ((bits + 0x200000) & 0xFF800000) & 0xFFFFFFFF
    exp_field = (bits >> 23) & 0xFF
    e = exp_field.astype(np.float64) - 127.0
    e[exp_field == 0] = -np.inf   # rounded amax == 0 -> log2 = -inf
    e[exp_field == 255] = np.inf  # rounded amax == inf
    e = np.clip(e - 2.0, -127.0, 127.0)
    return e.astype(np.int32)


def _pow2_f32(e: np.ndarray) -> np.ndarray:
    """Exact float32 2**e for integer e in [-149, 127] (subnormals included)."""
    return np.ldexp(np.float32(1.0), e.astype(np.int32)).astype(np.float32)


def e2m1_round_inline(qx: np.ndarray) -> np.ndarray:
    """float32 -> 4-bit e2m1 code with sign, v5.py:43-70.

    Magnitudes >= 6 saturate to code 7; magnitudes < 1 go through the
    "denormal" path (add 2**22 in float32 so the FPU rounds to a multiple of
    0.5 with ties-to-even); the rest round the mantissa to 1 bit with
    ties-to-even by integer add of ``0x1FFFFF + lsb``.
    """
    qx = np.ascontiguousarray(qx, dtype=np.float32)
    qbits = qx.view(np.uint32)
    sign = qbits & np.uint32(0x80000000)
    abits = qbits ^ sign
    qabs = abits.view(np.float32)
    with np.errstate(invalid="ignore"):
        sat = qabs >= np.float32(6.0)
        den = (~sat) & (qabs < np.float32(1.0))
    nrm = ~(sat | den)
    # denormal path: (127-1) + (23-1) + 1 = 149 -> magic 2**22 (v5.py:51-57)
    magic = np.uint32(149 << 23)
    den_code = ((qabs + np.float32(2.0 ** 22)).view(np.uint32) - magic).astype(np.uint8)
    # normal path (v5.py:58-64); arithmetic is modulo 2**32 as in uint32
    mant_odd = (abits >> np.uint32(22)) & np.uint32(1)
    add = np.uint32((((1 - 127) << 23) + (1 << 21) - 1) & 0xFFFFFFFF)
    nrm_bits = (abits.astype(np.uint64) + int(add) + mant_odd.astype(np.uint64)) & 0xFFFFFFFF
    nrm_code = (nrm_bits >> 22).astype(np.uint8)
    code = np.full(qx.shape, 7, dtype=np.uint8)
    code = np.where(nrm, nrm_code, code)
    code = np.where(den, den_code, code)
    code = code | (sign >> np.uint32(28)).astype(np.uint8)  # sign -> bit 3 (v5.py:68-70)
    return code.astype(np.uint8)


def quantize_inline(x: np.ndarray):
    """[N, D] float32 or bf16-bits -> (nibbles uint8 [N, D/2], scales uint8 [N, D/32]).

    The scale byte is ``e + 127`` for the unbiased exponent ``e`` in
    [-127, 127] (v5.py:41).
    """
    xf = _as_f32(x)
    n, d = xf.shape
    assert d % GROUP == 0
    g = xf.reshape(n, d // GROUP, GROUP)
    amax = np.abs(g).max(axis=-1)
    e = scale_exponent_inline(amax)
    scales = (e + 127).astype(np.uint8)
    qx = g * _pow2_f32(-e)[..., None]  # v5.py:42-43, exact power-of-two scaling
    codes = e2m1_round_inline(qx).reshape(n, d)
    return _pack_pairs(codes), scales


# --------------------------------------------------------------------------
# Legacy torch rule -- v5.py:421-438
# --------------------------------------------------------------------------
def scale_exponent_legacy(amax: np.ndarray) -> np.ndarray:
    """``floor(log2(max(amax, 1e-12))) + 2`` clamped to [-127, 127] (v5.py:425-427).

    For bf16-valued inputs (the cache input dtype) ``amax`` has at most 8
    significant bits, so the float32 ``log2`` of the reference never rounds
    up to the next integer and the floor equals the exponent field, which is
    what this reads.
    """
    a = np.maximum(np.ascontiguousarray(amax, dtype=np.float32), np.float32(1e-12))
    _, exp2 = np.frexp(a)  # a = m * 2**exp2 with m in [0.5, 1)
    e = exp2.astype(np.int64) - 1 + 2
    return np.clip(e, -127, 127).astype(np.int32)


def e2m1_round_legacy(t_scaled: np.ndarray) -> np.ndarray:
    """Nearest e2m1 magnitude by ``argmin |t| - value`` (ties -> lower code),
    sign from ``t < 0`` (v5.py:431-435)."""
    t = np.ascontiguousarray(t_scaled, dtype=np.float32)
    sign = (t < 0).astype(np.uint8)
    ta = np.abs(t)
    diffs = np.abs(ta[..., None] - E2M1_VALUES)
    mag = np.argmin(diffs, axis=-1).astype(np.uint8)  # first minimum == lower code on ties
    return (sign << 3) | mag


def quantize_legacy(x: np.ndarray):
    """[N, D] float32 or bf16-bits -> (nibbles [N, D/2], scales [N, D/32]) by the
    legacy torch rule (scale byte ``clamp(e + 127, 0, 254)``, v5.py:428)."""
    xf = _as_f32(x)
    n, d = xf.shape
    assert d % GROUP == 0
    g = xf.reshape(n, d // GROUP, GROUP)
    amax = np.abs(g).max(axis=-1)
    e = scale_exponent_legacy(amax)
    scales = np.clip(e + 127, 0, 254).astype(np.uint8)
    t_scaled = g / _pow2_f32(e)[..., None]
    codes = e2m1_round_legacy(t_scaled).reshape(n, d)
    return _pack_pairs(codes), scales


# --------------------------------------------------------------------------
# Dequantiser -- v5.py:381-400
# --------------------------------------------------------------------------
def dequantize(nibbles: np.ndarray, scales: np.ndarray, dim: int | None = None) -> np.ndarray:
    """(nibbles [N, D/2], scales [N, D/32]) -> float32 [N, D].

    ``(-1)**b3 * E2M1[b2..b0] * 2**(s - 127)`` with the low nibble holding the
    even element.  Scale byte 255 decodes to +inf as ``torch.pow(2.0, 128.)``
    does in the reference.
    """
    nib = np.asarray(nibbles, dtype=np.uint8)
    sc = np.asarray(scales, dtype=np.uint8)
    n = nib.shape[0]
    d = nib.shape[1] * 2 if dim is None else dim
    lo = nib & 0x0F
    hi = (nib >> 4) & 0x0F
    vals = np.empty((n, d), dtype=np.float32)
    vals[:, 0::2] = np.where(lo & 8, -1.0, 1.0).astype(np.float32) * E2M1_VALUES[lo & 7]
    vals[:, 1::2] = np.where(hi & 8, -1.0, 1.0).astype(np.float32) * E2M1_VALUES[hi & 7]
    with np.errstate(over="ignore"):
        scale_f = np.ldexp(np.float32(1.0), sc.astype(np.int32) - 127).astype(np.float32)
    scale_f = np.repeat(scale_f, GROUP, axis=1)[:, :d]
    with np.errstate(invalid="ignore", over="ignore"):
        return (vals * scale_f).astype(np.float32)
