// MXFP4 (e2m1 elements, e8m0 scale per 32) device helpers shared by the
// KV-append quantiser and the decode kernels.
//
// Quantiser rules (bit-exact restatements; paths inside ianye23301/kimi):
//   inline  -- `_mxfp4_quant_inline`, archive/mla-mxfp4-dead-end/mla_decode_mxfp4_v5.py:18-75
//   legacy  -- `_quantize_mxfp4_torch`, archive/mla-mxfp4-dead-end/mla_decode_mxfp4_v5.py:421-438
// Dequant -- `_dequant_mxfp4_torch`, same file :381-400.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>

namespace kimi {

// ---------------------------------------------------------------------------
// Scale choice
// ---------------------------------------------------------------------------

// Inline rule, v5.py:36-41: round amax up when its mantissa is >= 0b11
// (add 0x200000, clear the mantissa), take floor(log2()) - 2 and clamp to
// [-127, 127].  The rounded amax is a power of two, 0 or inf, so the floor
// of its log2 is its exponent field.  Returns the unbiased exponent e.
__device__ __forceinline__ int scale_exp_inline(float amax) {
  const uint32_t r = (__float_as_uint(amax) + 0x200000u) & 0xFF800000u;
  const int ef = static_cast<int>(r >> 23);
  if (ef == 0) return -127;   // log2(0) = -inf, clamped
  if (ef >= 255) return 127;  // inf, clamped
  int e = ef - 127 - 2;
  return e < -127 ? -127 : e;
}

// Legacy rule, v5.py:425-427: floor(log2(max(amax, 1e-12))) + 2 clamped to
// [-127, 127].  max(amax, 1e-12) is a normal float, so floor(log2()) is its
// exponent field (inputs are bf16-valued; see the oracle's note).
__device__ __forceinline__ int scale_exp_legacy(float amax) {
  const float a = fmaxf(amax, 1e-12f);
  const int ef = static_cast<int>((__float_as_uint(a) >> 23) & 0xFF);
  if (ef >= 255) return 127;
  int e = ef - 127 + 2;
  return e > 127 ? 127 : e;
}

// Exact float 2^k for integer k in [-127, 127] (2^-127 is a subnormal).
__device__ __forceinline__ float exp2i(int k) {
  return k >= -126 ? __uint_as_float(static_cast<uint32_t>(k + 127) << 23) : __uint_as_float(0x00400000u);
}

// ---------------------------------------------------------------------------
// Element rounding
// ---------------------------------------------------------------------------

// Inline rule, v5.py:43-70: saturate at 6 to code 7; magnitudes below 1 are
// rounded to a multiple of 0.5 by a float add of 2^22 (ties to even); the rest
// round the mantissa to one bit with ties to even by integer add.  The sign
// lands in bit 3 (so -0.0 gives code 8).
__device__ __forceinline__ uint32_t e2m1_code_inline(float qx) {
  const uint32_t bits = __float_as_uint(qx);
  const uint32_t s = bits & 0x80000000u;
  const uint32_t a = bits ^ s;
  const float qa = __uint_as_float(a);
  uint32_t code;
  if (qa >= 6.0f) {
    code = 7u;
  } else if (qa < 1.0f) {
    code = __float_as_uint(__fadd_rn(qa, 4194304.0f)) - (149u << 23);
  } else {
    // ((1 - 127) << 23) + (1 << 21) - 1 modulo 2^32, plus the mantissa lsb
    code = (a + 0xC11FFFFFu + ((a >> 22) & 1u)) >> 22;
  }
  return (code & 0xFFu) | (s >> 28);
}

// Legacy rule, v5.py:431-435: nearest e2m1 value by argmin of |t| - value,
// the lower code on ties (so the comparisons against the midpoints are
// strict); sign bit set for t < 0 (so -0.0 gives code 0).  +-inf picks the
// first table entry, as argmin over an all-inf row does.
__device__ __forceinline__ uint32_t e2m1_code_legacy(float t) {
  const float ta = fabsf(t);
  uint32_t mag = 0;
  if (!(ta == __int_as_float(0x7F800000))) {
    mag = (ta > 0.25f) + (ta > 0.75f) + (ta > 1.25f) + (ta > 1.75f) + (ta > 2.5f) + (ta > 3.5f) +
          (ta > 5.0f);
  }
  return mag | (t < 0.0f ? 8u : 0u);
}

// Quantise one group of 32 floats held by the caller (in registers) into 16
// packed bytes (4 x u32, element 2j in the low nibble of byte j) and a scale
// byte.  LEGACY selects the rule.
template <bool LEGACY>
__device__ __forceinline__ void quantize_group32(const float (&x)[32], uint32_t (&packed)[4],
                                                 uint8_t& scale_byte) {
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(x[i]));
  if (LEGACY) {
    const int e = scale_exp_legacy(amax);
    int sb = e + 127;
    sb = sb < 0 ? 0 : (sb > 254 ? 254 : sb);
    scale_byte = static_cast<uint8_t>(sb);
    // t = x / 2^e, computed as an exact-rounded multiply by 2^-e (same value)
    const float inv = exp2i(-e < -127 ? -127 : -e);
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      uint32_t v = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) v |= e2m1_code_legacy(__fmul_rn(x[w * 8 + j], inv)) << (4 * j);
      packed[w] = v;
    }
  } else {
    const int e = scale_exp_inline(amax);
    scale_byte = static_cast<uint8_t>(e + 127);
    const float qs = exp2i(-e);
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      uint32_t v = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) v |= e2m1_code_inline(__fmul_rn(x[w * 8 + j], qs)) << (4 * j);
      packed[w] = v;
    }
  }
}

// ---------------------------------------------------------------------------
// Dequant
// ---------------------------------------------------------------------------

// e2m1 code (4 bits, sign in bit 3) -> float, v5.py:381-390.
__device__ __forceinline__ float e2m1_to_float(uint32_t code) {
  const uint32_t mag = code & 7u;
  const uint32_t e = mag >> 1;
  uint32_t bits = e ? (((e + 126u) << 23) | ((mag & 1u) << 22)) : (mag ? 0x3F000000u : 0u);
  return __uint_as_float(bits | ((code & 8u) << 28));
}

// e8m0 scale byte -> float 2^(s - 127) (255 -> +inf as torch.pow(2, 128)).
__device__ __forceinline__ float e8m0_to_float(uint32_t s) {
  if (s == 0u) return __uint_as_float(0x00400000u);
  if (s == 255u) return __uint_as_float(0x7F800000u);
  return __uint_as_float(s << 23);
}

// Eight packed nibbles (one u32 of the cache) times a scale -> four bf16x2
// words, element order preserved.  Exact: every e2m1 * 2^k is a bf16 value.
__device__ __forceinline__ void dequant8_bf16(uint32_t nib8, float scale, uint32_t (&out)[4]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float lo = __fmul_rn(e2m1_to_float((nib8 >> (8 * j)) & 0xFu), scale);
    const float hi = __fmul_rn(e2m1_to_float((nib8 >> (8 * j + 4)) & 0xFu), scale);
    __nv_bfloat162 h2 = __floats2bfloat162_rn(lo, hi);
    out[j] = *reinterpret_cast<uint32_t*>(&h2);
  }
}

}  // namespace kimi
