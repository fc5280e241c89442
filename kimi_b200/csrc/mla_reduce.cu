// Split-K log-sum-exp merge of the decode partials.
//
// Restates `_mla_reduce` (archive/mla-mxfp4-dead-end/mla_decode_mxfp4_v5.py:264-306)
// in the natural-log form: w_s = exp(lse_s - max_s lse), o = sum_s w_s O_s /
// sum_s w_s, written as bf16 through arbitrary (sequence, head) strides so the
// heads-first view (patches/atom-optimizations.patch:261-289) is written in
// place.  Splits with lse = -inf (no tokens) carry no weight and their partial
// rows are never read.
//
// One 128-thread CTA per (sequence, head): each thread owns 4 consecutive
// latent columns (four values per split: bf16 partials from this library's
// decode, fp32 ones through kimi_mla_reduce), so every partial row is read once,
// fully coalesced; the kernel is bound by HBM reads of the partials.
//
// Split mode: the partials of sequence b are slots b * num_splits + s.
// Balanced mode (seq_meta set): they are slots b + c for the CTAs c in
// [meta.x, meta.y] that held b's tiles; a sequence held by one CTA was written
// by the decode kernel itself and is skipped, one without pages gets zeros.
#include <cuda_runtime.h>
#include <math_constants.h>

#include "kernels.cuh"

namespace kimi {
namespace {

__global__ void __launch_bounds__(128) mla_reduce_kernel(ReduceArgs a) {
  const int b = blockIdx.y;
  const int h = blockIdx.x;
  const int d = threadIdx.x * 4;
  int64_t first_slot = static_cast<int64_t>(b) * a.num_splits;
  int n_slots = a.num_splits;
  if (a.seq_meta) {
    if (a.kv_indptr[b + 1] <= a.kv_indptr[b]) {
      *reinterpret_cast<uint2*>(a.o + b * a.o_stride_b + h * a.o_stride_h + d) = make_uint2(0u, 0u);
      return;
    }
    const int2 span = a.seq_meta[b];
    if (span.x == span.y) return;
    first_slot = static_cast<int64_t>(b) + span.x;
    n_slots = span.y - span.x + 1;
  }
  const int64_t lse_base = first_slot * a.num_heads + h;
  float m = -CUDART_INF_F;
  for (int s = 0; s < n_slots; ++s) m = fmaxf(m, a.partial_lse[lse_base + s * a.num_heads]);
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  float wsum = 0.f;
  if (m != -CUDART_INF_F) {
    for (int s = 0; s < n_slots; ++s) {
      const float l = a.partial_lse[lse_base + s * a.num_heads];
      if (l == -CUDART_INF_F) continue;
      const float w = __expf(l - m);
      const int64_t off = (lse_base + static_cast<int64_t>(s) * a.num_heads) * kLatent + d;
      float4 v;
      if (a.partial_bf16) {
        const uint2 raw = *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(a.partial_o) + off);
        v = make_float4(__uint_as_float(raw.x << 16), __uint_as_float(raw.x & 0xFFFF0000u),
                        __uint_as_float(raw.y << 16), __uint_as_float(raw.y & 0xFFFF0000u));
      } else {
        v = *reinterpret_cast<const float4*>(static_cast<const float*>(a.partial_o) + off);
      }
      acc.x += w * v.x;
      acc.y += w * v.y;
      acc.z += w * v.z;
      acc.w += w * v.w;
      wsum += w;
    }
  }
  const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
  __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x * inv, acc.y * inv);
  __nv_bfloat162 hi = __floats2bfloat162_rn(acc.z * inv, acc.w * inv);
  uint2 packed;
  packed.x = *reinterpret_cast<uint32_t*>(&lo);
  packed.y = *reinterpret_cast<uint32_t*>(&hi);
  *reinterpret_cast<uint2*>(a.o + b * a.o_stride_b + h * a.o_stride_h + d) = packed;
}

}  // namespace

cudaError_t launch_reduce(const ReduceArgs& a, cudaStream_t stream) {
  if (a.batch == 0 || a.num_heads == 0) return cudaSuccess;
  mla_reduce_kernel<<<dim3(a.num_heads, a.batch), 128, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace kimi
