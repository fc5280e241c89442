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
// latent columns (one float4 per split), so every partial row is read once,
// fully coalesced; the kernel is bound by HBM reads of the partials.
#include <cuda_runtime.h>
#include <math_constants.h>

#include "kernels.cuh"

namespace kimi {
namespace {

__global__ void __launch_bounds__(128) mla_reduce_kernel(ReduceArgs a) {
  const int b = blockIdx.y;
  const int h = blockIdx.x;
  const int d = threadIdx.x * 4;
  const int64_t lse_base = static_cast<int64_t>(b) * a.num_splits * a.num_heads + h;
  float m = -CUDART_INF_F;
  for (int s = 0; s < a.num_splits; ++s) m = fmaxf(m, a.partial_lse[lse_base + s * a.num_heads]);
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  float wsum = 0.f;
  if (m != -CUDART_INF_F) {
    for (int s = 0; s < a.num_splits; ++s) {
      const float l = a.partial_lse[lse_base + s * a.num_heads];
      if (l == -CUDART_INF_F) continue;
      const float w = __expf(l - m);
      const float4 v = *reinterpret_cast<const float4*>(
          a.partial_o + (lse_base + static_cast<int64_t>(s) * a.num_heads) * kLatent + d);
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
