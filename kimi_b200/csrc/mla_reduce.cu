// Split-K log-sum-exp merge of the decode partials.
//
// Restates `_mla_reduce` (archive/mla-mxfp4-dead-end/mla_decode_mxfp4_v5.py:264-306)
// in the natural-log form: w_s = exp(lse_s - max_s lse), o = sum_s w_s O_s /
// sum_s w_s, written as bf16 through arbitrary (sequence, head) strides so the
// heads-first view (patches/atom-optimizations.patch:261-289) is written in
// place.  Splits with lse = -inf (no tokens) carry no weight and their partial
// rows are never read.
//
// One 256-thread CTA per (sequence, 8 heads): warp w merges head 8 x + w, lane
// l latents 16 l .. 16 l + 15.  The lanes read the splits' LSEs in parallel
// (a warp-wide max and sum give the weights), then every split row once,
// fully coalesced, four splits' loads in flight at a time; the kernel is
// bound by HBM reads of the partials.  Launched as a programmatic dependent
// of the decode kernel it waits for that grid before reading its outputs.
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

__device__ __forceinline__ void load_row16(const ReduceArgs& a, int64_t off, float (&v)[16]) {
  if (a.partial_bf16) {
    const uint4* p = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(a.partial_o) + off);
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const uint4 r = p[k];
      const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        v[8 * k + 2 * e] = __uint_as_float(w[e] << 16);
        v[8 * k + 2 * e + 1] = __uint_as_float(w[e] & 0xFFFF0000u);
      }
    }
  } else {
    const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(a.partial_o) + off);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float4 r = p[k];
      v[4 * k] = r.x;
      v[4 * k + 1] = r.y;
      v[4 * k + 2] = r.z;
      v[4 * k + 3] = r.w;
    }
  }
}

__global__ void __launch_bounds__(256) mla_reduce_kernel(ReduceArgs a) {
  const int b = blockIdx.y;
  const int lane = threadIdx.x & 31;
  const int h = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int d = 16 * lane;
  const bool empty_seq = a.seq_meta && a.kv_indptr[b + 1] <= a.kv_indptr[b];
  if (a.programmatic) asm volatile("griddepcontrol.wait;\n" ::: "memory");  // the decode grid is complete
  if (h >= a.num_heads) return;
  __nv_bfloat16* out = a.o + b * a.o_stride_b + h * a.o_stride_h + d;
  int64_t first_slot = static_cast<int64_t>(b) * a.num_splits;
  int n_slots = a.num_splits;
  if (a.seq_meta) {
    if (empty_seq) {
#pragma unroll
      for (int k = 0; k < 4; ++k) reinterpret_cast<uint2*>(out)[k] = make_uint2(0u, 0u);
      return;
    }
    const int2 span = a.seq_meta[b];
    if (span.x < 0 || span.y < span.x || span.y >= a.num_splits) {
      // Not a span the decode wrote (it gave up before recording it; its
      // status word says so): zeros, and no read outside the workspace.
#pragma unroll
      for (int k = 0; k < 4; ++k) reinterpret_cast<uint2*>(out)[k] = make_uint2(0u, 0u);
      return;
    }
    if (span.x == span.y) return;  // written by the decode kernel itself
    first_slot = static_cast<int64_t>(b) + span.x;
    n_slots = span.y - span.x + 1;
  }
  const int64_t lse_base = first_slot * a.num_heads + h;
  float acc[16];
#pragma unroll
  for (int e = 0; e < 16; ++e) acc[e] = 0.f;
  float wsum = 0.f;
  // slots in chunks of 32: lane c holds the LSE of slot c0 + c
  float m = -CUDART_INF_F, l_first = -CUDART_INF_F;
  for (int c0 = 0; c0 < n_slots; c0 += 32) {
    const float l = c0 + lane < n_slots ? a.partial_lse[lse_base + static_cast<int64_t>(c0 + lane) * a.num_heads]
                                        : -CUDART_INF_F;
    if (c0 == 0) l_first = l;
    m = fmaxf(m, l);
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (m != -CUDART_INF_F) {
    for (int c0 = 0; c0 < n_slots; c0 += 32) {
      const int nc = min(32, n_slots - c0);
      const float l = c0 == 0 ? l_first
                              : lane < nc ? a.partial_lse[lse_base + static_cast<int64_t>(c0 + lane) * a.num_heads]
                                          : -CUDART_INF_F;
      const float wl = l == -CUDART_INF_F ? 0.f : __expf(l - m);
      float ws = wl;
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) ws += __shfl_xor_sync(0xffffffffu, ws, o);
      wsum += ws;
      // four splits' rows in flight at a time (rows of weight-0 splits are not read)
      for (int c = 0; c < nc; c += 4) {
        float v[4][16];
        float w[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          w[k] = __shfl_sync(0xffffffffu, wl, (c + k) & 31);
          if (c + k < nc && w[k] != 0.f)
            load_row16(a, (lse_base + static_cast<int64_t>(c0 + c + k) * a.num_heads) * kLatent + d, v[k]);
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          if (c + k < nc && w[k] != 0.f) {
#pragma unroll
            for (int e = 0; e < 16; ++e) acc[e] += w[k] * v[k][e];
          }
        }
      }
    }
  }
  const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const __nv_bfloat162 lo = __floats2bfloat162_rn(acc[4 * k] * inv, acc[4 * k + 1] * inv);
    const __nv_bfloat162 hi = __floats2bfloat162_rn(acc[4 * k + 2] * inv, acc[4 * k + 3] * inv);
    reinterpret_cast<uint2*>(out)[k] =
        make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
  }
}

}  // namespace

cudaError_t launch_reduce(const ReduceArgs& a, cudaStream_t stream) {
  if (a.batch == 0 || a.num_heads == 0) return cudaSuccess;
  const dim3 grid((a.num_heads + 7) / 8, a.batch);
  if (!a.programmatic) {
    mla_reduce_kernel<<<grid, 256, 0, stream>>>(a);
    return cudaGetLastError();
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, mla_reduce_kernel, a);
}

}  // namespace kimi
