// Split-K log-sum-exp merge of the decode partials.
//
// Restates `_mla_reduce` (archive/mla-mxfp4-dead-end/mla_decode_mxfp4_v5.py:264-306)
// in the natural-log form: w_s = exp(lse_s - max_s lse), o = sum_s w_s O_s /
// sum_s w_s, written as bf16 through arbitrary (sequence, head) strides so the
// heads-first view (patches/atom-optimizations.patch:261-289) is written in
// place.  Splits with lse = -inf (no tokens) carry no weight and their partial
// rows are never read.
//
// One 128-thread CTA per (sequence, 8 heads): half-warp hw of the CTA merges
// head 8 x + hw, its lane l latents 32 l .. 32 l + 31.  The 16 lanes of a
// head read the splits' LSEs in parallel (a half-warp max and sum give the
// weights), then every split row once, fully coalesced (1 KB per head), two
// splits' rows in flight at a time.  The kernel is bound by the latency of
// these dependent loads, so it is sized to run in one wave (a batch of 64
// sequences x 64 heads is 512 CTAs at 4 per SM).  Launched as a programmatic
// dependent of the decode kernel it waits for that grid before reading its
// outputs.
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

// 32 fp32 latents of one partial row
__device__ __forceinline__ void load_row32(const ReduceArgs& a, int64_t off, float (&v)[32]) {
  const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(a.partial_o) + off);
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const float4 r = p[k];
    v[4 * k] = r.x;
    v[4 * k + 1] = r.y;
    v[4 * k + 2] = r.z;
    v[4 * k + 3] = r.w;
  }
}

// 32 latents of one output row (8-byte aligned) as bf16
__device__ __forceinline__ void store_row32(__nv_bfloat16* out, const float (&acc)[32], float scale) {
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const __nv_bfloat162 lo = __floats2bfloat162_rn(acc[4 * k] * scale, acc[4 * k + 1] * scale);
    const __nv_bfloat162 hi = __floats2bfloat162_rn(acc[4 * k + 2] * scale, acc[4 * k + 3] * scale);
    reinterpret_cast<uint2*>(out)[k] =
        make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
  }
}

template <bool kBf16>
__global__ void __launch_bounds__(128, 4) mla_reduce_kernel(ReduceArgs a) {
  constexpr unsigned kAll = 0xffffffffu;
  const int b = blockIdx.y;
  const int lane = threadIdx.x & 31, sl = lane & 15;
  const int h = blockIdx.x * 8 + (threadIdx.x >> 4);
  const bool live = h < a.num_heads;  // a half-warp past the last head still takes part in the shuffles
  const int d = 32 * sl;
  const bool empty_seq = a.seq_meta && a.kv_indptr[b + 1] <= a.kv_indptr[b];
  if (a.programmatic) asm volatile("griddepcontrol.wait;\n" ::: "memory");  // the decode grid is complete
  __nv_bfloat16* out = a.o + b * a.o_stride_b + h * a.o_stride_h + d;
  float acc[32];
#pragma unroll
  for (int e = 0; e < 32; ++e) acc[e] = 0.f;
  int64_t first_slot = static_cast<int64_t>(b) * a.num_splits;
  int n_slots = a.num_splits;
  if (a.seq_meta) {  // (uniform over the CTA: one sequence)
    const int2 span = empty_seq ? make_int2(0, 0) : a.seq_meta[b];
    if (empty_seq || span.x < 0 || span.y < span.x || span.y >= a.num_splits) {
      // No pages, or not a span the decode wrote (it gave up before recording
      // it; its status word says so): zeros, and no read outside the workspace.
      if (live) store_row32(out, acc, 0.f);
      return;
    }
    if (span.x == span.y) return;  // written by the decode kernel itself
    first_slot = static_cast<int64_t>(b) + span.x;
    n_slots = span.y - span.x + 1;
  }
  const int64_t lse_base = first_slot * a.num_heads + h;
  float wsum = 0.f;
  // slots in chunks of 16: lane l of the half-warp holds the LSE of slot c0 + l
  float m = -CUDART_INF_F, l_first = -CUDART_INF_F;
  for (int c0 = 0; c0 < n_slots; c0 += 16) {
    const float l = live && c0 + sl < n_slots
                        ? a.partial_lse[lse_base + static_cast<int64_t>(c0 + sl) * a.num_heads]
                        : -CUDART_INF_F;
    if (c0 == 0) l_first = l;
    m = fmaxf(m, l);
  }
#pragma unroll
  for (int o = 8; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(kAll, m, o, 16));
  // both half-warps run every step below (the shuffles need all 32 lanes);
  // a head without weight (m = -inf) adds nothing
  for (int c0 = 0; c0 < n_slots; c0 += 16) {
    const int nc = min(16, n_slots - c0);
    const float l = c0 == 0 ? l_first
                            : live && sl < nc
                                  ? a.partial_lse[lse_base + static_cast<int64_t>(c0 + sl) * a.num_heads]
                                  : -CUDART_INF_F;
    const float wl = (l == -CUDART_INF_F || m == -CUDART_INF_F) ? 0.f : __expf(l - m);
    float ws = wl;
#pragma unroll
    for (int o = 8; o >= 1; o >>= 1) ws += __shfl_xor_sync(kAll, ws, o, 16);
    wsum += ws;
    // two splits' rows in flight at a time, in slot order (rows of weight-0
    // splits are not read)
    for (int c = 0; c < nc; c += 2) {
      float w[2];
#pragma unroll
      for (int k = 0; k < 2; ++k) w[k] = __shfl_sync(kAll, wl, (c + k) & 15, 16);
      if constexpr (kBf16) {
        // the rows stay packed (16 registers each) until they are accumulated
        uint4 raw[2][4];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          if (c + k < nc && w[k] != 0.f) {
            const uint4* p = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(a.partial_o) +
                                                            (lse_base + static_cast<int64_t>(c0 + c + k) * a.num_heads) *
                                                                kLatent + d);
#pragma unroll
            for (int q = 0; q < 4; ++q) raw[k][q] = p[q];
          }
        }
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          if (c + k < nc && w[k] != 0.f) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const uint32_t wd[4] = {raw[k][q].x, raw[k][q].y, raw[k][q].z, raw[k][q].w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                acc[8 * q + 2 * e] += w[k] * __uint_as_float(wd[e] << 16);
                acc[8 * q + 2 * e + 1] += w[k] * __uint_as_float(wd[e] & 0xFFFF0000u);
              }
            }
          }
        }
      } else {
        float v[2][32];
#pragma unroll
        for (int k = 0; k < 2; ++k)
          if (c + k < nc && w[k] != 0.f)
            load_row32(a, (lse_base + static_cast<int64_t>(c0 + c + k) * a.num_heads) * kLatent + d, v[k]);
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          if (c + k < nc && w[k] != 0.f) {
#pragma unroll
            for (int e = 0; e < 32; ++e) acc[e] += w[k] * v[k][e];
          }
        }
      }
    }
  }
  if (live) store_row32(out, acc, wsum > 0.f ? 1.f / wsum : 0.f);
}

}  // namespace

cudaError_t launch_reduce(const ReduceArgs& a, cudaStream_t stream) {
  if (a.batch == 0 || a.num_heads == 0) return cudaSuccess;
  const dim3 grid((a.num_heads + 7) / 8, a.batch);
  if (!a.programmatic) {
    if (a.partial_bf16)
      mla_reduce_kernel<true><<<grid, 128, 0, stream>>>(a);
    else
      mla_reduce_kernel<false><<<grid, 128, 0, stream>>>(a);
    return cudaGetLastError();
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(128);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return a.partial_bf16 ? cudaLaunchKernelEx(&cfg, mla_reduce_kernel<true>, a)
                        : cudaLaunchKernelEx(&cfg, mla_reduce_kernel<false>, a);
}

}  // namespace kimi
