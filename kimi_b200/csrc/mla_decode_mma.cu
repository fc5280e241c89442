// Split-K absorbed-MLA decode over the MXFP4 paged cache, warp-level MMA
// (mma.sync m16n8k16 bf16) variant.
//
// Algorithm (paths inside ianye23301/kimi): the archive stage-1 kernel
// `_mla_decode_split_kv` (archive/mla-mxfp4-dead-end/mla_decode_mxfp4_v5.py:136-261)
// with the contract of `reference_mla_decode`
// (tests/test_triton_mla_decode.py:12-62): S = q_nope.k_nope + q_pe.k_pe,
// softmax(S * sm_scale) online in base 2 with sm_scale * log2(e) folded in,
// O = P . k_nope.  The latent is dequantised exactly to bf16 in shared memory
// (e2m1 * 2^(s-127) is a bf16 value), so QK^T and PV run on bf16 operands
// with fp32 accumulation.
//
// CTA = (split, sequence, 64-head block); 256 threads = 8 warps.  Warp w owns
// heads 16*(w&3)..+16; for QK^T it takes tokens 32*(w>>2)..+32 of the page,
// for PV latent columns 256*(w>>2)..+256.  One page (64 tokens) per
// iteration; the next page streams in with cp.async while this one is used.
#include <cuda_runtime.h>
#include <math_constants.h>

#include "kernels.cuh"
#include "mxfp4.cuh"

namespace kimi {
namespace {

constexpr int kHB = 64;                  // heads per CTA
constexpr int kThreads = 256;
constexpr int kPitch = kQkDim + 8;       // bf16 row pitch of the Q and K/V tiles (1168 B)
constexpr int kPPitch = kPageSize + 8;   // bf16 row pitch of P (144 B)
constexpr int kRawBytes = kPageBytes + kPageScaleBytes;

struct __align__(16) Smem {
  __nv_bfloat16 q[kHB * kPitch];
  __nv_bfloat16 k[kPageSize * kPitch];
  uint8_t raw[2][kRawBytes];
  __nv_bfloat16 p[kHB * kPPitch];
  float rmax[2][kHB];
  float rsum[2][kHB];
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(dst)), "l"(src));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Issue the cp.async copies of one page (384 B per token + 16 scale bytes per token).
// A page id outside [0, num_pages) is never dereferenced: its slot is zero-filled.
__device__ __forceinline__ void load_page(uint8_t* dst, const DecodeArgs& a, int page) {
  if (page < 0 || page >= a.num_pages) {
    for (int c = threadIdx.x; c < kRawBytes / 16; c += kThreads)
      *reinterpret_cast<uint4*>(dst + c * 16) = make_uint4(0, 0, 0, 0);
    return;
  }
  const uint8_t* src = a.kv_buffer + static_cast<int64_t>(page) * kPageBytes;
  const uint8_t* ssrc = a.kv_scales + static_cast<int64_t>(page) * kPageScaleBytes;
  for (int c = threadIdx.x; c < kPageBytes / 16; c += kThreads) cp_async16(dst + c * 16, src + c * 16);
  for (int c = threadIdx.x; c < kPageScaleBytes / 16; c += kThreads)
    cp_async16(dst + kPageBytes + c * 16, ssrc + c * 16);
}

__global__ void __launch_bounds__(kThreads, 1) mla_decode_mma_kernel(DecodeArgs a) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw);

  const int split = blockIdx.x;
  const int b = blockIdx.y;
  const int head_base = blockIdx.z * kHB;
  const int heads_here = min(kHB, a.num_heads - head_base);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int hg = warp & 3;
  const int half = warp >> 2;

  const int page_lo = a.kv_indptr[b];
  const int n_pages = a.kv_indptr[b + 1] - page_lo;
  const int last_len =
      n_pages == 0 ? 0 : min(max(a.kv_last_page_len ? a.kv_last_page_len[b] : kPageSize, 1), kPageSize);
  const int n_tok = n_pages == 0 ? 0 : (n_pages - 1) * kPageSize + last_len;
  const int pps = (n_pages + a.num_splits - 1) / a.num_splits;
  const int p_begin = split * pps;
  const int p_end = min(p_begin + pps, n_pages);
  const bool direct = a.num_splits == 1;

  if (p_begin >= p_end) {
    // Empty split: lse = -inf (the merge skips it); an empty sequence with a
    // single split writes zeros, as the reference leaves o at zero.
    if (direct) {
      for (int i = threadIdx.x; i < heads_here * (kLatent / 2); i += kThreads) {
        const int h = i / (kLatent / 2), d = (i % (kLatent / 2)) * 2;
        *reinterpret_cast<uint32_t*>(a.o + b * a.o_stride_b + (head_base + h) * a.o_stride_h + d) = 0u;
      }
    } else if (threadIdx.x < heads_here) {
      a.partial_lse[(static_cast<int64_t>(b) * a.num_splits + split) * a.num_heads + head_base + threadIdx.x] =
          -CUDART_INF_F;
    }
    return;
  }

  // Q (bf16 [heads, 576]) -> smem, zero rows beyond num_heads.
  for (int c = threadIdx.x; c < kHB * (kQkDim / 8); c += kThreads) {
    const int h = c / (kQkDim / 8), col = (c % (kQkDim / 8)) * 8;
    __nv_bfloat16* dst = sm.q + h * kPitch + col;
    if (h < heads_here)
      cp_async16(dst, a.q + b * a.q_stride_b + (head_base + h) * a.q_stride_h + col);
    else
      *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
  }
  load_page(sm.raw[0], a, a.kv_indices[page_lo + p_begin]);
  cp_async_commit();

  const float c_log2 = a.sm_scale * kLog2e;
  float m_r[2] = {-CUDART_INF_F, -CUDART_INF_F};  // running max (log2 units), rows r0 / r0+8
  float l_r[2] = {0.f, 0.f};                      // running sum over this warp's token half
  float o_acc[32][4];
#pragma unroll
  for (int j = 0; j < 32; ++j) o_acc[j][0] = o_acc[j][1] = o_acc[j][2] = o_acc[j][3] = 0.f;

  const int r0 = lane >> 2;
  const int cq = (lane & 3) * 2;

  for (int p = p_begin; p < p_end; ++p) {
    const int buf = (p - p_begin) & 1;
    if (p + 1 < p_end) {
      load_page(sm.raw[buf ^ 1], a, a.kv_indices[page_lo + p + 1]);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const int valid = min(kPageSize, n_tok - p * kPageSize);

    // ---- dequant: warp handles tokens warp*8..+8; lane covers 16 latent elements ----
    {
      const uint8_t* raw = sm.raw[buf];
#pragma unroll 2
      for (int i = 0; i < 8; ++i) {
        const int t = warp * 8 + i;
        uint4 w0, w1;
        if (t < valid) {
          const uint2 nib = *reinterpret_cast<const uint2*>(raw + t * kTokenBytes + lane * 8);
          const float sc = e8m0_to_float(raw[kPageBytes + t * kScaleBytes + (lane >> 1)]);
          uint32_t o0[4], o1[4];
          dequant8_bf16(nib.x, sc, o0);
          dequant8_bf16(nib.y, sc, o1);
          w0 = make_uint4(o0[0], o0[1], o0[2], o0[3]);
          w1 = make_uint4(o1[0], o1[1], o1[2], o1[3]);
        } else {
          w0 = w1 = make_uint4(0, 0, 0, 0);
        }
        uint4* dst = reinterpret_cast<uint4*>(sm.k + t * kPitch + lane * 16);
        dst[0] = w0;
        dst[1] = w1;
      }
      // RoPE part: 128 bytes per token, 8 lanes per token, 4 tokens per pass
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int t = warp * 8 + i * 4 + (lane >> 3);
        const int chunk = lane & 7;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (t < valid) v = *reinterpret_cast<const uint4*>(raw + t * kTokenBytes + kNibbleBytes + chunk * 16);
        *reinterpret_cast<uint4*>(sm.k + t * kPitch + kLatent + chunk * 8) = v;
      }
    }
    __syncthreads();

    // ---- S = Q K^T for heads 16*hg..+16, tokens 32*half..+32 ----
    float s_acc[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) s_acc[j][0] = s_acc[j][1] = s_acc[j][2] = s_acc[j][3] = 0.f;
    {
      const int a_row = hg * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
      const int a_col = (lane >> 4) * 8;
      const uint32_t a_base = smem_u32(sm.q + a_row * kPitch + a_col);
      const int mi = lane >> 3;
      const int b_tok = half * 32 + (lane & 7) + (mi >> 1) * 8;
      const int b_col = (mi & 1) * 8;
      const uint32_t b_base0 = smem_u32(sm.k + b_tok * kPitch + b_col);
      const uint32_t b_base1 = smem_u32(sm.k + (b_tok + 16) * kPitch + b_col);
#pragma unroll 4
      for (int kk = 0; kk < kQkDim / 16; ++kk) {
        uint32_t a0, a1, a2, a3, b0, b1, b2, b3, b4, b5, b6, b7;
        ldsm_x4(a_base + kk * 32, a0, a1, a2, a3);
        ldsm_x4(b_base0 + kk * 32, b0, b1, b2, b3);
        ldsm_x4(b_base1 + kk * 32, b4, b5, b6, b7);
        mma_bf16(s_acc[0], a0, a1, a2, a3, b0, b1);
        mma_bf16(s_acc[1], a0, a1, a2, a3, b2, b3);
        mma_bf16(s_acc[2], a0, a1, a2, a3, b4, b5);
        mma_bf16(s_acc[3], a0, a1, a2, a3, b6, b7);
      }
    }

    // ---- online softmax (base 2) ----
    float tmax[2] = {-CUDART_INF_F, -CUDART_INF_F};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int t = half * 32 + j * 8 + cq + (e & 1);
        const float x = t < valid ? s_acc[j][e] * c_log2 : -CUDART_INF_F;
        s_acc[j][e] = x;
        tmax[e >> 1] = fmaxf(tmax[e >> 1], x);
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      tmax[r] = fmaxf(tmax[r], __shfl_xor_sync(0xffffffffu, tmax[r], 1));
      tmax[r] = fmaxf(tmax[r], __shfl_xor_sync(0xffffffffu, tmax[r], 2));
    }
    if ((lane & 3) == 0) {
      sm.rmax[half][hg * 16 + r0] = tmax[0];
      sm.rmax[half][hg * 16 + r0 + 8] = tmax[1];
    }
    __syncthreads();
    float alpha[2], m_new[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int h = hg * 16 + r0 + r * 8;
      m_new[r] = fmaxf(m_r[r], fmaxf(sm.rmax[0][h], sm.rmax[1][h]));
      alpha[r] = (m_r[r] == -CUDART_INF_F) ? 0.f : exp2f(m_r[r] - m_new[r]);
      m_r[r] = m_new[r];
    }
    float psum[2] = {0.f, 0.f};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float p0 = exp2f(s_acc[j][0] - m_new[0]);
      const float p1 = exp2f(s_acc[j][1] - m_new[0]);
      const float p2 = exp2f(s_acc[j][2] - m_new[1]);
      const float p3 = exp2f(s_acc[j][3] - m_new[1]);
      psum[0] += p0 + p1;
      psum[1] += p2 + p3;
      const int t = half * 32 + j * 8 + cq;
      *reinterpret_cast<uint32_t*>(sm.p + (hg * 16 + r0) * kPPitch + t) = pack_bf16x2(p0, p1);
      *reinterpret_cast<uint32_t*>(sm.p + (hg * 16 + r0 + 8) * kPPitch + t) = pack_bf16x2(p2, p3);
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      psum[r] += __shfl_xor_sync(0xffffffffu, psum[r], 1);
      psum[r] += __shfl_xor_sync(0xffffffffu, psum[r], 2);
      l_r[r] = l_r[r] * alpha[r] + psum[r];
    }
    __syncthreads();

    // ---- O[16 heads, 256 cols] = alpha * O + P V ----
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      o_acc[j][0] *= alpha[0];
      o_acc[j][1] *= alpha[0];
      o_acc[j][2] *= alpha[1];
      o_acc[j][3] *= alpha[1];
    }
    {
      const int a_row = hg * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
      const int a_col = (lane >> 4) * 8;
      const uint32_t a_base = smem_u32(sm.p + a_row * kPPitch + a_col);
      const int mi = lane >> 3;
      const int v_tok = (lane & 7) + (mi & 1) * 8;
      const int v_col = half * 256 + (mi >> 1) * 8;
      const uint32_t v_base = smem_u32(sm.k + v_tok * kPitch + v_col);
#pragma unroll
      for (int kk = 0; kk < kPageSize / 16; ++kk) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4(a_base + kk * 32, a0, a1, a2, a3);
#pragma unroll
        for (int jn = 0; jn < 16; ++jn) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(v_base + (kk * 16 * kPitch + jn * 16) * 2, b0, b1, b2, b3);
          mma_bf16(o_acc[2 * jn], a0, a1, a2, a3, b0, b1);
          mma_bf16(o_acc[2 * jn + 1], a0, a1, a2, a3, b2, b3);
        }
      }
    }
  }

  // ---- epilogue: combine the two token halves' sums, normalise, store ----
  if ((lane & 3) == 0) {
    sm.rsum[half][hg * 16 + r0] = l_r[0];
    sm.rsum[half][hg * 16 + r0 + 8] = l_r[1];
  }
  __syncthreads();
  float inv_l[2], lse[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int h = hg * 16 + r0 + r * 8;
    const float l = sm.rsum[0][h] + sm.rsum[1][h];
    inv_l[r] = 1.f / l;
    lse[r] = (m_r[r] + __log2f(l)) * kLn2;
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int h = hg * 16 + r0 + r * 8;
    if (h >= heads_here) continue;
    const int hq = head_base + h;
    if (direct) {
      __nv_bfloat16* orow = a.o + b * a.o_stride_b + hq * a.o_stride_h + half * 256 + cq;
#pragma unroll
      for (int j = 0; j < 32; ++j)
        *reinterpret_cast<uint32_t*>(orow + j * 8) =
            pack_bf16x2(o_acc[j][2 * r] * inv_l[r], o_acc[j][2 * r + 1] * inv_l[r]);
    } else {
      const int64_t row = (static_cast<int64_t>(b) * a.num_splits + split) * a.num_heads + hq;
      __nv_bfloat16* prow = a.partial_o + row * kLatent + half * 256 + cq;
#pragma unroll
      for (int j = 0; j < 32; ++j)
        *reinterpret_cast<uint32_t*>(prow + j * 8) =
            pack_bf16x2(o_acc[j][2 * r] * inv_l[r], o_acc[j][2 * r + 1] * inv_l[r]);
      if (half == 0 && (lane & 3) == 0) a.partial_lse[row] = lse[r];
    }
  }
}

}  // namespace

cudaError_t launch_decode_mma(const DecodeArgs& a, cudaStream_t stream) {
  const int smem = static_cast<int>(sizeof(Smem));
  cudaError_t e = cudaFuncSetAttribute(mla_decode_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  const dim3 grid(a.num_splits, a.batch, (a.num_heads + kHB - 1) / kHB);
  mla_decode_mma_kernel<<<grid, kThreads, smem, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace kimi
