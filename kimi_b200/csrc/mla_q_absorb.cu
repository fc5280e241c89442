// The decode step before attention, in one launch: q absorption by W_UK on
// the tensor cores, RoPE of q_pe and k_pe, and the MXFP4 KV append.
//
// Reference (paths inside ianye23301/kimi): `MLAAttention.fused_kv_bmm` and
// the unfused `_q_proj_and_k_up_proj` + `fused_qk_rope_concat_and_cache_mla`
// path it replaces (patches/atom-optimizations.patch:468-639):
//   q_out[t, h, :512] = q_nope[t, h, :] @ W_UK[h]   (k_up_proj BMM, patch:306)
//   q_out[t, h, 512:] = rope(q_pe[t, h, :], positions[t])
//   cache[slot[t]]     = (MXFP4(kv_c[t]), rope(k_pe[t], positions[t]))   (is_nope_first, patch:632)
// RoPE as the engine's rotary embedding applies it: for each of 32 frequency
// pairs (x[i], x[i+32]) (neox style) or (x[2i], x[2i+1]), (a, b) ->
// (a cos - b sin, b cos + a sin) with cos / sin [max_position, 32] float32;
// every product and sum rounded to float32 on its own, the result to bf16.
//
// One CTA of 256 threads per (head h, 128-token tile, column slice z of
// kQSplit = 8): at the Kimi-K2 TP8 shape 64 CTAs, each copying 48 KB, where
// 2 slices per head (96 KB each) measured 10.7 us per call and 8 slices 7.7:
//   * q_nope[tile, h] (A, K-major) and columns 64 z .. 64 z + 63 of W_UK[h]
//     (B, MN-major: rows of output columns as the weight is stored) are
//     copied with cp.async into 128-byte-swizzled shared memory; one thread
//     issues 8 tcgen05.mma kind::f16 (M = 128 tokens, N = 64, K = 16) into
//     64 TMEM columns;
//   * meanwhile the z = 0 CTA rotates q_pe of its tile and head, and the z = 1
//     CTA appends its share of the tile's tokens to the cache (tokens 16 h ..
//     by stride 16 H, 16 threads per token as in the KV-append kernel);
//   * the epilogue reads D (lane = token) and writes its 64 columns of
//     q_out[..., :512] as bf16.
// The single wait is bounded; a give-up leaves q_out's latent part unwritten.
#include <cuda_runtime.h>

#include "kernels.cuh"
#include "mxfp4.cuh"
#include "sm100.cuh"

namespace kimi {
namespace {

using namespace sm100;

constexpr int kTileTokens = 128;
constexpr int kNopeDim = 128;
constexpr int kOffA = 0;                          // 2 K blocks x 128 rows x 128 B
constexpr int kQSplit = 8;                        // CTAs per head, each a slice of the 512 columns
constexpr int kQCols = kLatent / kQSplit;         // output columns per CTA (the MMA's N)
constexpr int kQNBlocks = kQCols / 64;            // 64-column blocks of W per CTA
static_assert(kQCols % 64 == 0 && kQCols <= 256, "N of one MMA, whole 64-column blocks");
constexpr int kOffB = 2 * 128 * 128;              // kQNBlocks N blocks x 128 K rows x 128 B
constexpr int kNBlock = 128 * 128;                // one 64-column block of W (16 KB)
constexpr int kOffMbar = kOffB + kQNBlocks * kNBlock;
constexpr int kOffPos = kOffMbar + 64;            // the tile's 128 positions (int64)
constexpr int kSmemQA = kOffPos + kTileTokens * 8;
constexpr uint32_t kPolls = 100000;               // suspend-hinted polls: about 2 s

__device__ __forceinline__ void rope_pair(float a, float b, float c, float s, float& ra, float& rb) {
  ra = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
  rb = __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s));
}

__device__ __forceinline__ float bf(const __nv_bfloat16* p) { return __bfloat162float(*p); }

// 16-byte asynchronous global -> shared copy (no register round trip, so a
// thread's copies are all in flight at once); src_bytes 0 writes zeros.
__device__ __forceinline__ void cp_async16(void* dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_addr(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}

__device__ __forceinline__ bool position_ok(const QAbsorbArgs& a, int64_t pos) {
  return pos >= 0 && pos < a.max_position;
}

__global__ void __launch_bounds__(256, 2) mla_q_absorb_kernel(const __grid_constant__ QAbsorbArgs a) {
  extern __shared__ __align__(1024) uint8_t sm[];
  uint64_t* mbar = reinterpret_cast<uint64_t*>(sm + kOffMbar);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + kOffMbar + 8);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int h = blockIdx.x, t0 = blockIdx.y * kTileTokens, z = blockIdx.z;
  const int ntok = min(kTileTokens, a.num_tokens - t0);

  if (tid == 0) {
    mbar_init(mbar, 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(tslot, kQCols < 32 ? 32 : kQCols);
  int64_t* pos_s = reinterpret_cast<int64_t*>(sm + kOffPos);
  if (tid < ntok) pos_s[tid] = a.positions[t0 + tid];

  // ---- operands into shared memory ----
  // A: token r, 16-byte chunk c of its 128 q_nope elements (c / 8 = K block)
  for (int i = tid; i < kTileTokens * 16; i += 256) {
    const int r = i >> 4, c = i & 15;
    const int rr = r < ntok ? r : 0;  // rows past the tokens read row 0's address and write zeros
    cp_async16(sm + kOffA + (c >> 3) * (128 * 128) + (r >> 3) * 1024 + sw128_offset(r & 7, c & 7),
               a.q_nope + (t0 + rr) * a.q_nope_stride_t + h * a.q_nope_stride_h + 8 * c, r < ntok ? 16u : 0u);
  }
  // B: K row k, 16-byte chunk c of this CTA's kQCols output columns (c / 8 = N block)
  const __nv_bfloat16* w = a.w_uk + static_cast<int64_t>(h) * kNopeDim * kLatent + kQCols * z;
  constexpr int kChunks = kQCols / 8;  // 16-byte chunks per K row
  for (int i = tid; i < kNopeDim * kChunks; i += 256) {
    const int k = i / kChunks, c = i % kChunks;
    cp_async16(sm + kOffB + (c >> 3) * kNBlock + (k >> 3) * 1024 + sw128_offset(k & 7, c & 7), w + k * kLatent + 8 * c,
               16u);
  }
  asm volatile("cp.async.wait_all;\n" ::: "memory");
  fence_proxy_async_smem();
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = *tslot;

  if (tid == 0) {
    const uint32_t idesc = instr_desc(kFmtBF16, kFmtBF16, false, true, 128, kQCols);
    const uint64_t da = smem_desc(smem_addr(sm + kOffA), 16, 1024, kSwizzle128B);
    const uint64_t db = smem_desc(smem_addr(sm + kOffB), kNBlock, 1024, kSwizzle128B);
#pragma unroll
    for (int k = 0; k < 8; ++k)
      mma_f16_ss(tmem, da + (((k >> 2) * (128 * 128) + (k & 3) * 32) >> 4), db + ((k * 2048) >> 4), idesc,
                 k > 0 ? 1u : 0u);
    mma_commit(mbar);
  }

  // ---- RoPE of q_pe (this head, this tile) while the MMAs run: two threads
  // per token, 16 pairs each, every load of a thread issued before its math ----
  if (z == 0) {
    const int r = tid >> 1, half = tid & 1, t = t0 + r;
    if (r < ntok) {
      const __nv_bfloat16* x = a.q_pe + t * a.q_pe_stride_t + h * a.q_pe_stride_h;
      __nv_bfloat16* out = a.q_out + t * a.q_out_stride_t + h * a.q_out_stride_h + kLatent;
      const int64_t pos = pos_s[r];
      const bool ok = position_ok(a, pos);
      // pairs p = 16 half .. 16 half + 15
      float c[16], sn[16], xa[16], xb[16];
      const float4* cp = reinterpret_cast<const float4*>(a.cos + (ok ? pos : 0) * 32 + 16 * half);
      const float4* sp = reinterpret_cast<const float4*>(a.sin + (ok ? pos : 0) * 32 + 16 * half);
      uint4 raw[4];
      if (a.is_neox) {  // elements 16 half + j and 32 + 16 half + j
        raw[0] = reinterpret_cast<const uint4*>(x + 16 * half)[0];
        raw[1] = reinterpret_cast<const uint4*>(x + 16 * half)[1];
        raw[2] = reinterpret_cast<const uint4*>(x + 32 + 16 * half)[0];
        raw[3] = reinterpret_cast<const uint4*>(x + 32 + 16 * half)[1];
      } else {  // elements 32 half .. 32 half + 31, interleaved pairs
#pragma unroll
        for (int v = 0; v < 4; ++v) raw[v] = reinterpret_cast<const uint4*>(x + 32 * half)[v];
      }
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        const float4 cv = cp[v], sv = sp[v];
        c[4 * v] = cv.x; c[4 * v + 1] = cv.y; c[4 * v + 2] = cv.z; c[4 * v + 3] = cv.w;
        sn[4 * v] = sv.x; sn[4 * v + 1] = sv.y; sn[4 * v + 2] = sv.z; sn[4 * v + 3] = sv.w;
      }
      float e[32];  // the loaded elements in order
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        const uint32_t wv[4] = {raw[v].x, raw[v].y, raw[v].z, raw[v].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          e[8 * v + 2 * j] = __uint_as_float(wv[j] << 16);
          e[8 * v + 2 * j + 1] = __uint_as_float(wv[j] & 0xFFFF0000u);
        }
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        xa[j] = a.is_neox ? e[j] : e[2 * j];
        xb[j] = a.is_neox ? e[16 + j] : e[2 * j + 1];
      }
      float ra[16], rb[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        rope_pair(xa[j], xb[j], c[j], sn[j], ra[j], rb[j]);
        if (!ok) ra[j] = rb[j] = 0.f;
      }
      uint32_t o[16];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        // neox: words 0..7 hold ra (elements 16 half ..), the other half rb;
        // interleaved: word j holds the pair (ra[j], rb[j])... two pairs per 4 bytes
        __nv_bfloat162 p0, p1;
        if (a.is_neox) {
          p0 = __floats2bfloat162_rn(ra[2 * j], ra[2 * j + 1]);
          p1 = __floats2bfloat162_rn(rb[2 * j], rb[2 * j + 1]);
        } else {
          p0 = __floats2bfloat162_rn(ra[j], rb[j]);
          p1 = __floats2bfloat162_rn(ra[8 + j], rb[8 + j]);
        }
        o[j] = *reinterpret_cast<const uint32_t*>(&p0);
        o[8 + j] = *reinterpret_cast<const uint32_t*>(&p1);
      }
      if (a.is_neox) {
        uint4* d0 = reinterpret_cast<uint4*>(out + 16 * half);
        uint4* d1 = reinterpret_cast<uint4*>(out + 32 + 16 * half);
        d0[0] = make_uint4(o[0], o[1], o[2], o[3]);
        d0[1] = make_uint4(o[4], o[5], o[6], o[7]);
        d1[0] = make_uint4(o[8], o[9], o[10], o[11]);
        d1[1] = make_uint4(o[12], o[13], o[14], o[15]);
      } else {
        uint4* d = reinterpret_cast<uint4*>(out + 32 * half);
        d[0] = make_uint4(o[0], o[1], o[2], o[3]);
        d[1] = make_uint4(o[4], o[5], o[6], o[7]);
        d[2] = make_uint4(o[8], o[9], o[10], o[11]);
        d[3] = make_uint4(o[12], o[13], o[14], o[15]);
      }
    }
  }

  // ---- KV append: this CTA's share of the tile's tokens ----
  for (int r = 16 * h + (tid >> 4); z == 1 && r < ntok; r += 16 * a.num_heads) {
    const int t = t0 + r, grp = tid & 15;
    const int64_t slot = a.slot_mapping[t];
    const int64_t pos = pos_s[r];
    if (slot < 0 || slot >= a.num_pages * kPageSize || !position_ok(a, pos)) continue;
    float x[32];
    const uint4* src = reinterpret_cast<const uint4*>(a.kv_c + t * a.kv_c_stride + 32 * grp);
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      const uint4 wv = src[v];
      const uint32_t ws[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        x[8 * v + 2 * j] = __uint_as_float(ws[j] << 16);
        x[8 * v + 2 * j + 1] = __uint_as_float(ws[j] & 0xFFFF0000u);
      }
    }
    uint32_t packed[4];
    uint8_t sb;
    if (a.legacy_rule)
      quantize_group32<true>(x, packed, sb);
    else
      quantize_group32<false>(x, packed, sb);
    uint8_t* row = a.kv_buffer + slot * kTokenBytes;
    *reinterpret_cast<uint4*>(row + 16 * grp) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    a.kv_scales[slot * kScaleBytes + grp] = sb;
    if (grp < 8) {
      // RoPE part: elements 8 grp .. 8 grp + 7 (their neox partners sit 32 away)
      const __nv_bfloat16* kp = a.k_pe + t * a.k_pe_stride;
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 8; j += 2) {
        float r0, r1;
        const int e0 = 8 * grp + j, e1 = e0 + 1;
        if (a.is_neox) {
          // e0, e1 are both in the first half or both in the second
          float q0, q1;
          if (e0 < 32) {
            rope_pair(bf(kp + e0), bf(kp + e0 + 32), a.cos[pos * 32 + e0], a.sin[pos * 32 + e0], r0, q0);
            rope_pair(bf(kp + e1), bf(kp + e1 + 32), a.cos[pos * 32 + e1], a.sin[pos * 32 + e1], r1, q1);
          } else {
            rope_pair(bf(kp + e0 - 32), bf(kp + e0), a.cos[pos * 32 + e0 - 32], a.sin[pos * 32 + e0 - 32], q0, r0);
            rope_pair(bf(kp + e1 - 32), bf(kp + e1), a.cos[pos * 32 + e1 - 32], a.sin[pos * 32 + e1 - 32], q1, r1);
          }
        } else {
          rope_pair(bf(kp + e0), bf(kp + e1), a.cos[pos * 32 + e0 / 2], a.sin[pos * 32 + e0 / 2], r0, r1);
        }
        const __nv_bfloat162 pr = __floats2bfloat162_rn(r0, r1);
        o[j / 2] = *reinterpret_cast<const uint32_t*>(&pr);
      }
      *reinterpret_cast<uint4*>(row + kNibbleBytes + 16 * grp) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }

  // ---- epilogue: D (lane = token, column = latent) -> q_out[..., :512] ----
  bool done = false;
  for (uint32_t i = 0; i < kPolls && !done; ++i) done = mbar_try_wait_sleep(mbar, 0, kWaitSleepNs);
  done = __all_sync(0xffffffffu, done);  // warp-uniform: the TMEM load below is warp-wide
  if (!done && lane == 0 && a.status) atomicOr(a.status, kStatusQAbsorbWait);
  fence_after_sync();
  const int q = warp & 3, half = warp >> 2, r = 32 * q + lane;
  if (done) {
#pragma unroll 1
    for (int cb = 0; cb < kQCols / 64; ++cb) {
      uint32_t v[32];
      const int tcol = (kQCols / 2) * half + 32 * cb, col = kQCols * z + tcol;
      tmem_ld32(tmem + (static_cast<uint32_t>(32 * q) << 16) + tcol, v);
      tmem_ld_wait();
      if (r < ntok) {
        uint4* dst = reinterpret_cast<uint4*>(a.q_out + (t0 + r) * a.q_out_stride_t + h * a.q_out_stride_h + col);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint32_t p[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const __nv_bfloat162 pr =
                __floats2bfloat162_rn(__uint_as_float(v[8 * j + 2 * e]), __uint_as_float(v[8 * j + 2 * e + 1]));
            p[e] = *reinterpret_cast<const uint32_t*>(&pr);
          }
          dst[j] = make_uint4(p[0], p[1], p[2], p[3]);
        }
      }
    }
  }
  fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    fence_after_sync();
    tmem_dealloc(tmem, kQCols < 32 ? 32 : kQCols);
  }
}

}  // namespace

cudaError_t launch_q_absorb(const QAbsorbArgs& a, cudaStream_t stream) {
  cudaError_t e = cudaFuncSetAttribute(mla_q_absorb_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemQA);
  if (e != cudaSuccess) return e;
  const dim3 grid(a.num_heads, (a.num_tokens + kTileTokens - 1) / kTileTokens, kQSplit);
  mla_q_absorb_kernel<<<grid, 256, kSmemQA, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace kimi
