// Split-K absorbed-MLA decode over the MXFP4 paged cache on the 5th-generation
// tensor cores (tcgen05 + TMEM), sm_100a.
//
// Math (paths inside ianye23301/kimi): the archive stage-1 kernel
// `_mla_decode_split_kv` (archive/mla-mxfp4-dead-end/mla_decode_mxfp4_v5.py:136-261)
// with the contract of `reference_mla_decode` (tests/test_triton_mla_decode.py:12-62):
//   S = q_nope . k_nope + q_pe . k_pe,  P = softmax(S * sm_scale),  O = P . k_nope.
//
// Layout of one CTA (a sequence, a range of its pages, up to 64 heads):
//   * The cache is consumed in tiles of 128 tokens (two pages).  Tokens sit on
//     the MMA's M dimension (M = 128) and heads on N ("swap AB"), so 64 heads
//     fill a full-rate tcgen05 MMA.
//   * Each latent element is dequantised ONCE per tile into an 8-bit tile V''
//     in shared memory: e2m1 -> f16 (cvt.rn.f16x2.e2m1x2), times the e8m0
//     scale relative to a per-split reference 2^sigma (one f16x2 multiply),
//     then the high byte of the f16, which is the e5m2 encoding of the same
//     value.  e2m1 * 2^k has one mantissa bit, so this is exact over e5m2's
//     29-binade range.  V'' is stored in no-swizzle core matrices
//     (8 tokens x 16 latent bytes) and read by the tensor core twice: K-major
//     as the A operand of S^T = V'' . Q''^T, and MN-major as the A operand of
//     O^T = V''^T . P''^T.
//   * q_nope is split into two e4m3 terms with a per-head power-of-two scale
//     a_h (q/a_h = hi + lo), stacked as one N = 128 B operand, which keeps
//     bf16-level accuracy for QK^T at fp8 tensor rate.  q_pe . k_pe runs as a
//     bf16 MMA into its own accumulator.
//   * P'' = exp2(x - R_h) as two e4m3 terms (hi + residual lo, two PV MMAs
//     into the same accumulator; one e4m3 term alone costs ~2% relative error
//     on short contexts), with R_h a per-head offset kept within
//     [max - 8.5, max - 6] of the running max (raised lazily, rescaling O and
//     the softmax sums when a score exceeds it).  The O accumulator therefore
//     holds sum_t exp2(x - R_h) V 2^-sigma; the epilogue multiplies by 2^sigma
//     and divides by l_h = sum_t exp2(x - R_h).
//   * TMEM (512 columns): S_hi|S_lo [0,128), S_pe [128,192), O^T [256,512)
//     as four 128-row latent chunks of 64 head columns.
//
// Threads: warps 0-7 dequantise and run the softmax; warp 8 owns TMEM and
// issues the MMAs.  Every mbarrier wait is bounded; on timeout the CTA sets
// an error bit in the status word and all threads leave at the same barrier.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math_constants.h>

#include "kernels.cuh"
#include "sm100.cuh"

namespace kimi {
namespace {

using namespace sm100;

constexpr int kNH = 64;             // heads per CTA (N of the MMAs)
constexpr int kCompute = 256;       // dequant + softmax threads
constexpr int kThreadsTC = kCompute + 32;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0, kColSpe = 128, kColO = 256;
constexpr uint32_t kPollLimit = 4u << 20;

// Shared memory (bytes).  Core matrix (r, c) of an operand lives at
// r * row_stride + c * 128, 16 bytes per row inside the core.
constexpr int kOffV = 0;            // V'' e5m2, cores (token group 0..15, latent byte group 0..31): 64 KB
constexpr int kVRow = 32 * 128;     // 4096 B per 8-token group
constexpr int kOffQ = 65536;        // Q'' e4m3 hi rows 0..63, lo rows 64..127: 64 KB
constexpr int kQRow = 32 * 128;
constexpr int kOffQpe = 131072;     // q_pe bf16, cores (head group 0..7, byte group 0..7): 8 KB
constexpr int kOffKpe = 139264;     // k_pe bf16, cores (token group 0..15, byte group 0..7): 16 KB
constexpr int kPeRow = 8 * 128;
constexpr int kOffP = 155648;       // P'' hi e4m3, MN-major cores (token group 0..15, head byte group 0..3): 8 KB
constexpr int kOffPlo = 163840;     // P'' lo (residual), same layout: 8 KB
constexpr int kPRow = 4 * 128;
constexpr int kOffMisc = 172032;

struct Misc {
  uint64_t bar_s;
  uint64_t bar_o;
  uint32_t tmem_base;
  int abort_flag;
  int rescale_flag;
  int sigma;              // latent reference exponent: V'' = V * 2^-sigma
  int tile_smax[2];       // max e8m0 byte of the current tile (double-buffered reset)
  float a[kNH];           // per-head q_nope scale (power of two)
  float coef[kNH];        // 2^sigma * a_h * sm_scale * log2(e)
  float R[kNH];           // per-head exp2 offset (log2 units)
  float alpha[kNH];       // rescale factors of a rescale event
  float red[4][kNH];      // cross-warp reduction scratch
};
constexpr int kSmemTC = kOffMisc + static_cast<int>(sizeof(Misc));

__device__ __forceinline__ uint8_t* smem_base() {
  extern __shared__ __align__(1024) uint8_t dyn_smem[];
  return dyn_smem;
}

__device__ __forceinline__ void named_bar(int id, int count) {
  asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(count) : "memory");
}

__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// Four e2m1 pairs (one u32 of packed nibbles) -> four f16x2 (exact).
__device__ __forceinline__ void cvt4_e2m1(uint32_t w, uint32_t (&o)[4]) {
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}\n"
      : "=r"(o[0]), "=r"(o[1]), "=r"(o[2]), "=r"(o[3])
      : "r"(w));
}

__device__ __forceinline__ uint32_t hmul2_u32(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;\n" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// f16 2^k (k in [-24, 15]) replicated in both halves; 0 below.
__device__ __forceinline__ uint32_t f16x2_pow2(int k) {
  uint32_t h;
  if (k >= -14)
    h = static_cast<uint32_t>(k + 15) << 10;
  else if (k >= -24)
    h = 1u << (k + 24);
  else
    h = 0u;
  return h | (h << 16);
}

// Sixteen packed nibble bytes (32 elements of one e8m0 group) times the f16
// multiplier -> 32 e5m2 bytes (two 16-byte rows of V'').
__device__ __forceinline__ void group_to_e5m2(const uint4& nib, uint32_t mult, uint4& out0, uint4& out1) {
  const uint32_t w[4] = {nib.x, nib.y, nib.z, nib.w};
  uint32_t r[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t f[4];
    cvt4_e2m1(w[i], f);
#pragma unroll
    for (int j = 0; j < 4; ++j) f[j] = hmul2_u32(f[j], mult);
    r[2 * i] = __byte_perm(f[0], f[1], 0x7531);
    r[2 * i + 1] = __byte_perm(f[2], f[3], 0x7531);
  }
  out0 = make_uint4(r[0], r[1], r[2], r[3]);
  out1 = make_uint4(r[4], r[5], r[6], r[7]);
}

// Raw data of one tile held by one thread: for its token, 16-byte chunk
// j = 2k + e of the nibbles (k = 0..7) and of the RoPE bytes (k = 0..3),
// plus the token's 16 scale bytes.
struct TileRegs {
  uint4 nib[8];
  uint4 pe[4];
  uint4 sc;
  int valid;
};

struct WorkItem {
  int b, split, head_base, heads_here;
  int page_lo, n_pages, n_tok, p_begin, p_end;
};

__device__ __forceinline__ int tile_page(const DecodeArgs& a, const WorkItem& w, int tile, int slot) {
  const int p = w.p_begin + 2 * tile + slot;
  if (p >= w.p_end) return -1;
  const int page = a.kv_indices[w.page_lo + p];
  return (page >= 0 && page < a.num_pages) ? page : -1;
}

__device__ __forceinline__ void load_tile(const DecodeArgs& a, const WorkItem& w, int tile, int t, int e,
                                          TileRegs& r) {
  const int page = tile_page(a, w, tile, t >> 6);
  const int seq_tok = (w.p_begin + 2 * tile) * kPageSize + t;
  r.valid = page >= 0 && seq_tok < w.n_tok;
  if (r.valid) {
    const uint8_t* row = a.kv_buffer + static_cast<int64_t>(page) * kPageBytes + (t & 63) * kTokenBytes;
#pragma unroll
    for (int k = 0; k < 8; ++k) r.nib[k] = ldg_stream(row + 16 * (2 * k + e));
#pragma unroll
    for (int k = 0; k < 4; ++k) r.pe[k] = ldg_stream(row + kNibbleBytes + 16 * (2 * k + e));
    r.sc = ldg_stream(a.kv_scales + static_cast<int64_t>(page) * kPageScaleBytes + (t & 63) * kScaleBytes);
  }
}

__device__ __forceinline__ uint32_t max_byte(const uint4& v) {
  uint32_t m = __vmaxu4(__vmaxu4(v.x, v.y), __vmaxu4(v.z, v.w));
  m = __vmaxu4(m, m >> 16);
  m = __vmaxu4(m, m >> 8);
  return m & 0xFFu;
}

__device__ __forceinline__ uint32_t scale_byte(const uint4& v, int g) {
  const uint32_t w = g < 4 ? v.x : (g < 8 ? v.y : (g < 12 ? v.z : v.w));
  return (w >> (8 * (g & 3))) & 0xFFu;
}

// Transpose-reduce (max or sum) of 32 per-lane values over the warp: lane j
// ends with the reduction of element j across all 32 lanes.
template <bool kMax>
__device__ __forceinline__ float warp_transpose_reduce(float (&v)[32], int lane) {
#pragma unroll
  for (int width = 16; width >= 1; width >>= 1) {
    const bool upper = (lane & width) != 0;
#pragma unroll
    for (int j = 0; j < width; ++j) {
      const float send = upper ? v[j] : v[j + width];
      const float keep = upper ? v[j + width] : v[j];
      const float got = __shfl_xor_sync(0xffffffffu, send, width);
      v[j] = kMax ? fmaxf(keep, got) : keep + got;
    }
  }
  return v[0];
}

__device__ __forceinline__ void record_status(const DecodeArgs& a, int bits) {
  if (a.status) atomicOr(a.status, bits);
}

__global__ void __launch_bounds__(kThreadsTC, 1) mla_decode_tc_kernel(DecodeArgs a) {
  uint8_t* sm = smem_base();
  Misc& ms = *reinterpret_cast<Misc*>(sm + kOffMisc);
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  WorkItem w;
  w.split = blockIdx.x;
  w.b = blockIdx.y;
  w.head_base = blockIdx.z * kNH;
  w.heads_here = min(kNH, a.num_heads - w.head_base);
  w.page_lo = a.kv_indptr[w.b];
  w.n_pages = a.kv_indptr[w.b + 1] - w.page_lo;
  const int last_len =
      w.n_pages <= 0 ? 0 : min(max(a.kv_last_page_len ? a.kv_last_page_len[w.b] : kPageSize, 1), kPageSize);
  w.n_tok = w.n_pages <= 0 ? 0 : (w.n_pages - 1) * kPageSize + last_len;
  const int pps = 2 * ((max(w.n_pages, 0) + 2 * a.num_splits - 1) / (2 * a.num_splits));
  w.p_begin = w.split * pps;
  w.p_end = min(w.p_begin + pps, max(w.n_pages, 0));
  const bool direct = a.num_splits == 1;

  if (w.p_begin >= w.p_end) {
    if (direct) {
      for (int i = tid; i < w.heads_here * (kLatent / 2); i += kThreadsTC) {
        const int h = i / (kLatent / 2), d = (i % (kLatent / 2)) * 2;
        *reinterpret_cast<uint32_t*>(a.o + w.b * a.o_stride_b + (w.head_base + h) * a.o_stride_h + d) = 0u;
      }
    } else if (tid < w.heads_here) {
      a.partial_lse[(static_cast<int64_t>(w.b) * a.num_splits + w.split) * a.num_heads + w.head_base + tid] =
          -CUDART_INF_F;
    }
    return;
  }
  const int n_tiles = (w.p_end - w.p_begin + 1) / 2;
  const float c_log2 = a.sm_scale * kLog2e;

  // ---------------- setup: TMEM, barriers, Q operands ----------------
  if (warp == 8) {
    tmem_alloc(&ms.tmem_base, kTmemCols);
    if (lane == 0) {
      mbar_init(&ms.bar_s, 1);
      mbar_init(&ms.bar_o, 1);
      fence_mbar_init();
      ms.abort_flag = 0;
      ms.rescale_flag = 0;
      ms.tile_smax[0] = 0;
      ms.tile_smax[1] = 0;
    }
  } else {
    // 4 threads per head: part p handles latent [128p, 128p + 128) and RoPE [16p, 16p + 16).
    const int h = tid >> 2, part = tid & 3;
    const bool live = h < w.heads_here;
    const __nv_bfloat16* qrow = a.q + w.b * a.q_stride_b + (w.head_base + h) * a.q_stride_h;
    float amax = 0.f;
    uint4 qv[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      qv[k] = live ? *reinterpret_cast<const uint4*>(qrow + 128 * part + 8 * k) : make_uint4(0, 0, 0, 0);
      const uint32_t ws[4] = {qv[k].x, qv[k].y, qv[k].z, qv[k].w};
#pragma unroll
      for (int j = 0; j < 4; ++j)
        amax = fmaxf(amax, fmaxf(fabsf(__uint_as_float(ws[j] << 16)), fabsf(__uint_as_float(ws[j] & 0xFFFF0000u))));
    }
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    // a_h = 2^(floor(log2 amax) - 7): |q / a_h| < 256 < 448 (e4m3 max)
    int ex = static_cast<int>((__float_as_uint(amax) >> 23) & 0xFF) - 127 - 7;
    if (amax == 0.f || ex < -126) ex = 0;
    const float a_h = __uint_as_float(static_cast<uint32_t>(ex + 127) << 23);
    const float inv_a = __uint_as_float(static_cast<uint32_t>(127 - ex) << 23);
    if (part == 0) ms.a[h] = a_h;
    uint8_t* qb = sm + kOffQ;
#pragma unroll
    for (int k = 0; k < 16; k += 2) {
      // 16 latent elements = one 16-byte core row of hi and of lo
      uint32_t hi_w[4], lo_w[4];
      const uint32_t ws[8] = {qv[k].x, qv[k].y, qv[k].z, qv[k].w, qv[k + 1].x, qv[k + 1].y, qv[k + 1].z, qv[k + 1].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float x[4];
        x[0] = __uint_as_float(ws[2 * j] << 16) * inv_a;
        x[1] = __uint_as_float(ws[2 * j] & 0xFFFF0000u) * inv_a;
        x[2] = __uint_as_float(ws[2 * j + 1] << 16) * inv_a;
        x[3] = __uint_as_float(ws[2 * j + 1] & 0xFFFF0000u) * inv_a;
        const uint16_t h01 = cvt_f32x2_e4m3x2(x[0], x[1]);
        const uint16_t h23 = cvt_f32x2_e4m3x2(x[2], x[3]);
        // residuals against the e4m3 values (e4m3 -> float is exact)
        const float2 g01 = e4m3x2_to_float2(h01);
        const float2 g23 = e4m3x2_to_float2(h23);
        const uint16_t l01 = cvt_f32x2_e4m3x2(x[0] - g01.x, x[1] - g01.y);
        const uint16_t l23 = cvt_f32x2_e4m3x2(x[2] - g23.x, x[3] - g23.y);
        hi_w[j] = static_cast<uint32_t>(h01) | (static_cast<uint32_t>(h23) << 16);
        lo_w[j] = static_cast<uint32_t>(l01) | (static_cast<uint32_t>(l23) << 16);
      }
      const int dc = 8 * part + k / 2;  // 16-byte latent group of this row (0..31)
      *reinterpret_cast<uint4*>(qb + (h >> 3) * kQRow + dc * 128 + (h & 7) * 16) =
          make_uint4(hi_w[0], hi_w[1], hi_w[2], hi_w[3]);
      *reinterpret_cast<uint4*>(qb + (8 + (h >> 3)) * kQRow + dc * 128 + (h & 7) * 16) =
          make_uint4(lo_w[0], lo_w[1], lo_w[2], lo_w[3]);
    }
    // q_pe: 16 bf16 = two 16-byte core rows
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const uint4 v = live ? *reinterpret_cast<const uint4*>(qrow + kLatent + 16 * part + 8 * k) : make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(sm + kOffQpe + (h >> 3) * kPeRow + (2 * part + k) * 128 + (h & 7) * 16) = v;
    }
  }
  fence_proxy_async_smem();
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = ms.tmem_base;

  if (warp == 8) {
    // ---------------- MMA issuer ----------------
    const uint32_t id_qk = instr_desc(kFmtE5M2, kFmtE4M3, false, false, 128, 128);
    const uint32_t id_pe = instr_desc(kFmtBF16, kFmtBF16, false, false, 128, 64);
    const uint32_t id_pv = instr_desc(kFmtE5M2, kFmtE4M3, true, true, 128, 64);
    const uint32_t sV = smem_addr(sm + kOffV), sQ = smem_addr(sm + kOffQ);
    const uint32_t sQpe = smem_addr(sm + kOffQpe), sKpe = smem_addr(sm + kOffKpe), sP = smem_addr(sm + kOffP);
    const uint32_t sPlo = smem_addr(sm + kOffPlo);
    for (int tile = 0; tile < n_tiles; ++tile) {
      named_bar(1, kThreadsTC);  // tile ready
      if (ms.abort_flag) break;
      fence_after_sync();
      if (lane == 0) {
#pragma unroll 1
        for (int k = 0; k < 16; ++k)
          mma_f8f6f4_ss(tmem + kColS, smem_desc(sV + k * 256, 128, kVRow), smem_desc(sQ + k * 256, 128, kQRow), id_qk,
                        k > 0);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_f16_ss(tmem + kColSpe, smem_desc(sKpe + k * 256, 128, kPeRow), smem_desc(sQpe + k * 256, 128, kPeRow),
                     id_pe, k > 0);
        mma_commit(&ms.bar_s);
      }
      __syncwarp();
      named_bar(2, kThreadsTC);  // P ready
      if (ms.abort_flag) break;
      fence_after_sync();
      if (lane == 0) {
#pragma unroll 1
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t va = smem_desc(sV + k * 4 * kVRow + c * 8 * 128, kVRow, 128);
            mma_f8f6f4_ss(tmem + kColO + 64 * c, va, smem_desc(sP + k * 4 * kPRow, kPRow, 128), id_pv,
                          (tile > 0 || k > 0) ? 1u : 0u);
            mma_f8f6f4_ss(tmem + kColO + 64 * c, va, smem_desc(sPlo + k * 4 * kPRow, kPRow, 128), id_pv, 1u);
          }
        mma_commit(&ms.bar_o);
      }
      __syncwarp();
    }
    named_bar(3, kThreadsTC);  // epilogue done
    fence_after_sync();
    tmem_dealloc(tmem, kTmemCols);
    return;
  }

  // ---------------- compute warps: dequant + softmax ----------------
  // Loader mapping: warp covers tokens 16*warp..+16; lanes l and l+16 share a token.
  const int lt = 16 * warp + (lane & 15);
  const int le = lane >> 4;
  // TMEM mapping: quadrant q = warp & 3 owns lanes / tokens 32q..32q+31; hf picks heads 32hf..+32.
  const int q = warp & 3;
  const int hf = warp >> 2;
  const int st = 32 * q + lane;  // token of this thread in the softmax
  const uint32_t lane_base = static_cast<uint32_t>(32 * q) << 16;

  float l_part[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) l_part[j] = 0.f;

  TileRegs r;
  load_tile(a, w, 0, lt, le, r);
  bool aborted = false;

  for (int tile = 0; tile < n_tiles; ++tile) {
    const uint32_t par = static_cast<uint32_t>(tile & 1);
    // Previous PV must be done before V'', k_pe and P'' are overwritten and before O is rescaled.
    if (tile > 0 && !mbar_wait_bounded(&ms.bar_o, par ^ 1u, kPollLimit)) {
      atomicExch(&ms.abort_flag, 1);
      record_status(a, 1);
    }
    fence_after_sync();

    // ---- tile max of the e8m0 bytes (valid tokens) ----
    uint32_t my_max = r.valid ? max_byte(r.sc) : 0u;
    my_max = __reduce_max_sync(0xffffffffu, my_max);
    if (lane == 0) atomicMax(&ms.tile_smax[par], static_cast<int>(my_max));
    named_bar(4, kCompute);
    const int tmax = ms.tile_smax[par];
    if (tid == 0) ms.tile_smax[par ^ 1] = 0;
    if (tile == 0 || tmax > ms.sigma + 127 + 13) {
      const int new_sigma = tmax - 127 - 8;  // tile max maps to <= 6 * 2^8 in V''
      if (tile > 0) {
        // raise sigma: O *= 2^(old - new) for every head (TMEM read-modify-write)
        const float f = exp2f(static_cast<float>(ms.sigma - new_sigma));
#pragma unroll 1
        for (int cc = 0; cc < 2; ++cc) {
          const int c = 2 * hf + cc;
#pragma unroll 1
          for (int half = 0; half < 2; ++half) {
            uint32_t v[32];
            const uint32_t ta = tmem + lane_base + kColO + 64 * c + 32 * half;
            tmem_ld32(ta, v);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __float_as_uint(__uint_as_float(v[j]) * f);
            tmem_st32(ta, v);
          }
        }
        tmem_st_wait();
      }
      named_bar(4, kCompute);
      if (tid < kNH) ms.coef[tid] = exp2f(static_cast<float>(new_sigma)) * ms.a[tid] * c_log2;
      if (tid == 0) ms.sigma = new_sigma;
      named_bar(4, kCompute);
    }
    const int sigma = ms.sigma;

    // ---- dequant this thread's token into V'' and k_pe ----
    {
      uint8_t* vrow = sm + kOffV + (lt >> 3) * kVRow + (lt & 7) * 16;
      uint8_t* prow = sm + kOffKpe + (lt >> 3) * kPeRow + (lt & 7) * 16;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int g = 2 * k + le;  // e8m0 group == 16-byte nibble chunk
        uint4 o0 = make_uint4(0, 0, 0, 0), o1 = o0;
        if (r.valid) {
          const int kexp = static_cast<int>(scale_byte(r.sc, g)) - 127 - sigma;
          group_to_e5m2(r.nib[k], f16x2_pow2(kexp), o0, o1);
        }
        *reinterpret_cast<uint4*>(vrow + (2 * g) * 128) = o0;
        *reinterpret_cast<uint4*>(vrow + (2 * g + 1) * 128) = o1;
      }
#pragma unroll
      for (int k = 0; k < 4; ++k)
        *reinterpret_cast<uint4*>(prow + (2 * k + le) * 128) = r.valid ? r.pe[k] : make_uint4(0, 0, 0, 0);
    }
    if (tile + 1 < n_tiles) load_tile(a, w, tile + 1, lt, le, r);
    fence_proxy_async_smem();
    fence_before_sync();
    named_bar(1, kThreadsTC);  // tile ready
    if (ms.abort_flag) {
      aborted = true;
      break;
    }

    // ---- softmax on S^T rows (this thread: token st, heads 32hf..32hf+31) ----
    if (!mbar_wait_bounded(&ms.bar_s, par, kPollLimit)) {
      atomicExch(&ms.abort_flag, 1);
      record_status(a, 2);
    }
    fence_after_sync();
    float x[32];
    {
      uint32_t s_hi[32], s_lo[32], s_pe[32];
      tmem_ld32(tmem + lane_base + kColS + 32 * hf, s_hi);
      tmem_ld32(tmem + lane_base + kColS + 64 + 32 * hf, s_lo);
      tmem_ld32(tmem + lane_base + kColSpe + 32 * hf, s_pe);
      tmem_ld_wait();
      const int seq_tok = (w.p_begin + 2 * tile) * kPageSize + st;
      const bool tvalid = tile_page(a, w, tile, st >> 6) >= 0 && seq_tok < w.n_tok;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float s = __uint_as_float(s_hi[j]) + __uint_as_float(s_lo[j]);
        x[j] = tvalid ? fmaf(s, ms.coef[32 * hf + j], __uint_as_float(s_pe[j]) * c_log2) : -CUDART_INF_F;
      }
    }
    fence_before_sync();

    // offsets: first tile sets R = max - 6; later tiles raise R when a score exceeds R + 8.5
    bool need = tile == 0;
    if (!need) {
      float ymax = -CUDART_INF_F;
#pragma unroll
      for (int j = 0; j < 32; ++j) ymax = fmaxf(ymax, x[j] - ms.R[32 * hf + j]);
      if (__any_sync(0xffffffffu, ymax > 8.5f) && lane == 0) ms.rescale_flag = 1;
      named_bar(4, kCompute);
      need = ms.rescale_flag != 0;
      named_bar(4, kCompute);
      if (tid == 0) ms.rescale_flag = 0;
    }
    if (need) {
      float v[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = x[j];
      const float m = warp_transpose_reduce<true>(v, lane);  // head 32hf + lane, over this warp's tokens
      ms.red[q][32 * hf + lane] = m;
      named_bar(4, kCompute);
      if (tid < kNH) {
        const float tmx = fmaxf(fmaxf(ms.red[0][tid], ms.red[1][tid]), fmaxf(ms.red[2][tid], ms.red[3][tid]));
        const float r_old = tile == 0 ? -CUDART_INF_F : ms.R[tid];
        const float r_new = fmaxf(fmaxf(r_old, tmx - 6.0f), -1e30f);
        ms.alpha[tid] = tile == 0 ? 1.0f : exp2f(r_old - r_new);
        ms.R[tid] = r_new;
      }
      named_bar(4, kCompute);
      if (tile > 0) {
        // rescale the running sums and O^T columns of every head
#pragma unroll
        for (int j = 0; j < 32; ++j) l_part[j] *= ms.alpha[32 * hf + j];
        fence_after_sync();
#pragma unroll 1
        for (int cc = 0; cc < 2; ++cc) {
          const int c = 2 * hf + cc;
#pragma unroll 1
          for (int hh = 0; hh < 2; ++hh) {
            uint32_t vv[32];
            const uint32_t ta = tmem + lane_base + kColO + 64 * c + 32 * hh;
            tmem_ld32(ta, vv);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 32; ++j)
              vv[j] = __float_as_uint(__uint_as_float(vv[j]) * ms.alpha[32 * hh + j]);
            tmem_st32(ta, vv);
          }
        }
        tmem_st_wait();
        fence_before_sync();
      }
    }

    // ---- P'' = exp2(x - R) as e4m3 hi + e4m3 residual, into the MN-major B operands ----
    {
      uint32_t pw[8], pl[8];
#pragma unroll
      for (int j = 0; j < 32; j += 2) {
        const float p0 = exp2f(x[j] - ms.R[32 * hf + j]);
        const float p1 = exp2f(x[j + 1] - ms.R[32 * hf + j + 1]);
        l_part[j] += p0;
        l_part[j + 1] += p1;
        const uint16_t h01 = cvt_f32x2_e4m3x2(p0, p1);
        const float2 hf01 = e4m3x2_to_float2(h01);
        const uint16_t l01 = cvt_f32x2_e4m3x2(p0 - hf01.x, p1 - hf01.y);
        if ((j & 2) == 0) {
          pw[j / 4] = h01;
          pl[j / 4] = l01;
        } else {
          pw[j / 4] |= static_cast<uint32_t>(h01) << 16;
          pl[j / 4] |= static_cast<uint32_t>(l01) << 16;
        }
      }
      const int prow = (st >> 3) * kPRow + (st & 7) * 16;
      *reinterpret_cast<uint4*>(sm + kOffP + prow + (2 * hf) * 128) = make_uint4(pw[0], pw[1], pw[2], pw[3]);
      *reinterpret_cast<uint4*>(sm + kOffP + prow + (2 * hf + 1) * 128) = make_uint4(pw[4], pw[5], pw[6], pw[7]);
      *reinterpret_cast<uint4*>(sm + kOffPlo + prow + (2 * hf) * 128) = make_uint4(pl[0], pl[1], pl[2], pl[3]);
      *reinterpret_cast<uint4*>(sm + kOffPlo + prow + (2 * hf + 1) * 128) = make_uint4(pl[4], pl[5], pl[6], pl[7]);
    }
    fence_proxy_async_smem();
    fence_before_sync();
    named_bar(2, kThreadsTC);  // P ready
    if (ms.abort_flag) {
      aborted = true;
      break;
    }
  }

  // ---------------- epilogue ----------------
  if (!aborted && !mbar_wait_bounded(&ms.bar_o, static_cast<uint32_t>((n_tiles - 1) & 1), kPollLimit)) {
    atomicExch(&ms.abort_flag, 1);
    record_status(a, 4);
  }
  fence_after_sync();
  // l_h: sum of this warp's tokens, then over the four quadrants
  {
    const float s = warp_transpose_reduce<false>(l_part, lane);
    ms.red[q][32 * hf + lane] = s;
  }
  named_bar(4, kCompute);
  const bool ok = !ms.abort_flag;
  if (ok) {
    const float sig = exp2f(static_cast<float>(ms.sigma));
    // thread reads O^T lanes 32q.. of chunks 2hf, 2hf+1: latent d = 128c + 32q + lane
#pragma unroll 1
    for (int cc = 0; cc < 2; ++cc) {
      const int c = 2 * hf + cc;
      const int d = 128 * c + 32 * q + lane;
#pragma unroll 1
      for (int hh = 0; hh < 2; ++hh) {
        uint32_t vv[32];
        tmem_ld32(tmem + lane_base + kColO + 64 * c + 32 * hh, vv);
        tmem_ld_wait();
#pragma unroll 4
        for (int j = 0; j < 32; ++j) {
          const int h = 32 * hh + j;
          if (h >= w.heads_here) continue;
          const float l = ms.red[0][h] + ms.red[1][h] + ms.red[2][h] + ms.red[3][h];
          const float val = l > 0.f ? __uint_as_float(vv[j]) * sig / l : 0.f;
          const int hq = w.head_base + h;
          if (direct) {
            a.o[w.b * a.o_stride_b + hq * a.o_stride_h + d] = __float2bfloat16_rn(val);
          } else {
            const int64_t row = (static_cast<int64_t>(w.b) * a.num_splits + w.split) * a.num_heads + hq;
            a.partial_o[row * kLatent + d] = val;
          }
        }
      }
    }
    if (!direct && tid < w.heads_here) {
      const float l = ms.red[0][tid] + ms.red[1][tid] + ms.red[2][tid] + ms.red[3][tid];
      const int64_t row = (static_cast<int64_t>(w.b) * a.num_splits + w.split) * a.num_heads + w.head_base + tid;
      a.partial_lse[row] = (ms.R[tid] + __log2f(l)) * kLn2;
    }
  }
  fence_before_sync();
  named_bar(3, kThreadsTC);  // epilogue done -> warp 8 frees TMEM
}

}  // namespace

int decode_tc_smem_bytes() { return kSmemTC; }

cudaError_t launch_decode_tc(const DecodeArgs& a, cudaStream_t stream) {
  cudaError_t e = cudaFuncSetAttribute(mla_decode_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemTC);
  if (e != cudaSuccess) return e;
  const dim3 grid(a.num_splits, a.batch, (a.num_heads + kNH - 1) / kNH);
  mla_decode_tc_kernel<<<grid, kThreadsTC, kSmemTC, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace kimi
