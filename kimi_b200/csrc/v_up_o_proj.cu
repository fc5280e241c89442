// The decode step after attention: the V up-projection of the heads-first
// latent output by W_UV, then o_proj, on the tensor cores.
//
// Reference (paths inside ianye23301/kimi): `MLAAttention._v_up_proj_and_o_proj(
// x, heads_first=True)` (patches/atom-optimizations.patch:131-143, called on
// the decode's heads-first output at :297-302), checked in
// tests/test_mla_heads_first_e2e.py:50-59:
//   x[t, h*128 + v] = bf16( sum_l o[h, t, l] * W_UV[h, l, v] )     (fp32 BMM, one rounding)
//   out[t, :]       = bf16( x[t, :] @ W_o^T )                      (o_proj, fp32 accumulation)
// with o bf16 [H, T, 512] (heads-first, as the decode writes it), W_UV bf16
// [H, 512, 128], W_o bf16 [hidden, H * 128] (the Linear weight), out bf16
// [T, hidden] (this rank's partial of the tensor-parallel all-reduce).
//
// Two launches on one stream, the second a programmatic dependent of the
// first.  Every operand arrives by TMA (tiled, 128-byte swizzle: the UMMA
// operand layout; no multicast) on mbarriers:
//   * phase 1, one CTA per (head, kVUpRows tokens, 64-column half of V): the
//     8 K blocks of its o rows (A, K-major) and of W_UV's half (B, MN-major
//     as stored, 8 KB each) are all requested at once, one mbarrier per K
//     block, and the MMAs of a block (tcgen05.mma kind::f16, M = 128, N = 64,
//     K = 16) issue as soon as it lands; x is written as bf16 to a scratch
//     [T, H * 128] that stays in L2;
//   * phase 2, one CTA per 64 outputs of the hidden dimension, warp roles:
//     warp 0 lane 0 loads the CTA's whole W_o slice (64 x H * 128, at most
//     128 KB, resident) BEFORE waiting for phase 1 (griddepcontrol.wait), so
//     the weight stream -- the step's HBM traffic -- overlaps phase 1, then
//     streams x through a ring of six 16 KB stages (K = 64 each); warp 1
//     lane 0 issues the MMAs (M = 128 tokens, N = 64) into one of two TMEM
//     accumulators; warps 4-7 read a finished accumulator and write out while
//     the next token tile accumulates in the other.
// Every wait is bounded; a give-up raises a shared abort flag that ends the
// other roles' waits, and leaves the output unwritten or partly written.
#include <cuda_runtime.h>

#include "kernels.cuh"
#include "sm100.cuh"

namespace kimi {
namespace {

using namespace sm100;

constexpr int kTile = 128;           // tokens per tile (the MMA's M)
constexpr int kVDim = 128;           // v_head_dim
constexpr int kCols = 64;            // the MMA's N in both phases
constexpr uint32_t kPolls = 100000;  // suspend-hinted polls: about 2 s

// phase 1 shared memory
// A CTA loads kVUpRows tokens of o; its MMA still has M = 128 and the rows
// past them (read from whatever follows in shared memory) are computed and
// dropped.  The A blocks are packed at kVUpRows rows.
constexpr int kP1Rows = kVUpRows;
static_assert(kP1Rows % 32 == 0 && kP1Rows <= kTile, "whole TMEM lane quarters");
constexpr int kP1ABlock = kP1Rows * 128;  // one K block (64) of the CTA's o rows
constexpr int kP1BBlock = 64 * 128;       // 64 K rows of W_UV's half: 64 rows x 128 B
constexpr int kP1OffB = 8 * kP1ABlock;
constexpr int kP1OffBar = kP1OffB + 8 * kP1BBlock;  // full[8], dfull, abort, tmem slot
constexpr int kP1Smem = kP1OffBar + 128;

// phase 2 shared memory: W_o slice (K / 64 blocks of 64 rows x 128 B), then
// the x ring, then the barriers
constexpr int kP2WBlock = kCols * 128;  // 8 KB
constexpr int kP2Stages = 6;
constexpr int kP2Stage = kTile * 128;   // 16 KB: K = 64 of 128 token rows
constexpr int kP2MaxK = 1024;
constexpr int kP2TmemCols = 2 * kCols;  // two accumulators

__host__ __device__ constexpr int p2_off_ring(int k) { return (k / 64) * kP2WBlock; }
__host__ __device__ constexpr int p2_off_bar(int k) { return p2_off_ring(k) + kP2Stages * kP2Stage; }
__host__ __device__ constexpr int p2_smem(int k) { return p2_off_bar(k) + 256; }

struct P2Bars {
  uint64_t w_full;
  uint64_t a_full[kP2Stages];
  uint64_t a_empty[kP2Stages];
  uint64_t d_full[2];
  uint64_t d_empty[2];
  int abort;
  uint32_t tmem;
};
static_assert(sizeof(P2Bars) <= 256, "phase 2 barrier block");

__device__ __forceinline__ void arrive1(uint64_t* mbar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_addr(mbar)) : "memory");
}

// bounded wait that also ends when another role has given up; gives up itself
// by raising the flag
__device__ __forceinline__ bool wait_or_abort(uint64_t* mbar, uint32_t parity, volatile int* abort) {
  if (mbar_wait_or_abort(mbar, parity, kPolls, abort)) return true;
  *abort = 1;
  return false;
}

// the caller's status word, once per CTA that gave up
__device__ __forceinline__ void report_give_up(const VUpOProjArgs& a, volatile int* abort) {
  if (*abort && a.status && threadIdx.x == 0) atomicOr(a.status, kStatusVupWait);
}

// fp32 TMEM columns of this thread's lane -> 32 bf16 at dst (64 B)
__device__ __forceinline__ void store_bf16x32(__nv_bfloat16* dst, const uint32_t (&v)[32]) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t p[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const __nv_bfloat162 pr =
          __floats2bfloat162_rn(__uint_as_float(v[8 * j + 2 * e]), __uint_as_float(v[8 * j + 2 * e + 1]));
      p[e] = *reinterpret_cast<const uint32_t*>(&pr);
    }
    d[j] = make_uint4(p[0], p[1], p[2], p[3]);
  }
}

// ---------------------------------------------------------------------------
// phase 1: x[tile, h*128 + 64 z ..] = bf16(o[h, tile, :] @ W_UV[h][:, 64 z ..])
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256, 1)
    v_up_kernel(const __grid_constant__ VUpOProjArgs a, const __grid_constant__ VUpOProjMaps maps) {
  extern __shared__ __align__(1024) uint8_t sm[];
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + kP1OffBar);  // [8]
  uint64_t* dfull = full + 8;
  volatile int* abort = reinterpret_cast<volatile int*>(full + 9);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(full + 10);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int h = blockIdx.x, t0 = blockIdx.y * kP1Rows, z = blockIdx.z;
  const int ntok = min(kP1Rows, a.num_tokens - t0);
  // the o_proj grid may start now: its prologue reads only W_o
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");

  if (tid == 0) {
    for (int i = 0; i < 9; ++i) mbar_init(&full[i], 1);
    *abort = 0;
    fence_mbar_init();
    prefetch_tensormap(&maps.o);
    prefetch_tensormap(&maps.w_uv);
#pragma unroll 1
    for (int kb = 0; kb < 8; ++kb) {
      mbar_arrive_expect_tx(&full[kb], kP1ABlock + kP1BBlock);
      tma_load_3d(sm + kb * kP1ABlock, &maps.o, 64 * kb, t0, h, &full[kb]);
      tma_load_2d(sm + kP1OffB + kb * kP1BBlock, &maps.w_uv, kCols * z, h * kLatent + 64 * kb, &full[kb]);
    }
  }
  if (warp == 0) tmem_alloc(tslot, kCols);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = *tslot;

  if (tid == 0) {
    const uint32_t idesc = instr_desc(kFmtBF16, kFmtBF16, false, true, kTile, kCols);
    const uint64_t da = smem_desc(smem_addr(sm), 16, 1024, kSwizzle128B);
    const uint64_t db = smem_desc(smem_addr(sm + kP1OffB), 8 * kP1BBlock, 1024, kSwizzle128B);
#pragma unroll 1
    for (int kb = 0; kb < 8; ++kb) {
      if (!wait_or_abort(&full[kb], 0, abort)) break;
      fence_after_sync();
#pragma unroll
      for (int j = 0; j < 4; ++j)  // K step 4 kb + j: 32 B into A's rows, 16 rows (2 KB) into B
        mma_f16_ss(tmem, da + ((kb * kP1ABlock + j * 32) >> 4), db + ((kb * kP1BBlock + j * 2048) >> 4), idesc,
                   (kb > 0 || j > 0) ? 1u : 0u);
    }
    mma_commit(dfull);  // arrives at once when no MMA was issued
  }
  // warp-uniform, as the TMEM load below is a warp-wide instruction
  const bool done = __all_sync(0xffffffffu, wait_or_abort(dfull, 0, abort) && *abort == 0);
  fence_after_sync();
  const int q = warp & 3, half = warp >> 2, r = 32 * q + lane;
  if (done) {
    uint32_t v[32];
    tmem_ld32(tmem + (static_cast<uint32_t>(32 * q) << 16) + 32 * half, v);
    tmem_ld_wait();
    if (r < ntok) {
      store_bf16x32(a.x + static_cast<int64_t>(t0 + r) * a.num_heads * kVDim + h * kVDim + kCols * z + 32 * half, v);
      // the o_proj grid reads x through the async proxy (TMA)
      asm volatile("fence.proxy.async.global;\n" ::: "memory");
    }
  }
  fence_before_sync();
  __syncthreads();
  report_give_up(a, abort);
  if (warp == 0) {
    fence_after_sync();
    tmem_dealloc(tmem, kCols);
  }
}

// ---------------------------------------------------------------------------
// phase 2: out[:, n0 .. n0 + 63] = bf16(x @ W_o[n0 .. n0 + 63, :]^T)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256, 1)
    o_proj_kernel(const __grid_constant__ VUpOProjArgs a, const __grid_constant__ VUpOProjMaps maps) {
  extern __shared__ __align__(1024) uint8_t sm[];
  const int K = a.num_heads * kVDim;
  const int kblocks = K / 64;  // x chunks per token tile = W_o blocks
  P2Bars* bars = reinterpret_cast<P2Bars*>(sm + p2_off_bar(K));
  volatile int* abort = &bars->abort;
  uint8_t* ring = sm + p2_off_ring(K);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = blockIdx.x * kCols;
  const int tiles = (a.num_tokens + kTile - 1) / kTile;
  const int total = tiles * kblocks;

  if (tid == 0) {
    mbar_init(&bars->w_full, 1);
    for (int s = 0; s < kP2Stages; ++s) {
      mbar_init(&bars->a_full[s], 1);
      mbar_init(&bars->a_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->d_full[b], 1);
      mbar_init(&bars->d_empty[b], 128);
    }
    bars->abort = 0;
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(&bars->tmem, kP2TmemCols);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = bars->tmem;

  if (warp == 0 && lane == 0) {
    // ---- producer: the weights (no dependency on phase 1), then the x ring ----
    prefetch_tensormap(&maps.w_o);
    prefetch_tensormap(&maps.x);
    mbar_arrive_expect_tx(&bars->w_full, static_cast<uint32_t>(kblocks * kP2WBlock));
#pragma unroll 1
    for (int kb = 0; kb < kblocks; ++kb) tma_load_2d(sm + kb * kP2WBlock, &maps.w_o, 64 * kb, n0, &bars->w_full);
    asm volatile("griddepcontrol.wait;\n" ::: "memory");  // phase 1 complete, x written
#pragma unroll 1
    for (int g = 0; g < total; ++g) {
      const int s = g % kP2Stages;
      if (g >= kP2Stages && !wait_or_abort(&bars->a_empty[s], ((g / kP2Stages) - 1) & 1, abort)) break;
      mbar_arrive_expect_tx(&bars->a_full[s], kP2Stage);
      tma_load_2d(ring + s * kP2Stage, &maps.x, 64 * (g % kblocks), (g / kblocks) * kTile, &bars->a_full[s]);
    }
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issue ----
    const uint32_t idesc = instr_desc(kFmtBF16, kFmtBF16, false, false, kTile, kCols);
    const uint64_t dw = smem_desc(smem_addr(sm), 16, 1024, kSwizzle128B);
    bool ok = wait_or_abort(&bars->w_full, 0, abort);
    fence_after_sync();
#pragma unroll 1
    for (int i = 0; ok && i < tiles; ++i) {
      const int b = i & 1;
      if (i >= 2 && !(ok = wait_or_abort(&bars->d_empty[b], ((i >> 1) - 1) & 1, abort))) break;
      fence_after_sync();
#pragma unroll 1
      for (int c = 0; c < kblocks; ++c) {
        const int g = i * kblocks + c, s = g % kP2Stages;
        if (!(ok = wait_or_abort(&bars->a_full[s], (g / kP2Stages) & 1, abort))) break;
        fence_after_sync();
        const uint64_t da = smem_desc(smem_addr(ring + s * kP2Stage), 16, 1024, kSwizzle128B);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          mma_f16_ss(tmem + b * kCols, da + ((j * 32) >> 4), dw + ((c * kP2WBlock + j * 32) >> 4), idesc,
                     (c > 0 || j > 0) ? 1u : 0u);
        mma_commit(&bars->a_empty[s]);  // the stage is free once these MMAs have read it
      }
      if (ok) mma_commit(&bars->d_full[b]);
    }
  } else if (warp >= 4) {
    // ---- epilogue: lanes 32 (warp % 4) .. + 31 of the accumulator ----
    const int q = warp & 3, r = 32 * q + lane;
#pragma unroll 1
    for (int i = 0; i < tiles; ++i) {
      const int b = i & 1, t0 = i * kTile, ntok = min(kTile, a.num_tokens - t0);
      if (!__all_sync(0xffffffffu, wait_or_abort(&bars->d_full[b], (i >> 1) & 1, abort))) break;
      fence_after_sync();
#pragma unroll 1
      for (int h2 = 0; h2 < 2; ++h2) {
        uint32_t v[32];
        tmem_ld32(tmem + (static_cast<uint32_t>(32 * q) << 16) + b * kCols + 32 * h2, v);
        tmem_ld_wait();
        if (r < ntok) store_bf16x32(a.out + static_cast<int64_t>(t0 + r) * a.out_stride + n0 + 32 * h2, v);
      }
      fence_before_sync();
      arrive1(&bars->d_empty[b]);  // this accumulator may take tile i + 2
    }
  }
  fence_before_sync();
  __syncthreads();
  report_give_up(a, abort);
  if (warp == 0) {
    fence_after_sync();
    tmem_dealloc(tmem, kP2TmemCols);
  }
}

}  // namespace

cudaError_t launch_v_up_o_proj(const VUpOProjArgs& a, const VUpOProjMaps& maps, cudaStream_t stream) {
  const int K = a.num_heads * kVDim;
  cudaError_t e = cudaFuncSetAttribute(v_up_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kP1Smem);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(o_proj_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, p2_smem(kP2MaxK));
  if (e != cudaSuccess) return e;
  const dim3 grid1(a.num_heads, (a.num_tokens + kP1Rows - 1) / kP1Rows, kVDim / kCols);
  v_up_kernel<<<grid1, 256, kP1Smem, stream>>>(a, maps);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.hidden / kCols);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = p2_smem(K);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, o_proj_kernel, a, maps);
}

}  // namespace kimi
