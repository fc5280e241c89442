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
// Two launches on one stream, the second a programmatic dependent of the first:
//   * phase 1, one CTA per (head, 128-token tile, 64-column half of V): o's
//     tile (A, K-major) and W_UV's half (B, MN-major as stored) copied with
//     cp.async into 128-byte-swizzled shared memory (192 KB), 32 tcgen05.mma
//     kind::f16 (M = 128 tokens, N = 64, K = 16) into TMEM, x written as bf16
//     to a scratch [T, H * 128] that stays in L2;
//   * phase 2, one CTA per 64 outputs of the hidden dimension: its whole W_o
//     slice (64 x H * 128, at most 128 KB) is copied into shared memory BEFORE
//     waiting for phase 1 (griddepcontrol.wait), so the weight stream -- the
//     step's HBM traffic -- overlaps phase 1; then x streams through two
//     32 KB stages (K = 128 each) and one thread issues the MMAs (M = 128
//     tokens, N = 64); the CTA loops over 128-token tiles with its weights
//     resident.
// Every wait on an MMA commit is bounded; a give-up leaves that tile of the
// output unwritten.
#include <cuda_runtime.h>

#include "kernels.cuh"
#include "sm100.cuh"

namespace kimi {
namespace {

using namespace sm100;

constexpr int kTile = 128;                  // tokens per tile (the MMA's M)
constexpr int kVDim = 128;                  // v_head_dim
constexpr int kColsPerCta = 64;             // the MMA's N in both phases
constexpr uint32_t kPolls = 100000;         // suspend-hinted polls: about 2 s

// phase 1 shared memory: A = 8 K blocks x 128 rows x 128 B, B = 512 K rows x 128 B
constexpr int kP1OffA = 0;
constexpr int kP1KBlock = kTile * 128;      // 16 KB
constexpr int kP1OffB = 8 * kP1KBlock;      // 128 KB
constexpr int kP1OffMbar = kP1OffB + kLatent * 128;
constexpr int kP1Smem = kP1OffMbar + 64;

// phase 2 shared memory: W_o slice (K / 64 blocks x 64 rows x 128 B), then two
// A stages of 2 K blocks x 128 rows x 128 B
constexpr int kP2WBlock = kColsPerCta * 128;  // 8 KB per 64 K
constexpr int kP2Stage = 2 * kP1KBlock;       // 32 KB: K = 128 of 128 rows
constexpr int kP2MaxK = 1024;

__host__ __device__ constexpr int p2_off_a(int k) { return (k / 64) * kP2WBlock; }
__host__ __device__ constexpr int p2_off_mbar(int k) { return p2_off_a(k) + 2 * kP2Stage; }
__host__ __device__ constexpr int p2_smem(int k) { return p2_off_mbar(k) + 64; }

__device__ __forceinline__ void cp_async16(void* dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_addr(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// fp32 TMEM columns [col, col + 32) of this thread's lane -> 32 bf16 at dst (64 B)
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
__global__ void __launch_bounds__(256, 1) v_up_kernel(const __grid_constant__ VUpOProjArgs a) {
  extern __shared__ __align__(1024) uint8_t sm[];
  uint64_t* mbar = reinterpret_cast<uint64_t*>(sm + kP1OffMbar);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + kP1OffMbar + 8);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int h = blockIdx.x, t0 = blockIdx.y * kTile, z = blockIdx.z;
  const int ntok = min(kTile, a.num_tokens - t0);
  // the o_proj grid may start now: its prologue reads only W_o
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");

  if (tid == 0) {
    mbar_init(mbar, 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(tslot, kColsPerCta);
  // A: token r, 16-byte chunk c of its 512 latent elements (c / 8 = K block)
  const __nv_bfloat16* o = a.o + h * a.o_stride_h;
  for (int i = tid; i < kTile * 64; i += 256) {
    const int r = i >> 6, c = i & 63;
    const int rr = r < ntok ? r : 0;  // rows past the tokens read row 0's address and write zeros
    cp_async16(sm + kP1OffA + (c >> 3) * kP1KBlock + (r >> 3) * 1024 + sw128_offset(r & 7, c & 7),
               o + (t0 + rr) * a.o_stride_t + 8 * c, r < ntok ? 16u : 0u);
  }
  // B: K row k, 16-byte chunk c of this CTA's 64 columns of W_UV[h]
  const __nv_bfloat16* w = a.w_uv + static_cast<int64_t>(h) * kLatent * kVDim + kColsPerCta * z;
  for (int i = tid; i < kLatent * 8; i += 256) {
    const int k = i >> 3, c = i & 7;
    cp_async16(sm + kP1OffB + (k >> 3) * 1024 + sw128_offset(k & 7, c), w + k * kVDim + 8 * c, 16u);
  }
  asm volatile("cp.async.wait_all;\n" ::: "memory");
  fence_proxy_async_smem();
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = *tslot;

  if (tid == 0) {
    const uint32_t idesc = instr_desc(kFmtBF16, kFmtBF16, false, true, kTile, kColsPerCta);
    const uint64_t da = smem_desc(smem_addr(sm + kP1OffA), 16, 1024, kSwizzle128B);
    const uint64_t db = smem_desc(smem_addr(sm + kP1OffB), kLatent * 128, 1024, kSwizzle128B);
#pragma unroll
    for (int k = 0; k < kLatent / 16; ++k)
      mma_f16_ss(tmem, da + (((k >> 2) * kP1KBlock + (k & 3) * 32) >> 4), db + ((k * 2048) >> 4), idesc,
                 k > 0 ? 1u : 0u);
    mma_commit(mbar);
  }
  // warp-uniform, as the TMEM load below is a warp-wide instruction
  const bool done = __all_sync(0xffffffffu, mbar_wait_bounded(mbar, 0, kPolls));
  fence_after_sync();
  const int q = warp & 3, half = warp >> 2, r = 32 * q + lane;
  if (done) {
    uint32_t v[32];
    tmem_ld32(tmem + (static_cast<uint32_t>(32 * q) << 16) + 32 * half, v);
    tmem_ld_wait();
    if (r < ntok)
      store_bf16x32(a.x + static_cast<int64_t>(t0 + r) * a.num_heads * kVDim + h * kVDim + kColsPerCta * z + 32 * half,
                    v);
  }
  fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    fence_after_sync();
    tmem_dealloc(tmem, kColsPerCta);
  }
}

// ---------------------------------------------------------------------------
// phase 2: out[:, n0 .. n0 + 63] = bf16(x @ W_o[n0 .. n0 + 63, :]^T)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256, 1) o_proj_kernel(const __grid_constant__ VUpOProjArgs a) {
  extern __shared__ __align__(1024) uint8_t sm[];
  const int K = a.num_heads * kVDim;
  const int off_a = p2_off_a(K);
  uint64_t* mbar = reinterpret_cast<uint64_t*>(sm + p2_off_mbar(K));  // [2]: one per A stage
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + p2_off_mbar(K) + 16);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = blockIdx.x * kColsPerCta;
  const int kchunks = K / 128, chunks16 = K / 8;  // K chunks of the A ring; 16-byte chunks per W_o row

  if (tid == 0) {
    mbar_init(&mbar[0], 1);
    mbar_init(&mbar[1], 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(tslot, kColsPerCta);
  // W_o rows n0 .. n0 + 63 (K-major: row n, 16-byte chunk c along K), issued
  // before the dependency wait -- nothing here depends on phase 1
  const __nv_bfloat16* w = a.w_o + static_cast<int64_t>(n0) * K;
  for (int i = tid; i < kColsPerCta * chunks16; i += 256) {
    const int n = i / chunks16, c = i - n * chunks16;
    cp_async16(sm + (c >> 3) * kP2WBlock + (n >> 3) * 1024 + sw128_offset(n & 7, c & 7), w + n * K + 8 * c, 16u);
  }
  cp_async_commit();
  asm volatile("griddepcontrol.wait;\n" ::: "memory");  // phase 1 complete, x visible

  const int tiles = (a.num_tokens + kTile - 1) / kTile;
  const int total = tiles * kchunks;  // A chunks over all token tiles, in order
  // A chunk g (token tile g / kchunks, K columns 128 (g % kchunks) ..) into stage g % 2
  auto load_a = [&](int g) {
    const int t0 = (g / kchunks) * kTile, kc = g % kchunks;
    const int ntok = min(kTile, a.num_tokens - t0);
    uint8_t* st = sm + off_a + (g & 1) * kP2Stage;
    for (int i = tid; i < kTile * 16; i += 256) {
      const int r = i >> 4, c = i & 15;
      const int rr = r < ntok ? r : 0;
      cp_async16(st + (c >> 3) * kP1KBlock + (r >> 3) * 1024 + sw128_offset(r & 7, c & 7),
                 a.x + static_cast<int64_t>(t0 + rr) * K + 128 * kc + 8 * c, r < ntok ? 16u : 0u);
    }
    cp_async_commit();
  };
  load_a(0);
  if (total > 1) load_a(1);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = *tslot;
  const uint32_t idesc = instr_desc(kFmtBF16, kFmtBF16, false, false, kTile, kColsPerCta);
  const uint64_t dw = smem_desc(smem_addr(sm), 16, 1024, kSwizzle128B);
  bool ok = true;
  uint32_t parity = 0u;  // bit s: parity of stage s's next commit (its commits so far, mod 2)

  for (int g = 0; g < total; ++g) {
    const int kc = g % kchunks, s = g & 1;
    // this thread's copies of chunk g (and the weights) have landed
    if (g + 1 < total)
      cp_async_wait<1>();
    else
      cp_async_wait<0>();
    fence_proxy_async_smem();
    fence_before_sync();
    __syncthreads();  // everyone's copies
    fence_after_sync();
    if (tid == 0) {
      const uint64_t da = smem_desc(smem_addr(sm + off_a + s * kP2Stage), 16, 1024, kSwizzle128B);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int kk = 8 * kc + k;  // K step of 16 over the whole row
        mma_f16_ss(tmem, da + (((k >> 2) * kP1KBlock + (k & 3) * 32) >> 4),
                   dw + (((kk >> 2) * kP2WBlock + (kk & 3) * 32) >> 4), idesc, (kc > 0 || k > 0) ? 1u : 0u);
      }
      mma_commit(&mbar[s]);
    }
    const bool last_of_tile = kc == kchunks - 1;
    if (g + 2 < total || last_of_tile) {
      // stage s is rewritten next (chunk g + 2), or the tile's D is read: wait
      // for this chunk's MMAs (commits complete in order)
      ok = __all_sync(0xffffffffu, ok && mbar_wait_bounded(&mbar[s], (parity >> s) & 1u, kPolls));
      fence_after_sync();
    }
    parity ^= 1u << s;
    if (last_of_tile) {
      const int t0 = (g / kchunks) * kTile, ntok = min(kTile, a.num_tokens - t0);
      const int q = warp & 3, half = warp >> 2, r = 32 * q + lane;
      if (ok) {
        uint32_t v[32];
        tmem_ld32(tmem + (static_cast<uint32_t>(32 * q) << 16) + 32 * half, v);
        tmem_ld_wait();
        if (r < ntok) store_bf16x32(a.out + static_cast<int64_t>(t0 + r) * a.out_stride + n0 + 32 * half, v);
      }
      fence_before_sync();
      __syncthreads();  // D read before the next tile's first MMA overwrites it
      fence_after_sync();
    }
    if (g + 2 < total) load_a(g + 2);
  }
  fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    fence_after_sync();
    tmem_dealloc(tmem, kColsPerCta);
  }
}

}  // namespace

int v_up_o_proj_max_k() { return kP2MaxK; }

cudaError_t launch_v_up_o_proj(const VUpOProjArgs& a, cudaStream_t stream) {
  const int K = a.num_heads * kVDim;
  cudaError_t e = cudaFuncSetAttribute(v_up_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kP1Smem);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(o_proj_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, p2_smem(kP2MaxK));
  if (e != cudaSuccess) return e;
  const dim3 grid1(a.num_heads, (a.num_tokens + kTile - 1) / kTile, kVDim / kColsPerCta);
  v_up_kernel<<<grid1, 256, kP1Smem, stream>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.hidden / kColsPerCta);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = p2_smem(K);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, o_proj_kernel, a);
}

}  // namespace kimi
