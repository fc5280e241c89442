// Split-K absorbed-MLA decode over the MXFP4 paged cache on the 5th-generation
// tensor cores (tcgen05 + TMEM), sm_100a.
//
// Math (paths inside ianye23301/kimi): the archive stage-1 kernel
// `_mla_decode_split_kv` (archive/mla-mxfp4-dead-end/mla_decode_mxfp4_v5.py:136-261)
// with the contract of `reference_mla_decode` (tests/test_triton_mla_decode.py:12-62):
//   S = q_nope . k_nope + q_pe . k_pe,  P = softmax(S * sm_scale),  O = P . k_nope.
//
// One CTA = up to 64 heads over a run of 128-token tiles: a range of one
// sequence (split mode) or a range of the whole batch's tiles laid end to end,
// which may cross sequence boundaries (balanced mode; see DecodeArgs).  The
// roles walk that run with identical cursors; at a sequence boundary the
// softmax warps finish the piece (its output or partial) and build the next
// sequence's Q'' before the QK issuer continues.
//   * The cache is consumed in tiles of 128 tokens (two pages).  Tokens sit on
//     the MMA's M dimension (M = 128) and heads on N ("swap AB").
//   * Each latent element is dequantised ONCE per tile into an 8-bit tile V''
//     in shared memory: the e2m1 code times its e8m0 scale relative to a
//     reference 2^sigma, written as e5m2 (e2m1 * 2^k has one mantissa bit, so
//     the value is exact while the exponent is in e5m2's range; sigma follows
//     the tile maxima, see below).  The conversion is a byte permute through a
//     two-register table per 32-element group (no conversion instructions).
//     V'' sits in 128B-swizzled atoms (8 tokens x 128 latent bytes) and is read
//     by the tensor core twice: K-major as the A operand of S^T = V'' . Q''^T
//     and MN-major as the A operand of O^T = V''^T . P''^T.
//   * q_nope is split into two e4m3 terms with a per-head power-of-two scale
//     a_h (q / a_h = hi + lo), stacked as one N = 128 B operand: bf16-level
//     accuracy for QK^T at fp8 tensor rate.  q_pe . k_pe is a bf16 MMA whose
//     A operand (k_pe) sits in TMEM.
//   * P'' = exp2(x - R_h) is likewise two e4m3 terms (hi + residual), two PV
//     MMAs into the same accumulator (one e4m3 term alone costs ~2% relative
//     error on short contexts).  R_h is a per-head offset kept within
//     [max - 8.5, max - 4] of the running max, raised lazily.
//   * The O accumulator holds sum_t exp2(x - R_h) V 2^-sigma.  When a tile
//     raises R_h, or needs a different sigma (its largest scale more than 13
//     binades above, or 4 below, the reference), O and the softmax sums are
//     rescaled in TMEM before that tile's PV.
//   * TMEM (512 columns): S_hi|S_lo [0,128), S_pe [128,192),
//     k_pe double buffer [192,256), O^T [256,512) as four 128-row latent
//     chunks of 64 head columns.
//
// Warp roles (16 warps, 512 threads):
//   warps 0-7   softmax: S(j) -> P''(j), O rescales, the epilogue;
//   warps 8-11  loaders: global -> registers one tile ahead, then V''(j) and
//               k_pe(j) (one TMEM lane quadrant each);
//   warp 12     allocates TMEM and issues QK(j) (+ the RoPE MMAs);
//   warps 13-14 issue PV(j) (latent chunks {0,1} and {2,3}): a single thread
//               issues one tcgen05.mma every ~64 cycles while the N = 64 PV
//               MMAs take ~48, so PV needs two issuers to keep the tensor pipe
//               fed; warp 15 only completes the warpgroup.
// V'' and k_pe are double-buffered, so QK(j+1) overlaps softmax(j) and the
// loaders' D(j+2) overlaps PV(j+1).  Every mbarrier wait is bounded; a wait
// that gives up sets a shared abort word that every other wait polls, each
// role leaves its loop collectively, the issuers drain their MMAs and TMEM is
// freed as usual.
#include <cstddef>

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math_constants.h>

#include "decode_common.cuh"
#include "kernels.cuh"
#include "sm100.cuh"

namespace kimi {
namespace {

using namespace sm100;
using namespace dec;

constexpr int kNH = 64;               // heads per CTA (N of the MMAs)
constexpr int kSoftmaxWarps = 8;
constexpr int kLoaderWarp0 = 8;       // warps 8..11
constexpr int kWarpQK = 12;
constexpr int kWarpPV0 = 13;          // warps 13, 14 (warp 15 idles)
constexpr int kPvIssuers = 2;
constexpr int kThreadsTC = 512;
constexpr int kSoftmaxThreads = 32 * kSoftmaxWarps;
constexpr int kLoaderThreads = 128;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0, kColSpe = 128, kColKpe = 192, kColO = 256;
constexpr uint32_t kPollLimit = 100000;  // polls of up to kWaitSleepNs each: about 2 s
// Register budgets: 512 threads launch with 128 registers each (65536).  The
// loader warpgroup takes 184, the issuer warpgroup gives back down to 72:
// 256 * 128 + 128 * 184 + 128 * 72 = 65536.
constexpr uint32_t kLoaderRegs = 184;
constexpr uint32_t kIssuerRegs = 72;
static_assert(256 * 128 + 128 * kLoaderRegs + 128 * kIssuerRegs <= kThreadsTC * 128, "register split");

// Named barriers (0 is __syncthreads)
constexpr int kBarSoftmax = 1;
constexpr int kBarLoader = 2;
constexpr int kBarSetup = 3;  // all 512 threads, once: barriers, TMEM and the first Q'' are ready

// Shared memory (bytes).  Core matrix (r, c) of an operand lives at
// r * row_stride + c * 128, 16 bytes per row inside the core.
// V'' (e5m2) and Q'' (e4m3) use 128B-swizzled atoms of 8 rows x 128 bytes:
// atom (row group rg, latent column dcol) at dcol * 16 KB + rg * 1 KB, so the
// same V'' bytes serve as a K-major (tokens x latent) and an MN-major
// (latent x tokens) operand.
constexpr int kVBytes = 65536;      // V'' tile: 16 token groups x 4 latent columns
constexpr int kVCol = 16384;        // one 128-byte latent column of 16 atoms
constexpr int kOffV = 0;            // two V'' buffers
constexpr int kOffQ = 2 * kVBytes;  // Q'' e4m3 hi rows 0..63, lo rows 64..127 (same atom layout): 64 KB
constexpr int kOffQpe = kOffQ + 65536;  // q_pe bf16, cores (head group 0..7, byte group 0..7): 8 KB
constexpr int kPeRow = 8 * 128;
constexpr int kOffP = kOffQpe + 8192;   // P'' hi e4m3, MN-major cores (token group 0..15, head byte group 0..3)
constexpr int kOffPlo = kOffP + 8192;   // P'' lo (residual), same layout
constexpr int kPRow = 4 * 128;
constexpr int kOffMisc = kOffPlo + 8192;

struct Misc {
  uint64_t mb_vfull[2];   // V''/k_pe buffer b written (4 loader warp arrivals)
  uint64_t mb_pvdone[2];  // PV of the tile in buffer b complete (one commit per PV issuer)
  uint64_t mb_sfull;      // QK(j) complete (tcgen05.commit)
  uint64_t mb_sfree;      // S(j) read out of TMEM (8 softmax warp arrivals)
  uint64_t mb_pfull;      // P''(j) written, O rescaled (8 softmax warp arrivals)
  uint64_t mb_drain;      // each issuer's last commit (1 + kPvIssuers arrivals)
  uint64_t mb_qready;     // Q'' of the next piece's sequence written (8 softmax warp arrivals)
  SchedScratch sched;     // balanced mode: block-scan scratch
  uint32_t tmem_base;
  int abort_flag;
  int tile_smax[4];       // max e8m0 byte of tile j in slot j % 4 (reset two tiles ahead)
  int sig[2];             // reference exponent sigma of the tile in V'' buffer b
  alignas(16) float ac[kNH];  // a_h * sm_scale * log2(e)   (read as float4)
  alignas(16) float R[kNH];   // per-head exp2 offset, log2 units (read as float4)
  float alpha[kNH];   // O rescale factors of the current event
  float beta[kNH];    // softmax-sum rescale factors of the current event
  float red[4][kNH];  // cross-warp reduction scratch
};
constexpr int kSmemTC = kOffMisc + static_cast<int>(sizeof(Misc));
static_assert(kSmemTC <= 232448, "shared memory budget");
static_assert(kOffMisc % 16 == 0 && offsetof(Misc, ac) % 16 == 0 && offsetof(Misc, R) % 16 == 0,
              "per-head arrays are read with 16-byte vector loads");
static_assert(offsetof(Misc, mb_vfull) % 8 == 0 && offsetof(Misc, mb_qready) % 8 == 0, "mbarriers are 8-byte aligned");

__device__ __forceinline__ uint8_t* smem_base() {
  extern __shared__ __align__(1024) uint8_t dyn_smem[];
  return dyn_smem;
}

__device__ __forceinline__ void setup_barrier() {
  fence_before_sync();
  named_bar(kBarSetup, kThreadsTC);
  fence_after_sync();
}

// Raw data of one tile held by one loader thread (quadrant q = its warp - 8,
// tokens 32q .. 32q + 31 of the tile, all in one page).  Latent nibbles: lane
// l holds e8m0 group g = (l % 4) + 4 (l / 8) (one 16-byte chunk) of token
// 32q + 2i + e, e = (l / 4) % 2, for i = 0..15, with the matching scale bytes.
// Every load instruction reads two whole token rows (four 128-byte lines), and
// each 8-lane phase of a V'' store covers two tokens of opposite parity x four
// groups: eight distinct 16-byte bank groups of the swizzled atoms.  RoPE: in
// load k (0..7) lane l reads 16-byte chunk l % 8 of token 32q + 4k + l / 8
// (line-coalesced); the loader transposes it to one token per lane.
struct RawTile {
  uint4 nib[16];
  uint32_t sb[16];
  uint4 pe[8];
  int nvalid;
  bool first;        // first tile of a piece
  int page_next[2];  // page ids of the tile loaded next (fetched one tile ahead)
  int page_pf[2];    // page ids of the tile prefetched into L2 next (loader thread 0 only)
};

// L2 prefetch distance in tiles: the register loads of tile j find its pages
// in L2, fetched while tiles j - kPrefetchTiles .. j - 1 were processed.
constexpr int kPrefetchTiles = 3;

__device__ __forceinline__ void fetch_pages(const DecodeArgs& a, const Cursor& c, int (&pg)[2]) {
#pragma unroll
  for (int slot = 0; slot < 2; ++slot) {
    const int p = 2 * c.tile + slot;
    const bool in_range = p < c.n_pages;
    pg[slot] = ldg_s32_or(a.kv_indices + c.page_lo + (in_range ? p : 0), in_range, -1);
  }
}

// Registers of tile `c` (page ids already in r.page_next); then the page ids of tile `next`.
__device__ __forceinline__ void load_tile(const DecodeArgs& a, const Cursor& c, const Cursor& next, int q, int lane,
                                          RawTile& r) {
  const int nvalid = cursor_valid(c);
  r.nvalid = nvalid;
  r.first = cursor_first(c);
  const int pid = (q >> 1) ? r.page_next[1] : r.page_next[0];  // (a select keeps page_next in registers)
  const int page = (pid >= 0 && pid < a.num_pages) ? pid : -1;
  const uint8_t* pbase = a.kv_buffer + static_cast<int64_t>(page < 0 ? 0 : page) * kPageBytes;
  const uint8_t* sbase = a.kv_scales + static_cast<int64_t>(page < 0 ? 0 : page) * kPageScaleBytes;
  const int e = (lane >> 2) & 1, g = (lane & 3) | ((lane >> 3) << 2);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int tk = 32 * q + 2 * i + e;
    r.nib[i] = ldg_stream_if(pbase + (tk & 63) * kTokenBytes + 16 * g, page >= 0 && tk < nvalid);
  }
  // (each byte stays in its own register: combining them here would wait for the loads)
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int tk = 32 * q + 2 * i + e;
    r.sb[i] = ldg_u8_if(sbase + (tk & 63) * kScaleBytes + g, page >= 0 && tk < nvalid);
  }
  // RoPE, line-coalesced: in load k lane l reads 16-byte chunk l % 8 of token 32q + 4k + l / 8
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int tk = 32 * q + 4 * k + (lane >> 3);
    r.pe[k] = ldg_stream_if(pbase + (tk & 63) * kTokenBytes + kNibbleBytes + 16 * (lane & 7),
                            page >= 0 && tk < nvalid);
  }
  fetch_pages(a, next, r.page_next);
}

// Loader thread 0: prefetch the pages (cache rows and scales) of one tile into L2.
__device__ __forceinline__ void prefetch_tile(const DecodeArgs& a, const int (&pg)[2]) {
#pragma unroll
  for (int slot = 0; slot < 2; ++slot) {
    if (pg[slot] >= 0 && pg[slot] < a.num_pages) {
      prefetch_l2(a.kv_buffer + static_cast<int64_t>(pg[slot]) * kPageBytes, kPageBytes);
      prefetch_l2(a.kv_scales + static_cast<int64_t>(pg[slot]) * kPageScaleBytes, kPageScaleBytes);
    }
  }
}

// Prefetch the q rows of sequence b (this CTA's heads) into L2; thread `i` of
// `n` cooperating threads issues its share.
__device__ __forceinline__ void prefetch_q(const DecodeArgs& a, int b, int head_base, int heads_here, int i, int n) {
  const __nv_bfloat16* base = a.q + static_cast<int64_t>(b) * a.q_stride_b + static_cast<int64_t>(head_base) * a.q_stride_h;
  if (a.q_stride_h == kQkDim) {
    if (i == 0) prefetch_l2(base, static_cast<uint32_t>(heads_here * kQkDim * 2));
  } else {
    for (int h = i; h < heads_here; h += n) prefetch_l2(base + static_cast<int64_t>(h) * a.q_stride_h, kQkDim * 2);
  }
}

__device__ __forceinline__ void record_status(const DecodeArgs& a, int bits) {
  if (a.status) atomicOr(a.status, bits);
}

// Per-thread bounded wait; on give-up records the failure and raises the abort word.
__device__ __forceinline__ bool wait_phase(uint64_t* mb, uint32_t parity, Misc& ms, const DecodeArgs& a, int bit) {
  if (mbar_wait_or_abort(mb, parity, kPollLimit, &ms.abort_flag)) return true;
  if (atomicExch(&ms.abort_flag, 1) == 0) record_status(a, bit);
  return false;
}

// Warp-uniform bounded wait: lane 0 polls, the warp gets its verdict.
__device__ __forceinline__ bool warp_wait(uint64_t* mb, uint32_t parity, Misc& ms, const DecodeArgs& a, int bit,
                                          int lane) {
  bool ok = true;
  if (lane == 0) ok = wait_phase(mb, parity, ms, a, bit);
  return __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
}

// ---------------------------------------------------------------------------
// Issuers (warps 12..15; lane 0 issues)
// ---------------------------------------------------------------------------
__device__ void qk_issuer(uint8_t* sm, Misc& ms, uint32_t tmem, const Sched& sc, int lane, const DecodeArgs& a) {
  const uint32_t id_qk = instr_desc(kFmtE5M2, kFmtE4M3, false, false, 128, 128);
  const uint32_t id_pe = instr_desc(kFmtBF16, kFmtBF16, false, false, 128, 64);
  const uint32_t sQ = smem_addr(sm + kOffQ), sQpe = smem_addr(sm + kOffQpe);
  Cursor cur;
  cursor_start(a, sc, cur);
  int pieces = 0;
  for (int j = 0; j < sc.count; ++j, cursor_next(a, cur)) {
    // QK(j) needs V''(j)/k_pe(j) written and S(j-1) read out of TMEM (single S
    // buffer); the first tile of a later piece also needs that sequence's Q''.
    if (!warp_wait(&ms.mb_vfull[j & 1], static_cast<uint32_t>((j >> 1) & 1), ms, a, 16, lane)) break;
    if (j > 0 && !warp_wait(&ms.mb_sfree, static_cast<uint32_t>((j - 1) & 1), ms, a, 16, lane)) break;
    if (j > 0 && cursor_first(cur)) {
      if (!warp_wait(&ms.mb_qready, static_cast<uint32_t>(pieces & 1), ms, a, 16, lane)) break;
      ++pieces;
    }
    fence_after_sync();
    if (lane == 0) {
      const uint32_t sV = smem_addr(sm + kOffV + (j & 1) * kVBytes);
      // The 16 latent MMAs chain on one accumulator; the 4 RoPE MMAs (own
      // accumulator) are interleaved so they fill the chain's latency.
      const uint32_t kpe = tmem + kColKpe + 32 * (j & 1);
#pragma unroll 1
      for (int k = 0; k < 16; ++k) {
        const uint32_t koff = (k >> 2) * kVCol + (k & 3) * 32;
        mma_f8f6f4_ss(tmem + kColS, smem_desc(sV + koff, 16, 1024, kSwizzle128B),
                      smem_desc(sQ + koff, 16, 1024, kSwizzle128B), id_qk, k > 0);
        if (k < 4) mma_f16_ts(tmem + kColSpe, kpe + 8 * k, smem_desc(sQpe + k * 256, 128, kPeRow), id_pe, k > 0);
      }
      mma_commit(&ms.mb_sfull);
    }
    __syncwarp();
  }
}

// PV issuer p owns latent chunks 2p and 2p + 1.
__device__ void pv_issuer(uint8_t* sm, Misc& ms, uint32_t tmem, const Sched& sc, int lane, int p,
                          const DecodeArgs& a) {
  const uint32_t id_pv = instr_desc(kFmtE5M2, kFmtE4M3, true, true, 128, 64);
  const uint32_t sP = smem_addr(sm + kOffP), sPlo = smem_addr(sm + kOffPlo);
  const int c0 = 2 * p;
  const int c1 = 2 * p + 2;
  Cursor cur;
  cursor_start(a, sc, cur);
  for (int j = 0; j < sc.count; ++j, cursor_next(a, cur)) {
    // PV(j) needs P''(j) (written after PV(j-1) completed and O was rescaled or,
    // at a piece start, read out by the previous piece's epilogue)
    if (!warp_wait(&ms.mb_pfull, static_cast<uint32_t>(j & 1), ms, a, 32, lane)) break;
    fence_after_sync();
    if (lane == 0) {
      const uint32_t sV = smem_addr(sm + kOffV + (j & 1) * kVBytes);
      const bool fresh = cursor_first(cur);  // the piece's first PV starts the accumulator
#pragma unroll 1
      for (int k = 0; k < 4; ++k) {
        const uint64_t phi = smem_desc(sP + k * 4 * kPRow, kPRow, 128);
        const uint64_t plo = smem_desc(sPlo + k * 4 * kPRow, kPRow, 128);
        for (int c = c0; c < c1; ++c)
          mma_f8f6f4_ss(tmem + kColO + 64 * c, smem_desc(sV + c * kVCol + k * 4096, kVCol, 1024, kSwizzle128B), phi,
                        id_pv, (fresh && k == 0) ? 0u : 1u);
        for (int c = c0; c < c1; ++c)
          mma_f8f6f4_ss(tmem + kColO + 64 * c, smem_desc(sV + c * kVCol + k * 4096, kVCol, 1024, kSwizzle128B), plo,
                        id_pv, 1u);
      }
      mma_commit(&ms.mb_pvdone[j & 1]);
    }
    __syncwarp();
  }
}

// ---------------------------------------------------------------------------
// Loaders (warps 8..11): V''(j) and k_pe(j) from registers, then the next tile's loads
// ---------------------------------------------------------------------------
__device__ void loader(uint8_t* sm, Misc& ms, const Sched& sc, int head_base, int heads_here, int q, int lane,
                       const DecodeArgs& a) {
  const int ltid = 32 * q + lane;
  const uint32_t lane_base = static_cast<uint32_t>(32 * q) << 16;
  const int e = (lane >> 2) & 1, g = (lane & 3) | ((lane >> 3) << 2);
  // lc: the tile whose registers are loaded; fc: the next one (its page ids are
  // fetched one tile ahead); pc: the tile loader thread 0 last prefetched into L2.
  Cursor lc, fc;
  cursor_start(a, sc, lc);
  fc = lc;
  cursor_next(a, fc);
  RawTile r;
  fetch_pages(a, lc, r.page_next);
  // page ids of tiles 1 .. kPrefetchTiles, requested together with tile 0's
  Cursor pc = lc;
  int pf_ids[kPrefetchTiles][2];
#pragma unroll
  for (int t = 0; t < kPrefetchTiles; ++t) {
    cursor_next(a, pc);
    if (ltid == 0 && t + 1 < sc.count) {
      fetch_pages(a, pc, pf_ids[t]);
    } else {
      pf_ids[t][0] = pf_ids[t][1] = -1;
    }
  }
  // the first tile's loads overlap the setup (TMEM, barriers, Q''), then the
  // next tiles are prefetched into L2
  load_tile(a, lc, fc, q, lane, r);
  if (ltid == 0) {
#pragma unroll
    for (int t = 0; t < kPrefetchTiles; ++t) prefetch_tile(a, pf_ids[t]);
  }
  setup_barrier();
  const uint32_t tmem = ms.tmem_base;
  int prev_sigma = 0;
  for (int j = 0; j < sc.count; ++j) {
    const int buf = j & 1;
    // V'' buffer j & 1 (and its k_pe TMEM buffer) was last read by PV(j-2) / QK(j-2)
    bool ok = true;
    if (j >= 2) ok = warp_wait(&ms.mb_pvdone[buf], static_cast<uint32_t>(((j >> 1) - 1) & 1), ms, a, 64, lane);
    // tile maximum of the e8m0 bytes (invalid tokens carry 0) -> reference exponent
    uint32_t my_max = 0u;
#pragma unroll
    for (int i = 0; i < 16; ++i) my_max = max(my_max, r.sb[i]);
    my_max = __reduce_max_sync(0xffffffffu, my_max);
    if (lane == 0) atomicMax(&ms.tile_smax[j & 3], static_cast<int>(my_max));
    if (bar_or(kBarLoader, kLoaderThreads, !ok)) break;
    const int smax = ms.tile_smax[j & 3];
    int sigma;
    if (r.first) {
      sigma = smax - 127 - 8;  // tile max maps to <= 6 * 2^8 in V''
    } else {
      const int kmax = smax - 127 - prev_sigma;
      sigma = (kmax > 13 || kmax < -4) ? smax - 127 - 8 : prev_sigma;
    }
    if (ltid == 0) {
      ms.tile_smax[(j + 2) & 3] = 0;
      ms.sig[buf] = sigma;
    }
    prev_sigma = sigma;

    // k_pe: token-per-lane transpose through this warp's own 4 KB of V'' (latent
    // column 0, tokens 32q .. 32q + 31; overwritten by the V'' stores below).
    // Chunk c of local token t sits at t * 128 + (c ^ (t & 7)) * 16: both the
    // coalesced write and the per-token read touch eight distinct 16-byte bank groups.
    uint32_t kpe[32];
    {
      uint8_t* scratch = sm + kOffV + buf * kVBytes + 4096 * q;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int t = 4 * k + (lane >> 3), c = lane & 7;
        *reinterpret_cast<uint4*>(scratch + t * 128 + ((c ^ (t & 7)) * 16)) = r.pe[k];
      }
      __syncwarp();
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint4 v = *reinterpret_cast<const uint4*>(scratch + lane * 128 + ((c ^ (lane & 7)) * 16));
        kpe[4 * c] = v.x;
        kpe[4 * c + 1] = v.y;
        kpe[4 * c + 2] = v.z;
        kpe[4 * c + 3] = v.w;
      }
      __syncwarp();
      // -> TMEM columns [kColKpe + 32 buf, +32) of this thread's TMEM lane (token 32q + lane)
      tmem_st32(tmem + lane_base + kColKpe + 32 * buf, kpe);
    }
    // group g of sixteen tokens -> two 16-byte chunks (latent bytes 32g .. 32g + 31) each
    uint8_t* vb = sm + kOffV + buf * kVBytes + (g >> 2) * kVCol;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int tk = 32 * q + 2 * i + e;
      const uint32_t sbyte = r.sb[i];
      uint32_t lo, hi;
      e5m2_tables(static_cast<int>(sbyte) - 127 - sigma, lo, hi);
      const uint4 nb = r.nib[i];
      uint8_t* atom = vb + (tk >> 3) * 1024;
      *reinterpret_cast<uint4*>(atom + sw128_offset(tk & 7, (2 * g) & 7)) = half_group_to_e5m2(nb.x, nb.y, lo, hi);
      *reinterpret_cast<uint4*>(atom + sw128_offset(tk & 7, (2 * g + 1) & 7)) = half_group_to_e5m2(nb.z, nb.w, lo, hi);
    }
    tmem_st_wait();
    fence_proxy_async_smem();
    fence_before_sync();
    __syncwarp();
    if (lane == 0) mbar_arrive(&ms.mb_vfull[buf]);
    if (j + 1 < sc.count) {
      lc = fc;
      cursor_next(a, fc);
      if (ltid == 0 && j + 1 + kPrefetchTiles < sc.count) {
        cursor_next(a, pc);  // tile j + 1 + kPrefetchTiles
        fetch_pages(a, pc, r.page_pf);
        prefetch_tile(a, r.page_pf);
        // a new sequence ahead: its q rows, for the softmax warps' Q'' rebuild
        if (cursor_first(pc)) prefetch_q(a, pc.b, head_base, heads_here, 0, 1);
      }
      load_tile(a, lc, fc, q, lane, r);
    }
  }
}

// ---------------------------------------------------------------------------
// Q'' of one sequence (softmax threads 0..255: 4 per head; part p handles latent
// [128p, 128p + 128) and RoPE [16p, 16p + 16))
// ---------------------------------------------------------------------------
__device__ void build_q(uint8_t* sm, Misc& ms, const DecodeArgs& a, int b, int head_base, int heads_here,
                        float c_log2) {
  const int tid = threadIdx.x;
  const int h = tid >> 2, part = tid & 3;
  const bool live = h < heads_here;
  const __nv_bfloat16* qrow = a.q + b * a.q_stride_b + (head_base + h) * a.q_stride_h;
  // Two passes over this thread's 128 latent values, every load of a pass in
  // flight at once (the rows were prefetched into L2; the second pass hits).
  float amax = 0.f;
  {
    uint4 v[16];
#pragma unroll
    for (int k = 0; k < 16; ++k)
      v[k] = live ? *reinterpret_cast<const uint4*>(qrow + 128 * part + 8 * k) : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const uint32_t ws[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
#pragma unroll
      for (int j = 0; j < 4; ++j)
        amax = fmaxf(amax, fmaxf(fabsf(__uint_as_float(ws[j] << 16)), fabsf(__uint_as_float(ws[j] & 0xFFFF0000u))));
    }
  }
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
  // a_h = 2^(floor(log2 amax) - 7): |q / a_h| < 256 < 448 (e4m3 max)
  int ex = static_cast<int>((__float_as_uint(amax) >> 23) & 0xFF) - 127 - 7;
  if (amax == 0.f || ex < -126) ex = 0;
  const float a_h = __uint_as_float(static_cast<uint32_t>(ex + 127) << 23);
  const float inv_a = __uint_as_float(static_cast<uint32_t>(127 - ex) << 23);
  if (part == 0) {
    ms.ac[h] = a_h * c_log2;
    ms.R[h] = 0.f;
  }
  uint8_t* qb = sm + kOffQ;
#pragma unroll 1
  for (int half = 0; half < 2; ++half) {
    uint4 v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k)
      v[k] = live ? *reinterpret_cast<const uint4*>(qrow + 128 * part + 64 * half + 8 * k) : make_uint4(0, 0, 0, 0);
#pragma unroll
  for (int k2 = 0; k2 < 8; k2 += 2) {
    const int k = 8 * half + k2;
    // 16 latent elements = one 16-byte core row of hi and of lo
    uint32_t hi_w[4], lo_w[4];
    const uint4 v0 = v[k2], v1 = v[k2 + 1];
    const uint32_t ws[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float x0 = __uint_as_float(ws[2 * j] << 16) * inv_a;
      const float x1 = __uint_as_float(ws[2 * j] & 0xFFFF0000u) * inv_a;
      const float x2 = __uint_as_float(ws[2 * j + 1] << 16) * inv_a;
      const float x3 = __uint_as_float(ws[2 * j + 1] & 0xFFFF0000u) * inv_a;
      const uint16_t h01 = cvt_f32x2_e4m3x2(x0, x1);
      const uint16_t h23 = cvt_f32x2_e4m3x2(x2, x3);
      const float2 g01 = e4m3x2_to_float2(h01);  // exact
      const float2 g23 = e4m3x2_to_float2(h23);
      const uint16_t l01 = cvt_f32x2_e4m3x2(x0 - g01.x, x1 - g01.y);
      const uint16_t l23 = cvt_f32x2_e4m3x2(x2 - g23.x, x3 - g23.y);
      hi_w[j] = static_cast<uint32_t>(h01) | (static_cast<uint32_t>(h23) << 16);
      lo_w[j] = static_cast<uint32_t>(l01) | (static_cast<uint32_t>(l23) << 16);
    }
    const int dc = 8 * part + k / 2;  // 16-byte latent chunk of this row (0..31)
    uint8_t* col = qb + (dc >> 3) * kVCol;
    *reinterpret_cast<uint4*>(col + (h >> 3) * 1024 + sw128_offset(h & 7, dc & 7)) =
        make_uint4(hi_w[0], hi_w[1], hi_w[2], hi_w[3]);
    *reinterpret_cast<uint4*>(col + (8 + (h >> 3)) * 1024 + sw128_offset(h & 7, dc & 7)) =
        make_uint4(lo_w[0], lo_w[1], lo_w[2], lo_w[3]);
  }
  }
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const uint4 v = live ? *reinterpret_cast<const uint4*>(qrow + kLatent + 16 * part + 8 * k) : make_uint4(0, 0, 0, 0);
    *reinterpret_cast<uint4*>(sm + kOffQpe + (h >> 3) * kPeRow + (2 * part + k) * 128 + (h & 7) * 16) = v;
  }
}

// ---------------------------------------------------------------------------
// Softmax warps (0..7) and the per-piece epilogue
// ---------------------------------------------------------------------------
__device__ void softmax(uint8_t* sm, Misc& ms, uint32_t tmem, const Sched& sc, int head_base, int heads_here,
                        int warp, int lane, float c_log2, const DecodeArgs& a) {
  const int tid = threadIdx.x;
  const int q = warp & 3;                  // TMEM lane quadrant
  const int hf = warp >> 2;                // heads 32 hf .. 32 hf + 31
  const int st = 32 * q + lane;            // softmax token
  const uint32_t lane_base = static_cast<uint32_t>(32 * q) << 16;

  float l_part[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) l_part[j] = 0.f;
  int sigma_prev = 0;
  Cursor cur;
  cursor_start(a, sc, cur);

  for (int tile = 0; tile < sc.count; ++tile, cursor_next(a, cur)) {
    const uint32_t par = static_cast<uint32_t>(tile & 1);
    const bool first = cursor_first(cur);
    if (tile > 0 && first) {
      // a new sequence: its Q'' replaces the previous one (whose last QK is
      // complete: its S was read), then the QK issuer may continue
      build_q(sm, ms, a, cur.b, head_base, heads_here, c_log2);
      fence_proxy_async_smem();
      fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ms.mb_qready);
      named_bar(kBarSoftmax, kSoftmaxThreads);  // ac and R of the new sequence are visible
    }
    // V''(j) written (for sigma of the tile), QK(j) complete
    bool ok = warp_wait(&ms.mb_vfull[tile & 1], static_cast<uint32_t>((tile >> 1) & 1), ms, a, 1, lane) &&
              warp_wait(&ms.mb_sfull, par, ms, a, 1, lane);
    fence_after_sync();
    float t[32];
    if (ok) {
      uint32_t s_hi[32], s_lo[32];
      tmem_ld32(tmem + lane_base + kColS + 32 * hf, s_hi);
      tmem_ld32(tmem + lane_base + kColS + 64 + 32 * hf, s_lo);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 32; ++j) t[j] = __uint_as_float(s_hi[j]) + __uint_as_float(s_lo[j]);
      uint32_t s_pe[32];
      tmem_ld32(tmem + lane_base + kColSpe + 32 * hf, s_pe);
      tmem_ld_wait();
      fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ms.mb_sfree);
      const int sigma = ms.sig[tile & 1];
      const float sig = __uint_as_float(static_cast<uint32_t>(min(max(sigma + 127, 1), 254)) << 23);
      const bool tvalid = st < cursor_valid(cur);
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        const float4 ac4 = *reinterpret_cast<const float4*>(&ms.ac[32 * hf + j]);
        const float4 r4 = *reinterpret_cast<const float4*>(&ms.R[32 * hf + j]);
        const float acv[4] = {ac4.x, ac4.y, ac4.z, ac4.w};
        const float rv[4] = {r4.x, r4.y, r4.z, r4.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float base = fmaf(__uint_as_float(s_pe[j + u]), c_log2, -rv[u]);
          t[j + u] = tvalid ? fmaf(t[j + u], acv[u] * sig, base) : -CUDART_INF_F;
        }
      }
      // PV(j-1) must be complete before O is rescaled or read, or P'' is overwritten
      if (tile > 0)
        ok = warp_wait(&ms.mb_pvdone[(tile - 1) & 1], static_cast<uint32_t>(((tile - 1) >> 1) & 1), ms, a, 2, lane);
    }
    // rescale event: a piece's first tile, a score above R + 8.5, or a new sigma.
    // One barrier ORs "event or failure"; only when it is raised does a second
    // one tell a failure (leave the loop) from an event.
    float tmaxv = -CUDART_INF_F;
#pragma unroll
    for (int j = 0; j < 32; ++j) tmaxv = fmaxf(tmaxv, t[j]);
    const int sigma_cur = ms.sig[tile & 1];
    const bool need =
        bar_or(kBarSoftmax, kSoftmaxThreads, !ok || first || tmaxv > 8.5f || sigma_cur != sigma_prev);
    if (need && bar_or(kBarSoftmax, kSoftmaxThreads, !ok)) break;
    fence_after_sync();
    if (need) {
      float v[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = t[j];
      ms.red[q][32 * hf + lane] = warp_transpose_reduce<true>(v, lane);  // tile max of x - R_old
      named_bar(kBarSoftmax, kSoftmaxThreads);
      if (tid < kNH) {
        const float tm = fmaxf(fmaxf(ms.red[0][tid], ms.red[1][tid]), fmaxf(ms.red[2][tid], ms.red[3][tid]));
        // raise R so that this tile's max maps to 2^4 (only raise; a piece's first tile sets it)
        const float shift = first ? tm - 4.0f : fmaxf(tm - 4.0f, 0.0f);
        const float dshift = fmaxf(shift, -1e30f);
        ms.R[tid] += dshift;
        ms.beta[tid] = first ? 1.0f : ex2(-dshift);
        ms.alpha[tid] = first ? 1.0f : ex2(-dshift + static_cast<float>(sigma_prev - sigma_cur));
        ms.red[0][tid] = dshift;  // reused below as the per-head shift of t
      }
      named_bar(kBarSoftmax, kSoftmaxThreads);
#pragma unroll
      for (int j = 0; j < 32; ++j) t[j] -= ms.red[0][32 * hf + j];
      if (!first) {
#pragma unroll
        for (int j = 0; j < 32; ++j) l_part[j] *= ms.beta[32 * hf + j];
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
            for (int j = 0; j < 32; ++j) vv[j] = __float_as_uint(__uint_as_float(vv[j]) * ms.alpha[32 * hh + j]);
            tmem_st32(ta, vv);
          }
        }
        tmem_st_wait();
      }
      // every thread has read red[0] and alpha before the next event overwrites them
      named_bar(kBarSoftmax, kSoftmaxThreads);
    }
    sigma_prev = sigma_cur;

    // ---- P'' = exp2(t) as e4m3 hi + residual, into the MN-major B operands ----
    {
      uint32_t pw[8], pl[8];
#pragma unroll
      for (int j = 0; j < 32; j += 2) {
        const float p0 = ex2(t[j]);
        const float p1 = ex2(t[j + 1]);
        l_part[j] += p0;
        l_part[j + 1] += p1;
        uint16_t h8, l8;
        split_e4m3x2(p0, p1, h8, l8);
        if ((j & 2) == 0) {
          pw[j / 4] = h8;
          pl[j / 4] = l8;
        } else {
          pw[j / 4] |= static_cast<uint32_t>(h8) << 16;
          pl[j / 4] |= static_cast<uint32_t>(l8) << 16;
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
    __syncwarp();
    if (lane == 0) mbar_arrive(&ms.mb_pfull);

    if (!cursor_last(cur)) continue;
    // ---------------- epilogue of the piece ----------------
    const bool done = warp_wait(&ms.mb_pvdone[tile & 1], static_cast<uint32_t>((tile >> 1) & 1), ms, a, 4, lane);
    if (bar_or(kBarSoftmax, kSoftmaxThreads, !done)) break;
    fence_after_sync();
    {
      const float s = warp_transpose_reduce<false>(l_part, lane);
      ms.red[q][32 * hf + lane] = s;
    }
#pragma unroll
    for (int j = 0; j < 32; ++j) l_part[j] = 0.f;
    // the piece covers its whole sequence -> final output; otherwise a partial in its slot
    const bool direct = a.balanced ? (cur.piece_begin == 0 && cur.piece_end == cursor_tiles(cur))
                                   : a.num_splits == 1;
    const int64_t slot = a.balanced ? static_cast<int64_t>(cur.b) + blockIdx.x
                                    : static_cast<int64_t>(cur.b) * a.num_splits + blockIdx.x;
    named_bar(kBarSoftmax, kSoftmaxThreads);
    if (tid < kNH) {
      const float l = ms.red[0][tid] + ms.red[1][tid] + ms.red[2][tid] + ms.red[3][tid];
      // output factor 2^sigma / l per head (alpha is free again)
      ms.alpha[tid] = l > 0.f ? exp2f(static_cast<float>(sigma_prev)) / l : 0.f;
      if (!direct && tid < heads_here)
        a.partial_lse[slot * a.num_heads + head_base + tid] = (ms.R[tid] + __log2f(l)) * kLn2;
    }
    if (a.balanced && tid == 0 && cur.piece_begin == 0) {
      // this CTA holds the sequence's first tile: record its CTA span for the merge
      const int last_cta = cta_of_tile(cur.seq_pos + cursor_tiles(cur) - 1, sc, gridDim.x);
      a.seq_meta[cur.b] = make_int2(blockIdx.x, last_cta);
    }
    named_bar(kBarSoftmax, kSoftmaxThreads);
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
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int h = 32 * hh + j;
          if (h < heads_here) {
            const float val = __uint_as_float(vv[j]) * ms.alpha[h];
            const int hq = head_base + h;
            if (direct)
              a.o[cur.b * a.o_stride_b + hq * a.o_stride_h + d] = __float2bfloat16_rn(val);
            else
              a.partial_o[(slot * a.num_heads + hq) * kLatent + d] = __float2bfloat16_rn(val);
          }
        }
      }
    }
    // O and alpha are read before the next piece's PV / rescale touch them
    fence_before_sync();
    named_bar(kBarSoftmax, kSoftmaxThreads);
  }
}

__global__ void __launch_bounds__(kThreadsTC, 1) mla_decode_tc_kernel(const __grid_constant__ DecodeArgs a) {
  uint8_t* sm = smem_base();
  Misc& ms = *reinterpret_cast<Misc*>(sm + kOffMisc);
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int head_base = blockIdx.z * kNH;
  const int heads_here = min(kNH, a.num_heads - head_base);

  Sched sc;
  if (a.balanced) {
    balanced_schedule<kThreadsTC>(a, ms.sched, sc);
    if (sc.count == 0) {
      // An empty run (fewer tiles than CTAs) can sit inside the CTA span of
      // the sequence at its position; its slot of that sequence carries no weight.
      if (sc.pos0 < sc.total && tid < heads_here)
        a.partial_lse[(static_cast<int64_t>(sc.b0) + blockIdx.x) * a.num_heads + head_base + tid] = -CUDART_INF_F;
      return;  // (uniform: every thread read the same count)
    }
  } else {
    const int b = blockIdx.y, tiles = seq_tiles_of(a, b);
    const int per_split = (tiles + a.num_splits - 1) / a.num_splits;
    sc.b0 = b;
    sc.off0 = blockIdx.x * per_split;
    sc.count = max(0, min(per_split, tiles - sc.off0));
    sc.pos0 = 0;
    sc.total = 0;
    sc.per_seq = sc.split_tiles = sc.seq_tiles = 0;
    if (sc.count == 0) {
      // nothing to attend to: zeros (one split) or a split that carries no weight
      if (a.num_splits == 1) {
        for (int i = tid; i < heads_here * (kLatent / 2); i += kThreadsTC) {
          const int h = i / (kLatent / 2), d = (i % (kLatent / 2)) * 2;
          *reinterpret_cast<uint32_t*>(a.o + b * a.o_stride_b + (head_base + h) * a.o_stride_h + d) = 0u;
        }
      } else if (tid < heads_here) {
        a.partial_lse[(static_cast<int64_t>(b) * a.num_splits + blockIdx.x) * a.num_heads + head_base + tid] =
            -CUDART_INF_F;
      }
      return;
    }
  }
  const float c_log2 = a.sm_scale * kLog2e;

  // ---------------- setup: TMEM, barriers, Q'' of the first sequence ----------------
  // Register budgets first (the loaders' increase waits for the issuers' decrease),
  // then each role sets up its part and meets the others at the setup barrier.
  if (warp >= kWarpQK) {
    setmaxnreg_dec<kIssuerRegs>();
    if (warp == kWarpQK) {
      tmem_alloc(&ms.tmem_base, kTmemCols);
      if (lane == 0) {
        mbar_init(&ms.mb_vfull[0], 4);
        mbar_init(&ms.mb_vfull[1], 4);
        mbar_init(&ms.mb_pvdone[0], kPvIssuers);
        mbar_init(&ms.mb_pvdone[1], kPvIssuers);
        mbar_init(&ms.mb_sfull, 1);
        mbar_init(&ms.mb_sfree, kSoftmaxWarps);
        mbar_init(&ms.mb_pfull, kSoftmaxWarps);
        mbar_init(&ms.mb_drain, 1 + kPvIssuers);
        mbar_init(&ms.mb_qready, kSoftmaxWarps);
        fence_mbar_init();
        ms.abort_flag = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) ms.tile_smax[i] = 0;
      }
    }
    setup_barrier();
    const uint32_t tmem = ms.tmem_base;
    const bool issuer = warp < kWarpPV0 + kPvIssuers;
    if (warp == kWarpQK)
      qk_issuer(sm, ms, tmem, sc, lane, a);
    else if (issuer)
      pv_issuer(sm, ms, tmem, sc, lane, warp - kWarpPV0, a);
    // drain: arrives once every MMA this thread issued has completed
    if (issuer && lane == 0) mma_commit(&ms.mb_drain);
    __syncwarp();
  } else if (warp >= kLoaderWarp0) {
    setmaxnreg_inc<kLoaderRegs>();
    loader(sm, ms, sc, head_base, heads_here, warp - kLoaderWarp0, lane, a);
  } else {
    prefetch_q(a, sc.b0, head_base, heads_here, tid, kSoftmaxThreads);
    build_q(sm, ms, a, sc.b0, head_base, heads_here, c_log2);
    fence_proxy_async_smem();
    setup_barrier();
    softmax(sm, ms, ms.tmem_base, sc, head_base, heads_here, warp, lane, c_log2, a);
  }

  fence_before_sync();
  __syncthreads();  // every TMEM read is done
  if (warp == kWarpQK) {
    if (lane == 0 && !mbar_wait_bounded(&ms.mb_drain, 0, kPollLimit)) record_status(a, 128);
    __syncwarp();
    fence_after_sync();
    tmem_dealloc(ms.tmem_base, kTmemCols);
  }
}

}  // namespace

cudaError_t launch_decode_tc(const DecodeArgs& a, cudaStream_t stream) {
  cudaError_t e = cudaFuncSetAttribute(mla_decode_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemTC);
  if (e != cudaSuccess) return e;
  const int head_blocks = (a.num_heads + kNH - 1) / kNH;
  const dim3 grid = a.balanced ? dim3(a.num_splits, 1, head_blocks) : dim3(a.num_splits, a.batch, head_blocks);
  mla_decode_tc_kernel<<<grid, kThreadsTC, kSmemTC, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace kimi
