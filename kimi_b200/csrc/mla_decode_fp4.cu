// Split-K absorbed-MLA decode over the MXFP4 paged cache, sm_100a: Q K^T as
// block-scaled e2m1 tensor-core MMAs straight from the cache bytes.
//
// Math (paths inside ianye23301/kimi): the archive stage-1 kernel
// `_mla_decode_split_kv` (archive/mla-mxfp4-dead-end/mla_decode_mxfp4_v5.py:136-261),
// which likewise computes Q K^T with an MXFP4 x MXFP4 block-scaled dot
// (`tl.dot_scaled(q_fp4, q_scale, "e2m1", k_u8, k_scale, "e2m1")`), under the
// contract of `reference_mla_decode` (tests/test_triton_mla_decode.py:12-62):
//   S = q_nope . k_nope + q_pe . k_pe,  P = softmax(S * sm_scale),  O = P . k_nope.
//
// Scheduling is that of the other tensor-core kernel (decode_common.cuh): one
// CTA = up to 64 heads over a run of 128-token tiles (two pages), tokens on
// the MMA's M dimension and heads on N.
//   * Q K^T: the tile's nibbles and e8m0 scales are loaded by TMA as they lie
//     in the cache (nibbles as two 128-byte-swizzled K-major column blocks of
//     128 rows; scales row by row) and consumed by tcgen05.mma kind::mxf4 with
//     the scales in TMEM.  q_nope is written as three block-scaled e2m1 terms
//     (q = t0 + t1 + t2, each term the e2m1 rounding of the remaining residual
//     with its own e8m0 scale per 32 elements), stacked as one N = 192 B
//     operand; the terms land in S column groups 0, 64 and 128 and are summed
//     by the softmax.  Three terms give bf16-level scores; the reference
//     quantises q to a single e2m1 term.  q_pe . k_pe is a bf16 MMA with k_pe
//     (TMA-loaded) and q_pe in shared memory, accumulated into column group 0.
//   * P V: P'' = exp2(x - R_h) as two e4m3 terms (hi + residual) against
//     V'' = e2m1 * 2^(scale - 127 - sigma) written as e5m2 (exact) by the
//     loader warps from the TMA-loaded nibbles; two PV MMAs per K step into
//     one accumulator (one e4m3 term alone costs ~2% relative error on short
//     contexts).  R_h (per-head offset, kept in [max - 8.5, max - 4] of the
//     running max) and sigma (per-tile reference exponent) are raised lazily;
//     O is rescaled in TMEM when either changes.
//   * Shared memory (228 KB): two stages of raw nibbles + scales, one k_pe
//     buffer, a two-slot V'' ring by latent half (the loaders fill half h of
//     tile j as soon as PV has finished half h of tile j - 1), Q, q_pe and P''.
//   * TMEM (512 columns): S [0,192), scale factors of A (two buffers, 16
//     columns each) [192,224), of B [224,256), O^T [256,512) as four 128-row
//     latent chunks of 64 head columns.
//
// Warp roles (20 warps, 640 threads):
//   warps 0-7   softmax: Q terms of each piece, S(j) -> P''(j), O rescales,
//               the epilogue;
//   warps 8-15  loaders: tile maximum scale (sigma), A scale factors to TMEM
//               (warps 8-11, one per TMEM lane quarter), V'' halves;
//   warp 16     allocates TMEM and issues QK(j) (RoPE MMAs first);
//   warps 17-18 issue PV(j), latent half 0 and half 1;
//   warp 19     TMA producer: nibbles + scales two tiles ahead, k_pe one tile
//               ahead.
// Every mbarrier wait is bounded; a wait that gives up sets a shared abort
// word that every other wait polls, each role leaves its loop, the issuers
// drain their MMAs and TMEM is freed as usual.
#include <cstddef>

#include <cuda.h>
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

constexpr int kNHMax = 64;  // heads per CTA of the wide form (the small form has 16)
constexpr int kSoftmaxWarps = 8;
constexpr int kSoftmaxThreads = 32 * kSoftmaxWarps;
constexpr int kLoaderWarp0 = 8;  // warps 8..15
constexpr int kLoaderWarps = 8;
constexpr int kLoaderThreads = 32 * kLoaderWarps;
constexpr int kWarpQK = 16;
constexpr int kWarpPV0 = 17;  // warps 17, 18
constexpr int kWarpTMA = 19;
constexpr int kThreads = 640;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0, kColSfa = 192, kColSfb = 224, kColO = 256;
constexpr uint32_t kPollLimit = 100000;  // polls of up to kWaitSleepNs each: about 2 s

// Register budgets: 640 threads launch with 96 registers each (61440); the
// softmax warpgroups take 144, the loaders give back down to 64, the
// issuer/producer warpgroup to 56.
constexpr uint32_t kLaunchRegs = 96;
constexpr uint32_t kSoftmaxRegs = 144, kLoaderRegs = 64, kIssuerRegs = 56;
static_assert(kSoftmaxThreads * kSoftmaxRegs + kLoaderThreads * kLoaderRegs + 128 * kIssuerRegs <=
                  kThreads * kLaunchRegs,
              "register split");

// Named barriers (0 is __syncthreads)
constexpr int kBarSoftmax = 1;
constexpr int kBarLoader = 2;

// Shared memory (bytes).  Swizzled operands use 128B-swizzled atoms of 8 rows
// x 128 bytes (1 KB), rows of a column block 128 bytes apart.
constexpr int kNibBlock = 128 * 128;        // 128 token rows x 128 nibble bytes (K 0..255 or 256..511)
constexpr int kNibStage = 2 * kNibBlock;    // one tile's nibbles
constexpr int kOffNib = 0;                  // two stages
constexpr int kScStage = 128 * kScaleBytes; // one tile's e8m0 scales, token-major
constexpr int kScSlots = 4;                 // scale ring: tiles j .. j + 3
constexpr int kOffSc = kOffNib + 2 * kNibStage;
constexpr int kOffKpe = kOffSc + kScSlots * kScStage;  // k_pe: 128 rows x 128 bytes
constexpr int kVCol = 16384;                // V'': one 128-latent column (16 atoms of 8 tokens)
constexpr int kOffV = kOffKpe + 128 * 128;  // one tile, four latent columns; ring of 4 token quarters
constexpr int kOffQ = kOffV + 4 * kVCol;    // Q terms, then q_pe, P'' and (small form) the epilogue stage
static_assert(kOffKpe % 1024 == 0 && kOffV % 1024 == 0 && kOffQ % 1024 == 0, "swizzled operands start on 1 KB boundaries");

// The part of the layout that depends on the heads per CTA, NH = 64 (wide
// form) or 16 (small form, calls with at most 16 heads).
template <int NH>
struct Form {
  static constexpr int kQRows = 3 * NH;               // B rows of the latent QK MMA: three Q terms
  static constexpr int kQBlock = kQRows * 128;        // Q terms: kQRows rows x 128 bytes per K column block
  static constexpr int kOffQpe = kOffQ + 2 * kQBlock;  // q_pe bf16: NH rows x 128 bytes
  // P'' hi e4m3, MN-major cores: per 8-token group NH / 16 core matrices of
  // 8 tokens x 16 head bytes; then P'' lo (residual) in the same layout
  static constexpr int kPRow = NH / 16 * 128;
  static constexpr int kPBytes = 16 * kPRow;          // 128 tokens
  static constexpr int kOffP = kOffQpe + NH * 128;
  static constexpr int kOffPlo = kOffP + kPBytes;
  // epilogue transposes: 2 KB per softmax warp, in P'' (wide form; its last
  // PV is complete) or in a stage of their own (small form)
  static constexpr int kOffStage = NH == 64 ? kOffP : kOffPlo + kPBytes;
  static constexpr int kOffMisc = NH == 64 ? kOffPlo + kPBytes : kOffStage + kSoftmaxWarps * 2048;
  // TMEM: S as three term column groups of NH, O as four 128-latent chunks of
  // NH head columns (wide: hi and lo accumulate together) or 2 NH (small: hi
  // then lo columns, one N = 32 MMA per chunk and K step)
  static constexpr uint32_t kOChunkCols = NH == 64 ? 64 : 2 * NH;
  static_assert(kOffQpe % 1024 == 0 && kOffP % 1024 == 0, "swizzled operands start on 1 KB boundaries");
  static_assert(kOffP + kQRows * kScaleBytes <= kOffMisc, "Q scale staging fits in P''");
  static_assert(2 * kQBlock == q_term_bytes(NH) && NH * 128 == q_pe_bytes(NH), "Q image layout");
};

struct Misc {
  uint64_t mb_rawfull[2];    // nibble stage s landed (producer expect_tx + TMA bytes)
  uint64_t mb_qkdone[2];     // stage s: QK of its tile complete (commit)
  uint64_t mb_nibread[2];    // stage s: the loader warps are done with its tile (8 arrivals)
  uint64_t mb_scfull[4];     // scale ring slot r landed (producer expect_tx + TMA bytes)
  uint64_t mb_sfafull[2];    // A scale-factor buffer s written (4 loader warps)
  uint64_t mb_vfull[4];      // V'' token quarter k of the current tile written (8 loader warps)
  uint64_t mb_pvq[4];        // PV of token quarter k complete (one commit per PV issuer)
  uint64_t mb_tiledone[2];   // all of PV(j) complete, slot j % 2 (one commit per PV issuer)
  uint64_t mb_sigready[4];   // sigma of tile j published in sig[j % 4] (1 arrival)
  uint64_t mb_kpefull;       // k_pe of the next tile landed
  uint64_t mb_kpefree;       // RoPE MMAs of the tile in the k_pe buffer complete (commit)
  uint64_t mb_sfull;         // QK(j) complete (commit)
  uint64_t mb_sfree;         // S(j) read out of TMEM (8 softmax warps)
  uint64_t mb_pfull[4];      // P''(j) token quarter k written, O rescaled (2 softmax warps)
  uint64_t mb_qready;        // Q terms, their scales and q_pe of a piece written (8 softmax warps)
  uint64_t mb_qload;         // Q image of a piece landed (bulk copy; Q images in the workspace only)
  uint64_t mb_drain;         // each issuer's last commit (3 arrivals)
  SchedScratch sched;        // balanced mode: block-scan scratch
  uint32_t tmem_base;
  int abort_flag;
  int tile_smax[4];          // max e8m0 byte of tile j in slot j % 4 (reset two tiles ahead)
  int sig[4];                // reference exponent sigma of tile j in slot j % 4
  alignas(16) float R[kNHMax];  // per-head exp2 offset, log2 units (read as float4)
  float alpha[kNHMax];          // O rescale factors of the current event
  float beta[kNHMax];           // softmax-sum rescale factors of the current event
  float red[4][kNHMax];         // cross-warp reduction scratch
};
template <int NH>
constexpr int smem_bytes() { return Form<NH>::kOffMisc + static_cast<int>(sizeof(Misc)); }
static_assert(smem_bytes<64>() <= 232448 && smem_bytes<16>() <= 232448, "shared memory budget");
static_assert(Form<64>::kOffMisc % 16 == 0 && Form<16>::kOffMisc % 16 == 0 && offsetof(Misc, R) % 16 == 0,
              "per-head arrays are read with 16-byte loads");

__device__ __forceinline__ uint8_t* smem_base() {
  extern __shared__ __align__(1024) uint8_t dyn_smem[];
  return dyn_smem;
}

// The grid's x index interleaves the head blocks fastest: CTA x is head
// block x % head_blocks of schedule CTA (split) x / head_blocks, so the CTAs
// that read the same tiles for different head blocks run side by side and
// the second read is an L2 hit.
template <int NH>
__device__ __forceinline__ int head_blocks(const DecodeArgs& a) { return (a.num_heads + NH - 1) / NH; }
template <int NH>
__device__ __forceinline__ int cta_index(const DecodeArgs& a) { return static_cast<int>(blockIdx.x) / head_blocks<NH>(a); }
template <int NH>
__device__ __forceinline__ int cta_count(const DecodeArgs& a) { return static_cast<int>(gridDim.x) / head_blocks<NH>(a); }
template <int NH>
__device__ __forceinline__ int head_block(const DecodeArgs& a) { return static_cast<int>(blockIdx.x) % head_blocks<NH>(a); }

__device__ __forceinline__ void record_status(const DecodeArgs& a, int bits) {
  if (a.status) atomicOr(a.status, bits);
}

// Per-thread bounded wait: one plain probe first (a phase that has already
// completed costs only that), then polls with a suspend-time hint for at most
// the call's timeout_ns; on give-up records the failure and raises the abort
// word.  (The drain waits before exit keep their fixed bound, kPollLimit
// polls, whatever the call's timeout: copies and MMAs already issued must
// land before the CTA leaves.)
__device__ __forceinline__ bool wait_phase(uint64_t* mb, uint32_t parity, Misc& ms, const DecodeArgs& a, int bit) {
  if (mbar_try_wait(mb, parity)) return true;
  if (mbar_wait_timed(mb, parity, a.timeout_ns, &ms.abort_flag)) return true;
  if (atomicExch(&ms.abort_flag, 1) == 0) record_status(a, bit);
  return false;
}

// Warp-uniform bounded wait.  Every lane probes (one warp-wide instruction per
// poll) and a vote makes the verdict uniform: an elected lane polling inside a
// divergent branch and broadcasting its verdict costs several hundred cycles
// per call even when the phase is already complete.
__device__ __forceinline__ bool warp_wait(uint64_t* mb, uint32_t parity, Misc& ms, const DecodeArgs& a, int bit,
                                          int lane) {
  if (__all_sync(0xffffffffu, mbar_try_wait(mb, parity))) return true;
  const bool ok = __all_sync(0xffffffffu, mbar_wait_timed(mb, parity, a.timeout_ns, &ms.abort_flag));
  if (!ok && lane == 0 && atomicExch(&ms.abort_flag, 1) == 0) record_status(a, bit);
  return ok;
}

// Page rows (y coordinates of the cache tensor maps) of the two pages of the
// cursor's tile: -1 for a slot past the sequence's pages (nothing loaded).  A
// page id outside [0, num_pages) maps to a row outside the tensor, which TMA
// fills with zeros, and (when `report`) sets kStatusBadPage.
__device__ __forceinline__ void tile_rows(const DecodeArgs& a, const Cursor& c, int (&y)[2], bool report = false) {
#pragma unroll
  for (int slot = 0; slot < 2; ++slot) {
    const int p = 2 * c.tile + slot;
    const bool in_range = p < c.n_pages;
    const int pid = ldg_s32_or(a.kv_indices + c.page_lo + (in_range ? p : 0), in_range, -1);
    const bool good = pid >= 0 && pid < a.num_pages;
    if (report && in_range && !good) record_status(a, kStatusBadPage);
    y[slot] = !in_range ? -1 : good ? pid * kPageSize : -kPageSize;
  }
}

// ---------------------------------------------------------------------------
// TMA producer (warp 19, lane 0)
// ---------------------------------------------------------------------------
// Nibbles go to a two-stage ring (tile j waits for QK(j - 2) and the loaders'
// V'' of tile j - 2), scales to a four-slot ring up to two tiles ahead of the
// nibbles (the loaders need tile j + 1's scales while converting tile j), k_pe
// to one buffer (tile j waits for the RoPE MMAs of tile j - 1).  Tile 0's
// nibbles, scales and k_pe are issued before anything else.  There is no L2
// prefetch ahead of the TMA loads: measured at config 2, dropping it (and
// with it a third of this role's code) made stage 1 4% faster.
__device__ void producer(uint8_t* sm, Misc& ms, const Sched& sc, const DecodeArgs& a, const CacheMaps& maps) {
  prefetch_tensormap(&maps.kv);
  prefetch_tensormap(&maps.sc);
  Cursor cur, sc_cur;  // nibbles and k_pe of tile j; the next tile's scales
  cursor_start(a, sc, cur);
  sc_cur = cur;
  int sc_issued = 0;
  auto load_scales = [&]() {  // tile sc_issued -> ring slot sc_issued % 4
    int y[2];
    tile_rows(a, sc_cur, y);
    uint64_t* mb = &ms.mb_scfull[sc_issued % kScSlots];
    const int slots = (y[0] != -1 ? 1 : 0) + (y[1] != -1 ? 1 : 0);
    mbar_arrive_expect_tx(mb, static_cast<uint32_t>(slots * kPageScaleBytes));
#pragma unroll
    for (int slot = 0; slot < 2; ++slot)
      if (y[slot] != -1)
        tma_load_2d(sm + kOffSc + (sc_issued % kScSlots) * kScStage + slot * kPageScaleBytes, &maps.sc, 0, y[slot], mb);
    ++sc_issued;
    cursor_next(a, sc_cur);
  };
  int issued = 0;
  for (int j = 0; j < sc.count; ++j, cursor_next(a, cur)) {
    const int s = j & 1;
    // stage s (and scale slot (j + 2) % 4) were last used by tile j - 2
    if (j >= 2) {
      const uint32_t par = static_cast<uint32_t>(((j - 2) >> 1) & 1);
      bool ok = true;  // (both waits through one copy of the wait code)
#pragma unroll 1
      for (int w = 0; w < 2 && ok; ++w) ok = wait_phase(w == 0 ? &ms.mb_qkdone[s] : &ms.mb_nibread[s], par, ms, a, 256);
      if (!ok) break;
    }
    int y[2];
    tile_rows(a, cur, y, true);
    const int slots = (y[0] != -1 ? 1 : 0) + (y[1] != -1 ? 1 : 0);
    mbar_arrive_expect_tx(&ms.mb_rawfull[s], static_cast<uint32_t>(slots * 2 * 64 * 128));
#pragma unroll
    for (int slot = 0; slot < 2; ++slot) {
      if (y[slot] == -1) continue;
      uint8_t* nib = sm + kOffNib + s * kNibStage + slot * (64 * 128);
      tma_load_2d(nib, &maps.kv, 0, y[slot], &ms.mb_rawfull[s]);
      tma_load_2d(nib + kNibBlock, &maps.kv, 128, y[slot], &ms.mb_rawfull[s]);
    }
    auto load_kpe = [&]() {
      mbar_arrive_expect_tx(&ms.mb_kpefull, static_cast<uint32_t>(slots * 64 * 128));
#pragma unroll
      for (int slot = 0; slot < 2; ++slot) {
        if (y[slot] == -1) continue;
        tma_load_2d(sm + kOffKpe + slot * (64 * 128), &maps.kv, kNibbleBytes, y[slot], &ms.mb_kpefull);
      }
    };
    // scales run up to two tiles ahead of the nibbles (tile 0's right after
    // its nibbles)
    while (sc_issued < min(j + 3, sc.count)) load_scales();
    // k_pe (one buffer): free once the RoPE MMAs of tile j - 1 are complete.
    // Every load kind is issued from one place in the loop: the producer's
    // code is fetched by its sub-partition every tile.
    if (j >= 1 && !wait_phase(&ms.mb_kpefree, static_cast<uint32_t>((j - 1) & 1), ms, a, 256)) break;
    load_kpe();
    issued = j + 1;
  }
  // every load issued has landed before the CTA may exit (normally the
  // consumers have already waited for all of them)
  for (int j = max(0, issued - 2); j < issued; ++j)
    mbar_wait_bounded(&ms.mb_rawfull[j & 1], static_cast<uint32_t>((j >> 1) & 1), kPollLimit);
  if (issued > 0) mbar_wait_bounded(&ms.mb_kpefull, static_cast<uint32_t>((issued - 1) & 1), kPollLimit);
  for (int t = max(0, sc_issued - kScSlots); t < sc_issued; ++t)
    mbar_wait_bounded(&ms.mb_scfull[t % kScSlots], static_cast<uint32_t>((t / kScSlots) & 1), kPollLimit);
}

// ---------------------------------------------------------------------------
// Issuers (warp 16: QK, warps 17-18: PV; lane 0 issues)
// ---------------------------------------------------------------------------
template <int NH>
__device__ void qk_issuer(uint8_t* sm, Misc& ms, uint32_t tmem, const Sched& sc, int lane, const DecodeArgs& a) {
  using F = Form<NH>;
  const uint32_t id_pe = instr_desc(kFmtBF16, kFmtBF16, false, false, 128, NH);
  const uint32_t sQ = smem_addr(sm + kOffQ), sQpe = smem_addr(sm + F::kOffQpe), sKpe = smem_addr(sm + kOffKpe);
  Cursor cur;
  cursor_start(a, sc, cur);
  int pieces = 0;
  for (int j = 0; j < sc.count; ++j, cursor_next(a, cur)) {
    const int s = j & 1;
    const uint32_t use = static_cast<uint32_t>((j >> 1) & 1);
    // QK(j) needs S(j-1) read out of TMEM (single S buffer), the tile's
    // nibbles/scales, its k_pe and A scale factors, and at a piece start that
    // sequence's Q.  The waits go through one copy of the wait code: the
    // kernel is bound by instruction fetch, and each inlined wait adds its
    // bounded slow path to the code every sub-partition runs.
    {
      const bool first = cursor_first(cur);
      const int nw = first ? (a.q_img ? 6 : 5) : 4;
      bool ok = true;
#pragma unroll 1
      for (int w = (j > 0 ? 0 : 1); w < nw && ok; ++w) {
        uint64_t* mb;
        uint32_t par;
        switch (w) {
          case 0: mb = &ms.mb_sfree; par = static_cast<uint32_t>((j - 1) & 1); break;
          case 1: mb = &ms.mb_rawfull[s]; par = use; break;
          case 2: mb = &ms.mb_kpefull; par = static_cast<uint32_t>(j & 1); break;
          case 3: mb = &ms.mb_sfafull[s]; par = use; break;
          case 4: mb = &ms.mb_qready; par = static_cast<uint32_t>(pieces & 1); break;
          default: mb = &ms.mb_qload; par = static_cast<uint32_t>(pieces & 1); break;
        }
        ok = warp_wait(mb, par, ms, a, 16, lane);
      }
      if (!ok) break;
      if (first) ++pieces;
    }
    fence_after_sync();
    if (lane == 0 && NH == 16) {
      // small form: latent first (8 K steps of 64, N = 48: the three terms of
      // 16 heads, the first step starting S), then the RoPE MMAs add
      // k_pe . q_pe^T onto the term-0 columns
      const uint32_t sA = smem_addr(sm + kOffNib + s * kNibStage);
      const uint32_t sfa0 = tmem + kColSfa + 16 * s, sfb0 = tmem + kColSfb;
#pragma unroll 1
      for (int k = 0; k < 8; ++k) {
        const uint32_t koff = (k & 3) * 32;
        const uint32_t byte = 2 * (k & 1);
        const uint32_t sfa = (sfa0 + 4 * (k >> 1)) | (byte << 30);
        const uint32_t sfb = (sfb0 + 8 * (k >> 1)) | (byte << 30);
        const uint64_t da = smem_desc(sA + (k >> 2) * kNibBlock + koff, 16, 1024, kSwizzle128B);
        const uint32_t qb = sQ + (k >> 2) * F::kQBlock + koff;
        mma_mxf4_ss(tmem + kColS, da, smem_desc(qb, 16, 1024, kSwizzle128B), instr_desc_mxf4(F::kQRows, byte, byte),
                    sfa, sfb, k > 0 ? 1u : 0u);
      }
#pragma unroll
      for (int k = 0; k < 4; ++k)
        mma_f16_ss(tmem + kColS, smem_desc(sKpe + 32 * k, 16, 1024, kSwizzle128B),
                   smem_desc(sQpe + 32 * k, 16, 1024, kSwizzle128B), id_pe, 1u);
      mma_commit(&ms.mb_kpefree);
      mma_commit(&ms.mb_sfull);
      mma_commit(&ms.mb_qkdone[s]);
    } else if (lane == 0) {
      // RoPE first (k_pe is single-buffered): S[:, 0:64) = k_pe . q_pe^T
#pragma unroll
      for (int k = 0; k < 4; ++k)
        mma_f16_ss(tmem + kColS, smem_desc(sKpe + 32 * k, 16, 1024, kSwizzle128B),
                   smem_desc(sQpe + 32 * k, 16, 1024, kSwizzle128B), id_pe, k > 0 ? 1u : 0u);
      mma_commit(&ms.mb_kpefree);
      // latent: 8 K steps of 64; the first adds onto the RoPE columns (term 0)
      // and starts the columns of terms 1 and 2
      const uint32_t sA = smem_addr(sm + kOffNib + s * kNibStage);
      const uint32_t sfa0 = tmem + kColSfa + 16 * s, sfb0 = tmem + kColSfb;
#pragma unroll 1
      for (int k = 0; k < 8; ++k) {
        const uint32_t koff = (k & 3) * 32;
        const uint32_t byte = 2 * (k & 1);
        const uint32_t sfa = (sfa0 + 4 * (k >> 1)) | (byte << 30);
        const uint32_t sfb = (sfb0 + 8 * (k >> 1)) | (byte << 30);
        const uint64_t da = smem_desc(sA + (k >> 2) * kNibBlock + koff, 16, 1024, kSwizzle128B);
        const uint32_t qb = sQ + (k >> 2) * F::kQBlock + koff;
        if (k == 0) {
          mma_mxf4_ss(tmem + kColS, da, smem_desc(qb, 16, 1024, kSwizzle128B), instr_desc_mxf4(64, byte, byte),
                      sfa, sfb, 1u);
          mma_mxf4_ss(tmem + kColS + 64, da, smem_desc(qb + 8 * 1024, 16, 1024, kSwizzle128B),
                      instr_desc_mxf4(128, byte, byte), sfa, (sfb0 + 2) | (byte << 30), 0u);
        } else {
          mma_mxf4_ss(tmem + kColS, da, smem_desc(qb, 16, 1024, kSwizzle128B), instr_desc_mxf4(192, byte, byte),
                      sfa, sfb, 1u);
        }
      }
      mma_commit(&ms.mb_sfull);
      mma_commit(&ms.mb_qkdone[s]);
    }
    __syncwarp();
  }
}

// PV issuer h owns latent half h (chunks 2h, 2h + 1) and walks the tile's
// four token quarters as the loaders finish them.
// Small form: P'' hi and lo are one N = 32 B operand (the lo cores one
// P'' buffer further on), so each chunk and K step is one MMA into 32 columns
// of O (hi heads, then lo heads) instead of two into the same 64.
template <int NH>
__device__ void pv_issuer(uint8_t* sm, Misc& ms, uint32_t tmem, const Sched& sc, int lane, int h,
                          const DecodeArgs& a) {
  using F = Form<NH>;
  const uint32_t id_pv = instr_desc(kFmtE5M2, kFmtE4M3, true, true, 128, NH == 64 ? 64 : 2 * NH);
  const uint32_t sP = smem_addr(sm + F::kOffP), sPlo = smem_addr(sm + F::kOffPlo);
  const uint32_t sV = smem_addr(sm + kOffV + 2 * h * kVCol);
  Cursor cur;
  cursor_start(a, sc, cur);
  for (int j = 0; j < sc.count; ++j, cursor_next(a, cur)) {
    const uint32_t par = static_cast<uint32_t>(j & 1);
    const bool fresh = cursor_first(cur);  // the piece's first PV starts the accumulator
    bool ok = true;
#pragma unroll 1
    for (int k = 0; k < 4 && ok; ++k) {
      ok = warp_wait(&ms.mb_pfull[k], par, ms, a, 32, lane) && warp_wait(&ms.mb_vfull[k], par, ms, a, 32, lane);
      if (!ok) break;
      fence_after_sync();
      if (lane == 0 && NH == 16) {
        const uint64_t pb = smem_desc(sP + k * 4 * F::kPRow, F::kPRow, F::kPBytes);
#pragma unroll
        for (int c = 0; c < 2; ++c)
          mma_f8f6f4_ss(tmem + kColO + F::kOChunkCols * (2 * h + c),
                        smem_desc(sV + c * kVCol + k * 4096, kVCol, 1024, kSwizzle128B), pb, id_pv,
                        (fresh && k == 0) ? 0u : 1u);
        mma_commit(&ms.mb_pvq[k]);
      } else if (lane == 0) {
        const uint64_t phi = smem_desc(sP + k * 4 * F::kPRow, F::kPRow, 128);
        const uint64_t plo = smem_desc(sPlo + k * 4 * F::kPRow, F::kPRow, 128);
#pragma unroll
        for (int c = 0; c < 2; ++c)
          mma_f8f6f4_ss(tmem + kColO + 64 * (2 * h + c),
                        smem_desc(sV + c * kVCol + k * 4096, kVCol, 1024, kSwizzle128B), phi, id_pv,
                        (fresh && k == 0) ? 0u : 1u);
#pragma unroll
        for (int c = 0; c < 2; ++c)
          mma_f8f6f4_ss(tmem + kColO + 64 * (2 * h + c),
                        smem_desc(sV + c * kVCol + k * 4096, kVCol, 1024, kSwizzle128B), plo, id_pv, 1u);
        mma_commit(&ms.mb_pvq[k]);
      }
      __syncwarp();
    }
    if (!ok) break;
    if (lane == 0) mma_commit(&ms.mb_tiledone[j & 1]);  // this half of all of PV(j)
    __syncwarp();
  }
}

// ---------------------------------------------------------------------------
// Loaders (warps 8..15)
// ---------------------------------------------------------------------------
// Per tile j: first the reference exponent sigma and the A scale factors of
// tile j + 1 (QK(j + 1) needs them while PV(j) still runs), then V''(j) one
// token quarter at a time, each as soon as PV(j - 1) has finished reading that
// quarter of the ring.
__device__ void loader(uint8_t* sm, Misc& ms, uint32_t tmem, const Sched& sc, int warp, int lane,
                       const DecodeArgs& a) {
  const int lt = threadIdx.x - 32 * kLoaderWarp0;  // 0..255
  const int lw = lt >> 5;
  const uint32_t lane_base = static_cast<uint32_t>(32 * (warp & 3)) << 16;
  int prev_sigma = 0;
  // sigma and A scale factors of tile tt (cursor c); false when the CTA aborts
  auto scales = [&](int tt, const Cursor& c) -> bool {
    const int r = tt % kScSlots;
    const uint8_t* scb = sm + kOffSc + r * kScStage;
    const bool ok = warp_wait(&ms.mb_scfull[r], static_cast<uint32_t>((tt / kScSlots) & 1), ms, a, 64, lane);
    const int nvalid = cursor_valid(c);
    // tile maximum of the e8m0 bytes of valid tokens -> reference exponent
    uint32_t my_max = 0u;
    if (ok && (lt >> 1) < nvalid) {
      const uint2 w = *reinterpret_cast<const uint2*>(scb + (lt >> 1) * kScaleBytes + 8 * (lt & 1));
      const uint32_t m4 = __vmaxu4(w.x, w.y);
      my_max = max(max(m4 & 0xFFu, (m4 >> 8) & 0xFFu), max((m4 >> 16) & 0xFFu, m4 >> 24));
    }
    my_max = __reduce_max_sync(0xffffffffu, my_max);
    if (lane == 0) atomicMax(&ms.tile_smax[tt & 3], static_cast<int>(my_max));
    if (bar_or(kBarLoader, kLoaderThreads, !ok)) return false;
    const int smax = ms.tile_smax[tt & 3];
    int sigma;
    if (cursor_first(c)) {
      sigma = smax - 127 - 8;  // tile max maps to <= 6 * 2^8 in V''
    } else {
      const int kmax = smax - 127 - prev_sigma;
      sigma = (kmax > 13 || kmax < -4) ? smax - 127 - 8 : prev_sigma;
    }
    prev_sigma = sigma;
    if (lt == 0) {
      ms.tile_smax[(tt + 2) & 3] = 0;
      ms.sig[tt & 3] = sigma;
      mbar_arrive(&ms.mb_sigready[tt & 3]);
    }
    // A scale factors -> TMEM buffer tt % 2 (last read by QK(tt - 2)); warp
    // 8 + q writes TMEM lane quarter q: column 4 k4 + r1 of lane r0 holds the
    // scale word k4 of token r0 + 32 r1.
    if (lw < 4) {
      const int s = tt & 1;
      const bool free_ok =
          tt < 2 || warp_wait(&ms.mb_qkdone[s], static_cast<uint32_t>(((tt - 2) >> 1) & 1), ms, a, 64, lane);
      if (free_ok) {
        uint32_t v[16];  // word k4 of token lane + 32 r1 in v[4 k4 + r1]
#pragma unroll
        for (int r1 = 0; r1 < 4; ++r1) {
          const uint4 w = *reinterpret_cast<const uint4*>(scb + (lane + 32 * r1) * kScaleBytes);
          v[r1] = w.x;
          v[4 + r1] = w.y;
          v[8 + r1] = w.z;
          v[12 + r1] = w.w;
        }
        tmem_st16(tmem + lane_base + kColSfa + 16 * s, v);
        tmem_st_wait();
      }
      fence_before_sync();
      __syncwarp();
      if (lane == 0 && free_ok) mbar_arrive(&ms.mb_sfafull[s]);
    }
    return true;
  };

  Cursor cur, nxt;  // tile j (V''), tile j + 1 (scales)
  cursor_start(a, sc, cur);
  nxt = cur;
  // Iteration j = -1 only prepares tile 0's scales: scales() is inlined
  // once (the loaders' code is fetched by every sub-partition every tile).
  int sigma = 0;  // of tile j
  for (int j = -1; j < sc.count; ++j) {
    if (j + 1 < sc.count) {
      if (j >= 0) cursor_next(a, nxt);
      if (!scales(j + 1, nxt)) break;
    }
    if (j < 0) {
      sigma = prev_sigma;
      continue;
    }
    if (j > 0) cursor_next(a, cur);
    const int s = j & 1;
    const uint8_t* nib = sm + kOffNib + s * kNibStage;
    const uint8_t* scb = sm + kOffSc + (j % kScSlots) * kScStage;
    const bool raw_ok = warp_wait(&ms.mb_rawfull[s], static_cast<uint32_t>((j >> 1) & 1), ms, a, 64, lane);
    // V'' quarter k: warp lw converts 4 tokens of the quarter's 8-token atom
    // lw / 2, rows {0, 2, 5, 7} (lw even) or {1, 3, 4, 6} (lw odd); lane l
    // the 32-element groups 8h + c, h = 0, 1, with c % 4 = l % 4 (bits 0-1),
    // c / 4 = bit 4, and the row chosen by bits 2-3.  Every 8-lane phase of a
    // 16-byte access then meets 8 distinct bank groups, for the swizzled
    // nibble loads (c ^ row) and the V'' stores (2 (c % 4) ^ row) alike.
#pragma unroll 1
    for (int k = 0; k < 4; ++k) {
      const bool slot_ok =
          raw_ok && (j == 0 || warp_wait(&ms.mb_pvq[k], static_cast<uint32_t>((j - 1) & 1), ms, a, 64, lane));
      if (slot_ok) {
        const int c = (lane & 3) | ((lane >> 2) & 4);
        const int t = 32 * k + 8 * (lw >> 1) + (((2 * ((lane >> 3) & 1)) | (lw & 1)) ^ (5 * ((lane >> 2) & 1)));
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint4 nb =
              *reinterpret_cast<const uint4*>(nib + h * kNibBlock + (t >> 3) * 1024 + sw128_offset(t & 7, c));
          const int sbyte = scb[t * kScaleBytes + 8 * h + c];
          // Rows past the tile's valid tokens (a tail page's unused slots, or
          // stale bytes of a slot that was not loaded) are converted like the
          // others: the exponent clamp keeps every byte finite (<= 6 * 2^13),
          // and their P'' is exactly zero, so they add nothing to O.  Valid
          // rows never reach the clamp (sigma keeps them at k <= 13).
          uint32_t lo, hi;
          e5m2_tables(min(sbyte - 127 - sigma, 13), lo, hi);
          const uint4 o0 = half_group_to_e5m2(nb.x, nb.y, lo, hi);
          const uint4 o1 = half_group_to_e5m2(nb.z, nb.w, lo, hi);
          uint8_t* atom = sm + kOffV + (2 * h + (c >> 2)) * kVCol + (t >> 3) * 1024;
          *reinterpret_cast<uint4*>(atom + sw128_offset(t & 7, 2 * (c & 3))) = o0;
          *reinterpret_cast<uint4*>(atom + sw128_offset(t & 7, 2 * (c & 3) + 1)) = o1;
        }
        fence_proxy_async_smem();
      }
      __syncwarp();
      if (lane == 0 && slot_ok) mbar_arrive(&ms.mb_vfull[k]);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&ms.mb_nibread[s]);
    sigma = prev_sigma;  // tile j + 1's, computed above
  }
}

// ---------------------------------------------------------------------------
// Q of one sequence for a block of NH heads (256 threads: 256 / NH per head;
// with 4 per head (NH = 64) part p handles the 32-element blocks 4p .. 4p + 3
// of the latent and 16-byte chunks 2p, 2p + 1 of q_pe, with 16 per head
// (NH = 16) block p and chunk p < 8).  Writes the QK operand images: the terms
// at qdst (the layout of kOffQ: term t of head h is row NH t + h), q_pe at
// pedst (the layout of the form's kOffQpe) and the terms' scale bytes at sfdst
// as [3 NH rows][16 blocks].  Used in shared memory by the decode kernel (no
// workspace) and in global memory by the Q prep kernel.
// ---------------------------------------------------------------------------
template <int NH>
__device__ __forceinline__ void q_block(const uint4 (&v)[4], int h, int bl, uint8_t* qdst, uint8_t* sfdst) {
  float x[32];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint32_t ws[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      x[8 * k + 2 * i] = __uint_as_float(ws[i] << 16);
      x[8 * k + 2 * i + 1] = __uint_as_float(ws[i] & 0xFFFF0000u);
    }
  }
#pragma unroll
  for (int t = 0; t < 3; ++t) {
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(x[i]));
    // smallest e with amax <= 6 * 2^e: amax = 1.m * 2^f -> f - 2, or f - 1 when 1.m > 1.5
    const uint32_t ab = __float_as_uint(amax);
    int e = static_cast<int>(ab >> 23) - 129 + ((ab & 0x7FFFFFu) > 0x400000u ? 1 : 0);
    e = max(-127, min(126, e));
    const float inv = __uint_as_float(static_cast<uint32_t>(127 - e) << 23);
    const float scl = e >= -126 ? __uint_as_float(static_cast<uint32_t>(e + 127) << 23) : __uint_as_float(0x00400000u);
    uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const uint32_t byte = cvt_f32x2_e2m1x2(x[2 * i] * inv, x[2 * i + 1] * inv);
      w[i >> 2] |= byte << (8 * (i & 3));
      if (t < 2) {
        const uint32_t h2 = cvt_e2m1x2_f16x2(byte);
        x[2 * i] -= __half2float(__ushort_as_half(static_cast<unsigned short>(h2 & 0xFFFFu))) * scl;
        x[2 * i + 1] -= __half2float(__ushort_as_half(static_cast<unsigned short>(h2 >> 16))) * scl;
      }
    }
    const int n = NH * t + h;
    *reinterpret_cast<uint4*>(qdst + (bl >> 3) * Form<NH>::kQBlock + (n >> 3) * 1024 + sw128_offset(n & 7, bl & 7)) =
        make_uint4(w[0], w[1], w[2], w[3]);
    sfdst[n * kScaleBytes + bl] = static_cast<uint8_t>(e + 127);
  }
}

template <int NH>
__device__ void q_operands(const DecodeArgs& a, int b, int head_base, int heads_here, int tid, uint8_t* qdst,
                           uint8_t* pedst, uint8_t* sfdst) {
  constexpr int kParts = kSoftmaxThreads / NH;    // threads per head
  constexpr int kBlocks = 16 / kParts;            // 32-element blocks per thread
  constexpr int kPeChunks = kParts >= 8 ? 1 : 8 / kParts;  // 16-byte q_pe chunks per thread
  const int h = tid / kParts, part = tid % kParts;
  const bool live = h < heads_here;
  const __nv_bfloat16* qrow = a.q + b * a.q_stride_b + (head_base + h) * a.q_stride_h;
#pragma unroll 1
  for (int blk = 0; blk < kBlocks; ++blk) {
    uint4 v[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) v[k] = ldg_stream_if(qrow + 32 * (kBlocks * part + blk) + 8 * k, live);
    q_block<NH>(v, h, kBlocks * part + blk, qdst, sfdst);
  }
  if (kPeChunks * part < 8) {
#pragma unroll
    for (int k = 0; k < kPeChunks; ++k)
      *reinterpret_cast<uint4*>(pedst + (h >> 3) * 1024 + sw128_offset(h & 7, kPeChunks * part + k)) =
          ldg_stream_if(qrow + kLatent + 8 * (kPeChunks * part + k), live);
  }
}

// B scale factors of the Q terms into TMEM (softmax warps 0-3, one TMEM lane
// quarter each): column 8 k4 + n1 of lane n0 (every quarter alike) holds the
// scale word k4 of row n0 + 32 n1 (rows >= 3 NH are not read).  `global` says
// whether sf ([3 NH][16] bytes) lies in global memory.
template <int NH>
__device__ __forceinline__ void store_q_scales(uint32_t tmem, const uint8_t* sf, bool global, int warp, int lane) {
  constexpr int kRows = Form<NH>::kQRows;
  uint32_t u[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const int n = lane + 32 * (i & 7);
    const uint8_t* src = sf + min(n, kRows - 1) * kScaleBytes + 4 * (i >> 3);
    const uint32_t w = global ? static_cast<uint32_t>(ldg_s32_or(reinterpret_cast<const int32_t*>(src), true, 0))
                              : *reinterpret_cast<const uint32_t*>(src);
    u[i] = n < kRows ? w : 0x7F7F7F7Fu;
  }
  tmem_st32(tmem + (static_cast<uint32_t>(32 * warp) << 16) + kColSfb, u);
  tmem_st_wait();
}

// Q operands of a new piece's sequence (softmax threads).  With Q images in
// the workspace: one bulk copy of the terms and q_pe (completing mb_qload)
// and the scale factors from global memory; otherwise quantised here.
template <int NH, bool kQImg>
__device__ void build_q(uint8_t* sm, Misc& ms, uint32_t tmem, const DecodeArgs& a, int b, int head_base,
                        int heads_here, int warp, int lane) {
  using F = Form<NH>;
  constexpr uint32_t kLoadBytes = q_term_bytes(NH) + q_pe_bytes(NH);
  const int tid = threadIdx.x;
  if constexpr (kQImg) {
    const uint8_t* img =
        a.q_img + (static_cast<int64_t>(b) * head_blocks<NH>(a) + head_block<NH>(a)) * q_image_bytes(NH);
    asm volatile("griddepcontrol.wait;\n" ::: "memory");  // the Q prep grid is complete (no-op later)
    if (tid == 0) {
      mbar_arrive_expect_tx(&ms.mb_qload, kLoadBytes);
      bulk_load(sm + kOffQ, img, kLoadBytes, &ms.mb_qload);
    }
    if (tid < NH) ms.R[tid] = 0.f;
    if (warp < 4) store_q_scales<NH>(tmem, img + kLoadBytes, true, warp, lane);
  } else {
    uint8_t* sf_stage = sm + F::kOffP;  // [3 NH rows][16] e8m0 (P'' is free at a piece start)
    q_operands<NH>(a, b, head_base, heads_here, tid, sm + kOffQ, sm + F::kOffQpe, sf_stage);
    if (tid < NH) ms.R[tid] = 0.f;
    named_bar(kBarSoftmax, kSoftmaxThreads);  // the scale bytes are staged
    if (warp < 4) store_q_scales<NH>(tmem, sf_stage, false, warp, lane);
  }
}

// ---------------------------------------------------------------------------
// Softmax warps (0..7) and the per-piece epilogue
// ---------------------------------------------------------------------------
// HT = NH / 2 heads per thread: warp w takes TMEM lane quadrant (token
// quarter) w % 4 and heads HT (w / 4) .. HT (w / 4) + HT - 1.
template <int HT>
__device__ __forceinline__ void tmem_ld_heads(uint32_t taddr, uint32_t (&r)[HT]) {
  if constexpr (HT == 32) tmem_ld32(taddr, r);
  else tmem_ld8(taddr, r);
}

template <int NH, bool kQImg>
__device__ void softmax(uint8_t* sm, Misc& ms, uint32_t tmem, const Sched& sc, int head_base, int heads_here,
                        int warp, int lane, float c_log2, const DecodeArgs& a) {
  using F = Form<NH>;
  constexpr int HT = NH / 2;
  static_assert(HT == 32 || HT == 8, "heads per softmax thread");
  const int tid = threadIdx.x;
  const int q = warp & 3;                  // TMEM lane quadrant
  const int hf = warp >> 2;                // heads HT hf .. HT hf + HT - 1
  const int st = 32 * q + lane;            // softmax token
  const uint32_t lane_base = static_cast<uint32_t>(32 * q) << 16;

  float l_part[HT];
#pragma unroll
  for (int j = 0; j < HT; ++j) l_part[j] = 0.f;
  int sigma_prev = 0;
  Cursor cur;
  cursor_start(a, sc, cur);

  for (int tile = 0; tile < sc.count; ++tile, cursor_next(a, cur)) {
    const uint32_t par = static_cast<uint32_t>(tile & 1);
    const bool first = cursor_first(cur);
    if (first) {
      // a new sequence: its Q replaces the previous one (whose last QK is
      // complete: its S was read; its last PV too: the epilogue waited for it)
      build_q<NH, kQImg>(sm, ms, tmem, a, cur.b, head_base, heads_here, warp, lane);
      fence_proxy_async_smem();
      fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ms.mb_qready);
      named_bar(kBarSoftmax, kSoftmaxThreads);  // R of the new sequence is visible
    }
    bool ok = warp_wait(&ms.mb_sfull, par, ms, a, 1, lane);
    fence_after_sync();
    float t[HT];
    int sigma_cur = sigma_prev;
    if (ok) {
      {
        uint32_t sv[HT];
        tmem_ld_heads<HT>(tmem + lane_base + kColS + HT * hf, sv);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < HT; ++j) t[j] = __uint_as_float(sv[j]);
        tmem_ld_heads<HT>(tmem + lane_base + kColS + NH + HT * hf, sv);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < HT; j += 2) add_f32x2(t[j], t[j + 1], __uint_as_float(sv[j]), __uint_as_float(sv[j + 1]));
        tmem_ld_heads<HT>(tmem + lane_base + kColS + 2 * NH + HT * hf, sv);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < HT; j += 2) add_f32x2(t[j], t[j + 1], __uint_as_float(sv[j]), __uint_as_float(sv[j + 1]));
      }
      fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ms.mb_sfree);
      ok = warp_wait(&ms.mb_sigready[tile & 3], static_cast<uint32_t>((tile >> 2) & 1), ms, a, 1, lane);
      sigma_cur = ms.sig[tile & 3];
      // x - R_h in log2 units; a full tile (every tile but a sequence's
      // last) needs no per-token mask and takes packed multiply-adds
      const int nvalid = cursor_valid(cur);
      if (nvalid == 2 * kPageSize) {
#pragma unroll
        for (int j = 0; j < HT; j += 4) {
          const float4 r4 = *reinterpret_cast<const float4*>(&ms.R[HT * hf + j]);
          fma_f32x2(t[j], t[j + 1], c_log2, -r4.x, -r4.y);
          fma_f32x2(t[j + 2], t[j + 3], c_log2, -r4.z, -r4.w);
        }
      } else {
        const bool tvalid = st < nvalid;
#pragma unroll
        for (int j = 0; j < HT; j += 4) {
          const float4 r4 = *reinterpret_cast<const float4*>(&ms.R[HT * hf + j]);
          const float rv[4] = {r4.x, r4.y, r4.z, r4.w};
#pragma unroll
          for (int u = 0; u < 4; ++u) t[j + u] = tvalid ? fmaf(t[j + u], c_log2, -rv[u]) : -CUDART_INF_F;
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < HT; ++j) t[j] = -CUDART_INF_F;
    }
    // rescale event: a piece's first tile, a score above R + 8.5, or a new sigma.
    // One barrier ORs "event or failure"; only when it is raised does a second
    // one tell a failure (leave the loop) from an event.
    float tmaxv = -CUDART_INF_F;
#pragma unroll
    for (int j = 0; j < HT; ++j) tmaxv = fmaxf(tmaxv, t[j]);
    const bool need =
        bar_or(kBarSoftmax, kSoftmaxThreads, !ok || first || tmaxv > 8.5f || sigma_cur != sigma_prev);
    if (need && bar_or(kBarSoftmax, kSoftmaxThreads, !ok)) break;
    fence_after_sync();
    // PV(j-1) must be complete before O is rescaled or P'' is overwritten.  The
    // wait sits right before the first of those, so the score work of tile j
    // overlaps PV(j-1).  A wait that gives up has raised the abort word; the
    // warp keeps to the common barrier sequence and leaves at the next check.
    bool pv_prev_done = tile == 0, pvq_prev_done = tile == 0;
    // All of PV(j - 1) is waited for on tiledone[(j - 1) % 2], not on
    // pvq[3]: a parity wait names the right phase only while the barrier is at
    // most one phase past it, and warps of quarters 0..2 wait on pvq[3] only
    // now and then (pvq[3] could match PV(j - 3) while PV(j - 2) ran).  Slot
    // (j - 1) % 2 holds tiles j - 3 and j + 1 on either side: PV(j - 3)
    // completed before the PV(j - 2) quarter this warp waited for in tile
    // j - 1, and PV(j + 1) needs this tile's P''.
    auto wait_pv_prev = [&]() {  // all of PV(j-1)
      if (!pv_prev_done) {
        warp_wait(&ms.mb_tiledone[(tile - 1) & 1], static_cast<uint32_t>(((tile - 1) >> 1) & 1), ms, a, 2, lane);
        fence_after_sync();
        pv_prev_done = pvq_prev_done = true;
      }
    };
    auto wait_pvq_prev = [&]() {  // PV(j-1) of this warp's token quarter (its P'' rows)
      if (!pvq_prev_done) {
        warp_wait(&ms.mb_pvq[q], static_cast<uint32_t>((tile - 1) & 1), ms, a, 2, lane);
        fence_after_sync();
        pvq_prev_done = true;
      }
    };
    if (need) {
      float v[HT];
#pragma unroll
      for (int j = 0; j < HT; ++j) v[j] = t[j];
      const float vmax = warp_transpose_reduce<true, HT>(v, lane);  // tile max of x - R_old, head lane % HT
      if (lane < HT) ms.red[q][HT * hf + lane] = vmax;
      named_bar(kBarSoftmax, kSoftmaxThreads);
      if (tid < NH) {
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
      for (int j = 0; j < HT; ++j) t[j] -= ms.red[0][HT * hf + j];
      if (!first) {
#pragma unroll
        for (int j = 0; j < HT; ++j) l_part[j] *= ms.beta[HT * hf + j];
        wait_pv_prev();
        // O chunks 2 hf, 2 hf + 1 of this lane quadrant, 32 columns at a time:
        // head column j (wide form), or hi / lo column of head j % 16 (small)
#pragma unroll 1
        for (int cc = 0; cc < 2; ++cc) {
          const int c = 2 * hf + cc;
#pragma unroll 1
          for (int hh = 0; hh < static_cast<int>(F::kOChunkCols) / 32; ++hh) {
            uint32_t vv[32];
            const uint32_t ta = tmem + lane_base + kColO + F::kOChunkCols * c + 32 * hh;
            tmem_ld32(ta, vv);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 32; ++j)
              vv[j] = __float_as_uint(__uint_as_float(vv[j]) * ms.alpha[NH == 64 ? 32 * hh + j : j % NH]);
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
      uint32_t pw[HT / 4], pl[HT / 4];
#pragma unroll
      for (int j = 0; j < HT; j += 2) {
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
      wait_pvq_prev();
      const int prow = (st >> 3) * F::kPRow + (st & 7) * 16;
      if constexpr (NH == 64) {
        // heads 32 hf .. : two 16-head cores of each term
        *reinterpret_cast<uint4*>(sm + F::kOffP + prow + (2 * hf) * 128) = make_uint4(pw[0], pw[1], pw[2], pw[3]);
        *reinterpret_cast<uint4*>(sm + F::kOffP + prow + (2 * hf + 1) * 128) = make_uint4(pw[4], pw[5], pw[6], pw[7]);
        *reinterpret_cast<uint4*>(sm + F::kOffPlo + prow + (2 * hf) * 128) = make_uint4(pl[0], pl[1], pl[2], pl[3]);
        *reinterpret_cast<uint4*>(sm + F::kOffPlo + prow + (2 * hf + 1) * 128) = make_uint4(pl[4], pl[5], pl[6], pl[7]);
      } else {
        // heads 8 hf .. 8 hf + 7: half of the one 16-head core row of each term
        *reinterpret_cast<uint2*>(sm + F::kOffP + prow + 8 * hf) = make_uint2(pw[0], pw[1]);
        *reinterpret_cast<uint2*>(sm + F::kOffPlo + prow + 8 * hf) = make_uint2(pl[0], pl[1]);
      }
    }
    fence_proxy_async_smem();
    fence_before_sync();
    __syncwarp();
    if (lane == 0) mbar_arrive(&ms.mb_pfull[q]);

    if (!cursor_last(cur)) continue;
    // ---------------- epilogue of the piece ----------------
    const bool done = warp_wait(&ms.mb_tiledone[tile & 1], static_cast<uint32_t>((tile >> 1) & 1), ms, a, 4, lane);
    if (bar_or(kBarSoftmax, kSoftmaxThreads, !done)) break;
    fence_after_sync();
    {
      const float s = warp_transpose_reduce<false, HT>(l_part, lane);
      if (lane < HT) ms.red[q][HT * hf + lane] = s;
    }
#pragma unroll
    for (int j = 0; j < HT; ++j) l_part[j] = 0.f;
    // the piece covers its whole sequence -> final output; otherwise a partial in its slot
    const bool direct = a.balanced ? (cur.piece_begin == 0 && cur.piece_end == cursor_tiles(cur))
                                   : a.num_splits == 1;
    const int64_t slot = a.balanced ? static_cast<int64_t>(cur.b) + cta_index<NH>(a)
                                    : static_cast<int64_t>(cur.b) * a.num_splits + cta_index<NH>(a);
    named_bar(kBarSoftmax, kSoftmaxThreads);
    if (tid < NH) {
      const float l = ms.red[0][tid] + ms.red[1][tid] + ms.red[2][tid] + ms.red[3][tid];
      // output factor 2^sigma / l per head (alpha is free again)
      ms.alpha[tid] = l > 0.f ? exp2f(static_cast<float>(sigma_prev)) / l : 0.f;
      if (!direct && tid < heads_here)
        a.partial_lse[slot * a.num_heads + head_base + tid] = (ms.R[tid] + __log2f(l)) * kLn2;
    }
    if (a.balanced && tid == 0 && cur.piece_begin == 0) {
      // this CTA holds the sequence's first tile: record its CTA span for the merge
      const int last_cta = cta_of_tile(cur.seq_pos + cursor_tiles(cur) - 1, sc, cta_count<NH>(a));
      a.seq_meta[cur.b] = make_int2(cta_index<NH>(a), last_cta);
    }
    named_bar(kBarSoftmax, kSoftmaxThreads);
    // thread reads O^T lanes 32q.. of chunks 2hf, 2hf+1: latent d = 128c + 32q + lane.
    // Each 32-latent x 32-head unit (wide form; 32 x 16 in the small form,
    // whose O holds each head's hi and lo sums apart) is transposed through
    // this warp's 2 KB of the stage (the wide form's P'' area, idle: the
    // piece's last PV is complete) into rows of 8 latents per head, stored as
    // 16-byte vectors.
    const bool vec = !direct || ((reinterpret_cast<uintptr_t>(a.o) |
                                  static_cast<uintptr_t>(a.o_stride_b * 2) |
                                  static_cast<uintptr_t>(a.o_stride_h * 2)) & 15) == 0;
    uint8_t* stage = sm + F::kOffStage + warp * 2048;
    constexpr int kUnitHeads = NH == 64 ? 32 : NH;  // heads of one transposed unit
#pragma unroll 1
    for (int cc = 0; cc < 2; ++cc) {
      const int c = 2 * hf + cc;
#pragma unroll 1
      for (int hh = 0; hh < NH / kUnitHeads; ++hh) {
        uint32_t vv[32];
        tmem_ld32(tmem + lane_base + kColO + F::kOChunkCols * c + 32 * hh, vv);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < kUnitHeads; ++j) {
          const float o = NH == 64 ? __uint_as_float(vv[j]) : __uint_as_float(vv[j]) + __uint_as_float(vv[j + NH]);
          reinterpret_cast<__nv_bfloat16*>(stage)[32 * j + lane] = __float2bfloat16_rn(o * ms.alpha[32 * hh + j]);
        }
        __syncwarp();
#pragma unroll
        for (int i = 0; i < kUnitHeads / 8; ++i) {
          const int idx = 32 * i + lane, hd = 32 * hh + (idx >> 2), d0 = 128 * c + 32 * q + 8 * (idx & 3);
          const uint4 v = *reinterpret_cast<const uint4*>(stage + 16 * idx);
          if (hd < heads_here) {
            const int hq = head_base + hd;
            __nv_bfloat16* dst = direct ? a.o + cur.b * a.o_stride_b + hq * a.o_stride_h + d0
                                        : a.partial_o + (slot * a.num_heads + hq) * kLatent + d0;
            if (vec) {
              *reinterpret_cast<uint4*>(dst) = v;
            } else {
              const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
              for (int e = 0; e < 8; ++e)
                dst[e] = __ushort_as_bfloat16(static_cast<unsigned short>(w[e >> 1] >> (16 * (e & 1))));
            }
          }
        }
        __syncwarp();  // the stage is rewritten by the next unit
      }
    }
    // O and alpha are read before the next piece's PV / rescale touch them
    fence_before_sync();
    named_bar(kBarSoftmax, kSoftmaxThreads);
  }
}

// Instances by heads per CTA (NH = 64, or 16 for calls with at most 16 heads)
// and by kQImg: Q operand images from the prep kernel in the workspace (the
// serving path), or, without them, Q quantised here at each piece start; the
// second's code stays out of the first (the kernel is bound by instruction
// fetch).
template <int NH, bool kQImg>
__global__ void __launch_bounds__(kThreads, 1) mla_decode_fp4_kernel(const __grid_constant__ DecodeArgs a,
                                                                  const __grid_constant__ CacheMaps maps) {
  // the merge kernel (launched next as a programmatic dependent) may be
  // scheduled once every CTA of this grid runs; it waits for this grid to
  // complete before reading anything
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
  uint8_t* sm = smem_base();
  Misc& ms = *reinterpret_cast<Misc*>(sm + Form<NH>::kOffMisc);
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int head_base = head_block<NH>(a) * NH;
  const int heads_here = min(NH, a.num_heads - head_base);

  Sched sc;
  if (a.balanced) {
    balanced_schedule<kThreads>(a, ms.sched, sc, cta_count<NH>(a), cta_index<NH>(a));
    if (sc.count == 0) {
      // An empty run (fewer tiles than CTAs) can sit inside the CTA span of
      // the sequence at its position; its slot of that sequence carries no weight.
      if (sc.pos0 < sc.total && tid < heads_here)
        a.partial_lse[(static_cast<int64_t>(sc.b0) + cta_index<NH>(a)) * a.num_heads + head_base + tid] = -CUDART_INF_F;
      return;  // (uniform: every thread read the same count)
    }
  } else {
    const int b = blockIdx.y, tiles = seq_tiles_of(a, b);
    const int per_split = (tiles + a.num_splits - 1) / a.num_splits;
    sc.b0 = b;
    sc.off0 = cta_index<NH>(a) * per_split;
    sc.count = max(0, min(per_split, tiles - sc.off0));
    sc.pos0 = 0;
    sc.total = 0;
    if (sc.count == 0) {
      // nothing to attend to: zeros (one split) or a split that carries no weight
      if (a.num_splits == 1) {
        for (int i = tid; i < heads_here * (kLatent / 2); i += kThreads) {
          const int h = i / (kLatent / 2), d = (i % (kLatent / 2)) * 2;
          *reinterpret_cast<uint32_t*>(a.o + b * a.o_stride_b + (head_base + h) * a.o_stride_h + d) = 0u;
        }
      } else if (tid < heads_here) {
        a.partial_lse[(static_cast<int64_t>(b) * a.num_splits + cta_index<NH>(a)) * a.num_heads + head_base + tid] =
            -CUDART_INF_F;
      }
      return;
    }
  }

  // ---------------- setup: barriers and TMEM ----------------
  if (tid == 0) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      mbar_init(&ms.mb_rawfull[i], 1);
      mbar_init(&ms.mb_qkdone[i], 1);
      mbar_init(&ms.mb_nibread[i], kLoaderWarps);
      mbar_init(&ms.mb_sfafull[i], 4);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      mbar_init(&ms.mb_scfull[i], 1);
      mbar_init(&ms.mb_vfull[i], kLoaderWarps);
      mbar_init(&ms.mb_pvq[i], 2);
      mbar_init(&ms.mb_sigready[i], 1);
      ms.tile_smax[i] = 0;
    }
    mbar_init(&ms.mb_tiledone[0], 2);
    mbar_init(&ms.mb_tiledone[1], 2);
    mbar_init(&ms.mb_kpefull, 1);
    mbar_init(&ms.mb_kpefree, 1);
    mbar_init(&ms.mb_sfull, 1);
    mbar_init(&ms.mb_sfree, kSoftmaxWarps);
    for (int i = 0; i < 4; ++i) mbar_init(&ms.mb_pfull[i], 2);
    mbar_init(&ms.mb_qready, kSoftmaxWarps);
    mbar_init(&ms.mb_qload, 1);
    mbar_init(&ms.mb_drain, 3);
    ms.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kWarpQK) tmem_alloc(&ms.tmem_base, kTmemCols);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = ms.tmem_base;

  // Register budgets: the issuer and loader warpgroups give registers back
  // before the softmax warpgroups' increase can be granted.
  if (warp >= kWarpQK) {
    setmaxnreg_dec<kIssuerRegs>();
    if (warp == kWarpQK) {
      qk_issuer<NH>(sm, ms, tmem, sc, lane, a);
    } else if (warp < kWarpTMA) {
      pv_issuer<NH>(sm, ms, tmem, sc, lane, warp - kWarpPV0, a);
    } else if (lane == 0) {
      producer(sm, ms, sc, a, maps);
    }
    // drain: arrives once every MMA this thread issued has completed
    if (warp < kWarpTMA && lane == 0) mma_commit(&ms.mb_drain);
    __syncwarp();
  } else if (warp >= kLoaderWarp0) {
    setmaxnreg_dec<kLoaderRegs>();
    loader(sm, ms, tmem, sc, warp, lane, a);
  } else {
    setmaxnreg_inc<kSoftmaxRegs>();
    softmax<NH, kQImg>(sm, ms, tmem, sc, head_base, heads_here, warp, lane, a.sm_scale * kLog2e, a);
  }

  fence_before_sync();
  __syncthreads();  // every TMEM read is done
  if (warp == kWarpQK) {
    if (lane == 0 && !mbar_wait_bounded(&ms.mb_drain, 0, kPollLimit)) record_status(a, 128);
    __syncwarp();
    fence_after_sync();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// Q operand images of every (sequence, head block): one CTA of 16 NH threads
// each, thread (h, bl) quantising the 32-element block bl of head h (and the
// 16-byte chunk bl < 8 of its q_pe).  It lets the decode kernel launched
// after it start at once; that kernel waits for this grid before reading
// the images.
template <int NH>
__global__ void __launch_bounds__(16 * NH) q_prep_fp4_kernel(const __grid_constant__ DecodeArgs a) {
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
  const int b = blockIdx.y, head_base = blockIdx.x * NH;
  const int h = threadIdx.x >> 4, bl = threadIdx.x & 15;
  const bool live = h < a.num_heads - head_base;
  uint8_t* img =
      const_cast<uint8_t*>(a.q_img) + (static_cast<int64_t>(b) * gridDim.x + blockIdx.x) * q_image_bytes(NH);
  const __nv_bfloat16* qrow = a.q + b * a.q_stride_b + (head_base + h) * a.q_stride_h;
  uint4 v[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) v[k] = ldg_stream_if(qrow + 32 * bl + 8 * k, live);
  const uint4 pe = ldg_stream_if(qrow + kLatent + 8 * (bl & 7), live && bl < 8);
  q_block<NH>(v, h, bl, img, img + q_term_bytes(NH) + q_pe_bytes(NH));
  if (bl < 8) *reinterpret_cast<uint4*>(img + q_term_bytes(NH) + (h >> 3) * 1024 + sw128_offset(h & 7, bl)) = pe;
}

template <int NH>
cudaError_t launch_decode_form(const DecodeArgs& a, const CacheMaps& maps, cudaStream_t stream) {
  constexpr int kSmem = smem_bytes<NH>();
  cudaError_t e = cudaFuncSetAttribute(mla_decode_fp4_kernel<NH, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       kSmem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(mla_decode_fp4_kernel<NH, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
  if (e != cudaSuccess) return e;
  const int head_blocks = (a.num_heads + NH - 1) / NH;
  const dim3 grid = a.balanced ? dim3(a.num_splits * head_blocks, 1, 1) : dim3(a.num_splits * head_blocks, a.batch, 1);
  if (!a.q_img) {
    mla_decode_fp4_kernel<NH, false><<<grid, kThreads, kSmem, stream>>>(a, maps);
    return cudaGetLastError();
  }
  // after the Q prep kernel: start while it runs (everything before the Q
  // images, the first cache loads included, overlaps it)
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, mla_decode_fp4_kernel<NH, true>, a, maps);
}

}  // namespace

cudaError_t launch_q_prep_fp4(const DecodeArgs& a, cudaStream_t stream) {
  if (decode_heads_per_cta(a.num_heads) == 16) {
    q_prep_fp4_kernel<16><<<dim3((a.num_heads + 15) / 16, a.batch), 16 * 16, 0, stream>>>(a);
  } else {
    q_prep_fp4_kernel<64><<<dim3((a.num_heads + 63) / 64, a.batch), 16 * 64, 0, stream>>>(a);
  }
  return cudaGetLastError();
}

cudaError_t launch_decode_fp4(const DecodeArgs& a, const CacheMaps& maps, cudaStream_t stream) {
  return decode_heads_per_cta(a.num_heads) == 16 ? launch_decode_form<16>(a, maps, stream)
                                                 : launch_decode_form<64>(a, maps, stream);
}

}  // namespace kimi
