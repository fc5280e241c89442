// Split-K absorbed-MLA decode over the MXFP4 paged cache, sm_100a, on pairs
// of CTAs (thread-block clusters of two): Q K^T as block-scaled e2m1
// tensor-core MMAs straight from the cache bytes in the first CTA, P V with
// the heads on the MMA's M dimension in the second.
//
// Math (paths inside ianye23301/kimi): the archive stage-1 kernel
// `_mla_decode_split_kv` (archive/mla-mxfp4-dead-end/mla_decode_mxfp4_v5.py:136-261),
// which likewise computes Q K^T with an MXFP4 x MXFP4 block-scaled dot
// (`tl.dot_scaled(q_fp4, q_scale, "e2m1", k_u8, k_scale, "e2m1")`), under the
// contract of `reference_mla_decode` (tests/test_triton_mla_decode.py:12-62):
//   S = q_nope . k_nope + q_pe . k_pe,  P = softmax(S * sm_scale),  O = P . k_nope.
//
// A pair takes up to 64 heads over a run of 128-token tiles (two pages);
// decode_common.cuh has the schedule (a run per pair).
//
// CTA 0 (QK): tokens on the MMA's M dimension, heads on N.
//   * The tile's nibbles arrive by TMA as they lie in the cache (two
//     128-byte-swizzled K-major column blocks of 128 rows), the K-major A
//     operand of tcgen05.mma kind::mxf4; a scale warp regroups the e8m0 bytes
//     in place and the MMA thread moves them into TMEM with tcgen05.cp.
//     q_nope is three block-scaled e2m1 terms (each the e2m1 rounding of the
//     remaining residual), one N = 192 B operand whose terms land in S column
//     groups 0, 64 and 128 and are summed by the softmax: bf16-level scores,
//     where the reference quantises q to one term.  q_pe . k_pe is a bf16 MMA
//     into column group 0.  S is double-buffered in TMEM.
//   * Softmax warps: P'' = exp2(x - R_h) (R_h per head, kept in [max - 8.5,
//     max - 4] of the running maximum, raised lazily) as two e4m3 terms
//     (hi + residual), stored straight into CTA 1's shared memory as the A
//     operand of its P V MMAs: one 128-byte row per token, the hi terms of
//     the 64 heads then the lo terms.
// CTA 1 (PV): heads on M (128 rows: the hi and the lo term of 64 heads),
// latent on N.
//   * Converter warps write V'' = e2m1 * 2^(scale - 127 - sigma) as e5m2
//     (exact; sigma a reference exponent per tile, moved only when the tile's
//     scales leave the exact e5m2 range) from the same nibbles, loaded by TMA
//     again (an L2 hit), by 32-token quarter into a four-slot ring.
//   * P V: 8 MMAs per tile (4 K steps x 2 latent halves of N = 256) into
//     O_hl, 128 TMEM lanes x 512 columns: row h holds head h's hi-term sum,
//     row 64 + h its lo-term sum; the epilogue adds the two.
//   * Epilogue warps rescale O when CTA 0 reports a move of R or sigma moves,
//     and write each piece's output (or partial and log-sum-exp).
//
// Both CTAs: 16 warps.  Warp 0 TMA producer (lane 0), warp 1 TMEM and the MMA
// thread (lane 0 issues every tcgen05 operation of its CTA), warp 3 scale
// warp; CTA 0: warp 2 k_pe producer, warps 4-11 softmax; CTA 1: warps 4-7
// epilogue, warps 8-15 converters.
//
// Cross-CTA traffic: P'' rows, a per-tile event record (did R move, and by
// how much) and a per-piece record (softmax sums, R) go from CTA 0 to CTA 1
// as distributed-shared-memory stores followed by a release arrive on CTA
// 1's mbarriers; CTA 1's MMA thread reports a P'' buffer free with a
// multicast commit onto CTA 0's mbarrier, and its epilogue frees the piece
// record with a remote arrive.  No TMA multicast.
//
// Every wait is bounded in time (DecodeArgs::timeout_ns); a wait that gives
// up records a status bit and raises its CTA's abort word, which ends the
// CTA's other waits; the peer's waits on it then run out in turn.  Each role
// leaves its loop, the producers wait for the copies they issued, the MMA
// thread's drain commit waits for its MMAs, TMEM is freed, and a cluster
// barrier keeps either CTA from exiting while the other may still touch its
// shared memory.
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

constexpr int kNH = 64;  // heads per pair
constexpr int kThreads = 512;
constexpr int kWarpTMA = 0, kWarpMMA = 1, kWarpKpe = 2, kWarpScale = 3;
constexpr int kSoftmaxWarp0 = 4, kSoftmaxWarps = 8, kSoftmaxThreads = 32 * kSoftmaxWarps;  // CTA 0
constexpr int kEpiWarp0 = 4, kEpiWarps = 4, kEpiThreads = 32 * kEpiWarps;                  // CTA 1
constexpr int kConvWarp0 = 8, kConvWarps = 8;                                              // CTA 1
constexpr uint32_t kTmemCols = 512;
// CTA 0 TMEM: S buffer b at 192 b (three 64-column term groups), A scale
// factors buffer b at 384 + 16 b, B scale factors at 416.  CTA 1 TMEM: O_hl,
// latent half h at 256 h.
constexpr uint32_t kColS = 0, kColSfa = 384, kColSfb = 416;
constexpr int kStages = 3;
constexpr int kPrefetchTiles = 4;  // L2 prefetch distance beyond the TMA loads (CTA 0)
constexpr int kBarSoftmax = 1, kBarEpi = 2;

// Shared memory (bytes).  Swizzled operands use 128B-swizzled atoms of 8 rows
// x 128 bytes (1 KB).  Misc sits at offset 0 in both CTAs, so an mbarrier has
// the same offset in each (what a multicast commit needs).
constexpr int kNibBlock = 128 * 128;                        // 128 token rows x 128 nibble bytes
constexpr int kStageNib = 2 * kNibBlock;                    // one tile's nibbles
constexpr int kStageBytes = kStageNib + 128 * kScaleBytes;  // + its e8m0 scales
constexpr int kOffMiscEnd = 3072;
// CTA 0
constexpr int kOffQ = kOffMiscEnd;  // Q image: terms, q_pe, scale factors (one bulk copy)
constexpr int kOffQpe = kOffQ + kQTermBytes;
constexpr int kOffQsf = kOffQpe + kQPeBytes;
constexpr int kOffStage0 = kOffQ + kQImageBytes;
constexpr int kOffKpe = kOffStage0 + kStages * kStageBytes;  // two buffers of 128 rows x 128 bytes
constexpr int kSmem0 = kOffKpe + 2 * 128 * 128;
// CTA 1
constexpr int kOffStage1 = kOffMiscEnd;
constexpr int kVChunk = 32 * 128;  // V'': 32 tokens x 128 latents (4 atoms)
constexpr int kVSlot = 4 * kVChunk;  // one token quarter, all 512 latents
constexpr int kOffV = kOffStage1 + kStages * kStageBytes;  // four quarter slots
constexpr int kPBuf = 128 * 128;  // P'' of a tile: 128 token rows x (64 hi + 64 lo) e4m3
constexpr int kOffP = kOffV + 4 * kVSlot;  // two buffers
constexpr int kOffEpi = kOffP + 2 * kPBuf;  // epilogue staging: 2 x 32 x 32 floats
constexpr int kSmem1 = kOffEpi + 2 * 4096;
constexpr int kSmem = kSmem0 > kSmem1 ? kSmem0 : kSmem1;
static_assert(kOffQ % 1024 == 0 && kOffQpe % 1024 == 0 && kOffStage0 % 1024 == 0 && kStageBytes % 1024 == 0 &&
                  kOffKpe % 1024 == 0 && kOffStage1 % 1024 == 0 && kOffV % 1024 == 0 && kOffP % 1024 == 0,
              "swizzled operands start on 1 KB boundaries");
static_assert(kSmem <= 232448, "shared memory budget");

struct Misc {
  // CTA 0
  uint64_t mb_stage_full[kStages];  // stage s landed (producer expect_tx + TMA bytes); both CTAs
  uint64_t mb_stage_free[kStages];  // CTA 0: QK done (commit); CTA 1: converters + scale warp done
  uint64_t mb_kpe_full[2];          // k_pe buffer b landed
  uint64_t mb_kpe_free[2];          // RoPE MMAs of the tile in k_pe buffer b complete (commit)
  uint64_t mb_q_full;               // a piece's Q image landed (bulk copy) or written (8 softmax warps)
  uint64_t mb_q_free;               // the last QK of a piece complete (commit)
  uint64_t mb_s_full[2];            // QK of the tile in S buffer b complete (commit)
  uint64_t mb_s_free[2];            // S buffer b read out of TMEM (8 softmax warps)
  uint64_t mb_sfa[kStages];         // stage s: scales regrouped for tcgen05.cp (scale warp)
  uint64_t mb_p_free[2];            // CTA 1's P'' buffer b read by its PV (CTA 1's multicast commit)
  uint64_t mb_stats_free;           // CTA 1 read the last piece record (remote arrive)
  // CTA 1
  uint64_t mb_sig[4];               // sigma of tile j published in sig[j % 4] (scale warp)
  uint64_t mb_p_full[2][4];         // P'' buffer b, token quarter k written (2 remote softmax warps)
  uint64_t mb_info_full[2];         // event record of the tile in P'' buffer b (remote)
  uint64_t mb_v_full[4];            // V'' ring slot k written (8 converter warps)
  uint64_t mb_pv_done[4];           // PV of token quarter k complete (commit; the converters wait on every phase)
  uint64_t mb_tile_done[2];         // PV of tile j complete, slot j % 2 (commit; the epilogue's waits)
  uint64_t mb_o_ready[2];           // O ready for the PV of tile j, slot j % 2 (4 epilogue warps)
  uint64_t mb_stats_full;           // a piece record arrived (remote)
  uint64_t mb_drain;                // the MMA thread's last commit
  SchedScratch sched;               // balanced mode: block-scan scratch
  uint32_t tmem_base;
  int abort_flag;
  int sig[4];                       // CTA 1: reference exponent of tile j in slot j % 4
  int info_event[2];                // CTA 1, written by CTA 0: 1 when the tile moved R
  alignas(16) float R[kNH];         // CTA 0: per-head exp2 offset, log2 units (read as float4)
  float red[4][kNH];                // CTA 0: cross-warp reduction scratch
  float info_alpha[2][kNH];         // CTA 1, written by CTA 0: O factor of the tile's R move
  float stat_l[kNH], stat_r[kNH];   // CTA 1, written by CTA 0: a piece's softmax sums and R
};
static_assert(sizeof(Misc) <= kOffMiscEnd, "Misc fits below the buffers");
static_assert(offsetof(Misc, R) % 16 == 0, "per-head arrays are read with 16-byte loads");

__device__ __forceinline__ uint8_t* smem_base() {
  extern __shared__ __align__(1024) uint8_t dyn_smem[];
  return dyn_smem;
}

__device__ __forceinline__ void record_status(const DecodeArgs& a, int bits) {
  if (a.status) atomicOr(a.status, bits);
}

// Per-thread bounded wait: one plain probe first (a phase that has already
// completed costs only that), then timed polls; on give-up records the
// failure and raises the abort word.
__device__ __forceinline__ bool wait_phase(uint64_t* mb, uint32_t parity, Misc& ms, const DecodeArgs& a, int bit) {
  if (mbar_try_wait(mb, parity)) return true;
  if (mbar_wait_timed(mb, parity, a.timeout_ns, &ms.abort_flag)) return true;
  if (atomicExch(&ms.abort_flag, 1) == 0) record_status(a, bit);
  return false;
}
// The same for a phase completed by arrivals from the other CTA (acquire at
// cluster scope).
__device__ __forceinline__ bool wait_phase_cluster(uint64_t* mb, uint32_t parity, Misc& ms, const DecodeArgs& a,
                                                   int bit) {
  if (mbar_try_wait_cluster(mb, parity)) return true;
  if (mbar_wait_timed_cluster(mb, parity, a.timeout_ns, &ms.abort_flag)) return true;
  if (atomicExch(&ms.abort_flag, 1) == 0) record_status(a, bit);
  return false;
}

// Warp-uniform bounded waits: every lane probes (one warp-wide instruction per
// poll) and a vote makes the verdict uniform.
__device__ __forceinline__ bool warp_wait(uint64_t* mb, uint32_t parity, Misc& ms, const DecodeArgs& a, int bit,
                                          int lane) {
  if (__all_sync(0xffffffffu, mbar_try_wait(mb, parity))) return true;
  const bool ok = __all_sync(0xffffffffu, mbar_wait_timed(mb, parity, a.timeout_ns, &ms.abort_flag));
  if (!ok && lane == 0 && atomicExch(&ms.abort_flag, 1) == 0) record_status(a, bit);
  return ok;
}
__device__ __forceinline__ bool warp_wait_cluster(uint64_t* mb, uint32_t parity, Misc& ms, const DecodeArgs& a,
                                                  int bit, int lane) {
  if (__all_sync(0xffffffffu, mbar_try_wait_cluster(mb, parity))) return true;
  const bool ok = __all_sync(0xffffffffu, mbar_wait_timed_cluster(mb, parity, a.timeout_ns, &ms.abort_flag));
  if (!ok && lane == 0 && atomicExch(&ms.abort_flag, 1) == 0) record_status(a, bit);
  return ok;
}

// Waits that let copies and MMAs already issued finish before the CTA exits:
// always the default bound, whatever the call's timeout.
__device__ __forceinline__ bool drain_wait(uint64_t* mb, uint32_t parity) {
  return mbar_wait_timed(mb, parity, kDefaultTimeoutNs, nullptr);
}

// Page rows (y coordinates of the cache tensor maps) of the two pages of the
// cursor's tile: -1 for a slot past the sequence's pages (nothing loaded).
// A page id outside [0, num_pages) maps to a row outside the tensor, which TMA
// fills with zeros, and is recorded in the status word (kStatusBadPage).
__device__ __forceinline__ void tile_rows(const DecodeArgs& a, const Cursor& c, int (&y)[2], bool report) {
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

__device__ __forceinline__ const uint8_t* q_image(const DecodeArgs& a, int b) {
  return a.q_img + (static_cast<int64_t>(b) * gridDim.z + blockIdx.z) * kQImageBytes;
}

// ---------------------------------------------------------------------------
// Stage producer (warp 0, lane 0; both CTAs)
// ---------------------------------------------------------------------------
// Tile j's nibbles and scales go to stage j % 3 once the stage's previous tile
// is done with.  CTA 0 also loads each piece's Q image (when the Q prep kernel
// wrote one) after its first tile's loads, once the previous piece's last QK
// is complete, and prefetches later tiles into L2 (CTA 1's loads of the same
// bytes then hit L2).
__device__ void producer(uint8_t* sm, Misc& ms, const Sched& sc, const DecodeArgs& a, const CacheMaps& maps,
                         bool qk_cta) {
  prefetch_tensormap(&maps.kv);
  prefetch_tensormap(&maps.sc);
  uint8_t* stages = sm + (qk_cta ? kOffStage0 : kOffStage1);
  Cursor cur, pc;  // tile j; L2 prefetch
  cursor_start(a, sc, cur);
  pc = cur;
  cursor_next(a, pc);
  cursor_next(a, pc);
  int prefetched = 2;
  // each call reads the page ids of at most two more tiles (those reads stall this thread)
  auto prefetch_upto = [&](int upto) {
    upto = min(upto, prefetched + 2);
    while (prefetched < min(upto, sc.count)) {
      int y[2];
      tile_rows(a, pc, y, false);
#pragma unroll
      for (int slot = 0; slot < 2; ++slot) {
        if (y[slot] >= 0) {
          prefetch_l2(a.kv_buffer + static_cast<int64_t>(y[slot]) * kTokenBytes, kPageBytes);
          prefetch_l2(a.kv_scales + static_cast<int64_t>(y[slot]) * kScaleBytes, kPageScaleBytes);
        }
      }
      ++prefetched;
      cursor_next(a, pc);
    }
  };
  int issued = 0, q_issued = 0, pieces = 0;
  bool grid_waited = false;
  for (int j = 0; j < sc.count; ++j, cursor_next(a, cur)) {
    const int s = j % kStages;
    if (j >= kStages && !wait_phase(&ms.mb_stage_free[s], static_cast<uint32_t>((j / kStages - 1) & 1), ms, a,
                                    kStatusProducerWait))
      break;
    int y[2];
    tile_rows(a, cur, y, qk_cta);
    const int slots = (y[0] != -1 ? 1 : 0) + (y[1] != -1 ? 1 : 0);
    uint8_t* stage = stages + s * kStageBytes;
    mbar_arrive_expect_tx(&ms.mb_stage_full[s], static_cast<uint32_t>(slots * (2 * 64 * 128 + kPageScaleBytes)));
#pragma unroll
    for (int slot = 0; slot < 2; ++slot) {
      if (y[slot] == -1) continue;
      tma_load_2d(stage + kStageNib + slot * kPageScaleBytes, &maps.sc, 0, y[slot], &ms.mb_stage_full[s]);
      tma_load_2d(stage + slot * (64 * 128), &maps.kv, 0, y[slot], &ms.mb_stage_full[s]);
      tma_load_2d(stage + kNibBlock + slot * (64 * 128), &maps.kv, 128, y[slot], &ms.mb_stage_full[s]);
    }
    issued = j + 1;
    if (qk_cta && cursor_first(cur)) {
      if (a.q_img) {
        if (pieces > 0 &&
            !wait_phase(&ms.mb_q_free, static_cast<uint32_t>((pieces - 1) & 1), ms, a, kStatusProducerWait))
          break;
        if (!grid_waited) {
          asm volatile("griddepcontrol.wait;\n" ::: "memory");  // the Q prep grid is complete
          grid_waited = true;
        }
        mbar_arrive_expect_tx(&ms.mb_q_full, kQImageBytes);
        bulk_load(sm + kOffQ, q_image(a, cur.b), kQImageBytes, &ms.mb_q_full);
        ++q_issued;
      }
      ++pieces;
    }
    if (qk_cta) prefetch_upto(j + kStages + kPrefetchTiles);
  }
  // every copy issued has landed before the CTA may exit (normally the
  // consumers have already waited for all of them)
  for (int j = max(0, issued - kStages); j < issued; ++j)
    drain_wait(&ms.mb_stage_full[j % kStages], static_cast<uint32_t>((j / kStages) & 1));
  if (q_issued > 0) drain_wait(&ms.mb_q_full, static_cast<uint32_t>((q_issued - 1) & 1));
}

// k_pe producer (CTA 0 warp 2, lane 0): tile j's k_pe into buffer j % 2 once
// the RoPE MMAs of tile j - 2 are complete.
__device__ void kpe_producer(uint8_t* sm, Misc& ms, const Sched& sc, const DecodeArgs& a, const CacheMaps& maps) {
  Cursor cur;
  cursor_start(a, sc, cur);
  int issued = 0;
  for (int j = 0; j < sc.count; ++j, cursor_next(a, cur)) {
    const int b = j & 1;
    if (j >= 2 && !wait_phase(&ms.mb_kpe_free[b], static_cast<uint32_t>(((j - 2) >> 1) & 1), ms, a,
                              kStatusProducerWait))
      break;
    int y[2];
    tile_rows(a, cur, y, false);
    const int slots = (y[0] != -1 ? 1 : 0) + (y[1] != -1 ? 1 : 0);
    mbar_arrive_expect_tx(&ms.mb_kpe_full[b], static_cast<uint32_t>(slots * 64 * 128));
#pragma unroll
    for (int slot = 0; slot < 2; ++slot)
      if (y[slot] != -1)
        tma_load_2d(sm + kOffKpe + b * (128 * 128) + slot * (64 * 128), &maps.kv, kNibbleBytes, y[slot],
                    &ms.mb_kpe_full[b]);
    issued = j + 1;
  }
  for (int j = max(0, issued - 2); j < issued; ++j)
    drain_wait(&ms.mb_kpe_full[j & 1], static_cast<uint32_t>((j >> 1) & 1));
}

// ---------------------------------------------------------------------------
// Scale warps (warp 3)
// ---------------------------------------------------------------------------
// CTA 0: once tile j's stage lands, regroup its token-major e8m0 rows in place
// into the tcgen05.cp order of the A scale factors (lane l reads tokens l,
// l + 32, l + 64, l + 96 and writes back the same four 16-byte rows: word k4
// of each token goes to block k4, row l); tokens past the sequence end get
// scale 1 (their scores are masked).
__device__ void scale_warp_qk(uint8_t* sm, Misc& ms, const Sched& sc, int lane, const DecodeArgs& a) {
  Cursor cur;
  cursor_start(a, sc, cur);
  for (int j = 0; j < sc.count; ++j, cursor_next(a, cur)) {
    const int s = j % kStages;
    if (!warp_wait(&ms.mb_stage_full[s], static_cast<uint32_t>((j / kStages) & 1), ms, a, kStatusScaleWait, lane))
      break;
    uint8_t* scb = sm + kOffStage0 + s * kStageBytes + kStageNib;
    const int nvalid = cursor_valid(cur);
    uint4 w[4];
#pragma unroll
    for (int m1 = 0; m1 < 4; ++m1) {
      const int t = lane + 32 * m1;
      w[m1] = t < nvalid ? *reinterpret_cast<const uint4*>(scb + t * kScaleBytes)
                         : make_uint4(0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu);
    }
    uint8_t* dst = scb + lane * 16;
    *reinterpret_cast<uint4*>(dst + 0 * 512) = make_uint4(w[0].x, w[1].x, w[2].x, w[3].x);
    *reinterpret_cast<uint4*>(dst + 1 * 512) = make_uint4(w[0].y, w[1].y, w[2].y, w[3].y);
    *reinterpret_cast<uint4*>(dst + 2 * 512) = make_uint4(w[0].z, w[1].z, w[2].z, w[3].z);
    *reinterpret_cast<uint4*>(dst + 3 * 512) = make_uint4(w[0].w, w[1].w, w[2].w, w[3].w);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(&ms.mb_sfa[s]);
  }
}

// CTA 1: once tile j's stage lands, the tile maximum of the valid tokens' e8m0
// bytes gives the tile's reference exponent sigma (the piece's first tile
// sets it so the maximum maps to <= 6 * 2^8 in V''; later tiles keep it while
// their maximum stays within the exact e5m2 range); published for the
// converters and the epilogue warps.
__device__ void scale_warp_pv(uint8_t* sm, Misc& ms, const Sched& sc, int lane, const DecodeArgs& a) {
  Cursor cur;
  cursor_start(a, sc, cur);
  int sigma_prev = 0;
  for (int j = 0; j < sc.count; ++j, cursor_next(a, cur)) {
    const int s = j % kStages;
    if (!warp_wait(&ms.mb_stage_full[s], static_cast<uint32_t>((j / kStages) & 1), ms, a, kStatusScaleWait, lane))
      break;
    const uint8_t* scb = sm + kOffStage1 + s * kStageBytes + kStageNib;
    const int nvalid = cursor_valid(cur);
    uint32_t mx = 0u;
#pragma unroll
    for (int m1 = 0; m1 < 4; ++m1) {
      const int t = lane + 32 * m1;
      if (t < nvalid) {
        const uint4 w = *reinterpret_cast<const uint4*>(scb + t * kScaleBytes);
        mx = __vmaxu4(mx, __vmaxu4(__vmaxu4(w.x, w.y), __vmaxu4(w.z, w.w)));
      }
    }
    mx = max(max(mx & 0xFFu, (mx >> 8) & 0xFFu), max((mx >> 16) & 0xFFu, mx >> 24));
    const int smax = static_cast<int>(__reduce_max_sync(0xffffffffu, mx));
    int sigma;
    if (cursor_first(cur)) {
      sigma = smax - 127 - 8;
    } else {
      const int kmax = smax - 127 - sigma_prev;
      sigma = (kmax > 13 || kmax < -4) ? smax - 127 - 8 : sigma_prev;
    }
    sigma_prev = sigma;
    __syncwarp();
    if (lane == 0) {
      ms.sig[j & 3] = sigma;
      mbar_arrive(&ms.mb_sig[j & 3]);
      mbar_arrive(&ms.mb_stage_free[s]);
    }
  }
}

// ---------------------------------------------------------------------------
// CTA 0 MMA thread (warp 1, lane 0): QK(j) into S buffer j % 2
// ---------------------------------------------------------------------------
__device__ void mma_qk(uint8_t* sm, Misc& ms, uint32_t tmem, const Sched& sc, int lane, const DecodeArgs& a) {
  if (lane != 0) return;
  const uint32_t id_pe = instr_desc(kFmtBF16, kFmtBF16, false, false, 128, 64);
  // Base descriptors; an operand at byte offset `off` from a base is the base
  // descriptor + off / 16 (the start-address field; shared memory addresses
  // stay below 2^18, so there is no carry).
  const uint64_t dQ = smem_desc(smem_addr(sm + kOffQ), 16, 1024, kSwizzle128B);
  const uint64_t dQpe = smem_desc(smem_addr(sm + kOffQpe), 16, 1024, kSwizzle128B);
  const uint64_t dQsf = smem_desc(smem_addr(sm + kOffQsf), 128, 128, kSwizzleNone);
  const uint64_t dKpe = smem_desc(smem_addr(sm + kOffKpe), 16, 1024, kSwizzle128B);
  const uint64_t dSfa = smem_desc(smem_addr(sm + kOffStage0 + kStageNib), 128, 128, kSwizzleNone);
  const uint64_t dNib = smem_desc(smem_addr(sm + kOffStage0), 16, 1024, kSwizzle128B);
  Cursor cur;
  cursor_start(a, sc, cur);
  int pieces = 0;
  for (int j = 0; j < sc.count; ++j, cursor_next(a, cur)) {
    const int s = j % kStages, b = j & 1;
    if (cursor_first(cur)) {
      if (!wait_phase(&ms.mb_q_full, static_cast<uint32_t>(pieces & 1), ms, a, kStatusIssuerWait)) break;
      ++pieces;
      fence_after_sync();
      // B scale factors of the Q terms (the previous piece's QKs are complete)
#pragma unroll
      for (int blk = 0; blk < 8; ++blk)
        tmem_cp_32x128b_x4(tmem + kColSfb + 8 * (blk >> 1) + 4 * (blk & 1), dQsf + 32 * blk);
    }
    if (j >= 2 && !wait_phase(&ms.mb_s_free[b], static_cast<uint32_t>(((j - 2) >> 1) & 1), ms, a, kStatusIssuerWait))
      break;
    if (!wait_phase(&ms.mb_kpe_full[b], static_cast<uint32_t>((j >> 1) & 1), ms, a, kStatusIssuerWait) ||
        !wait_phase(&ms.mb_sfa[s], static_cast<uint32_t>((j / kStages) & 1), ms, a, kStatusIssuerWait))
      break;
    fence_after_sync();
    const uint32_t sfa0 = tmem + kColSfa + 16 * b, sfb0 = tmem + kColSfb, dS = tmem + kColS + 192 * b;
#pragma unroll
    for (int k4 = 0; k4 < 4; ++k4) tmem_cp_32x128b_x4(sfa0 + 4 * k4, dSfa + ((s * kStageBytes + 512 * k4) >> 4));
    // RoPE first: S[:, 0:64) = k_pe . q_pe^T
#pragma unroll
    for (int k = 0; k < 4; ++k)
      mma_f16_ss(dS, dKpe + ((b * 128 * 128) >> 4) + 2 * k, dQpe + 2 * k, id_pe, k > 0 ? 1u : 0u);
    mma_commit(&ms.mb_kpe_free[b]);
    // latent: 8 K steps of 64; the first adds onto the RoPE columns (term 0)
    // and starts the columns of terms 1 and 2
    const uint64_t da0 = dNib + ((s * kStageBytes) >> 4);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const uint32_t koff = ((k >> 2) * kNibBlock + (k & 3) * 32) >> 4;
      const uint32_t qoff = ((k >> 2) * (kQTermBytes / 2) + (k & 3) * 32) >> 4;
      const uint32_t byte = 2 * (k & 1);
      const uint32_t sfa = (sfa0 + 4 * (k >> 1)) | (byte << 30);
      const uint32_t sfb = (sfb0 + 8 * (k >> 1)) | (byte << 30);
      if (k == 0) {
        mma_mxf4_ss(dS, da0 + koff, dQ + qoff, instr_desc_mxf4(64, byte, byte), sfa, sfb, 1u);
        mma_mxf4_ss(dS + 64, da0 + koff, dQ + qoff + (8 * 1024 >> 4), instr_desc_mxf4(128, byte, byte), sfa,
                    (sfb0 + 2) | (byte << 30), 0u);
      } else {
        mma_mxf4_ss(dS, da0 + koff, dQ + qoff, instr_desc_mxf4(192, byte, byte), sfa, sfb, 1u);
      }
    }
    mma_commit(&ms.mb_s_full[b]);
    mma_commit(&ms.mb_stage_free[s]);
    if (cursor_last(cur)) mma_commit(&ms.mb_q_free);
  }
}

// ---------------------------------------------------------------------------
// Q of one sequence: the three e2m1 terms of a 32-element block of one head
// (thread (h, bl)), written as the QK operand images: the terms at qdst (the
// layout of kOffQ) and their scales at sfdst in tcgen05.cp order
// (q_sf_offset).  Used by the Q prep kernel (global memory) and, without a
// workspace, by the decode kernel's softmax warps (shared memory).
// ---------------------------------------------------------------------------
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
    const int n = 64 * t + h;
    *reinterpret_cast<uint4*>(qdst + (bl >> 3) * (kQTermBytes / 2) + (n >> 3) * 1024 + sw128_offset(n & 7, bl & 7)) =
        make_uint4(w[0], w[1], w[2], w[3]);
    sfdst[q_sf_offset(n, bl)] = static_cast<uint8_t>(e + 127);
  }
}

// All of a sequence's Q operands with 256 threads (4 per head; part p
// handles the 32-element blocks 4p .. 4p + 3 and the q_pe chunks 2p, 2p + 1).
__device__ void q_operands(const DecodeArgs& a, int b, int head_base, int heads_here, int tid, uint8_t* img) {
  const int h = tid >> 2, part = tid & 3;
  const bool live = h < heads_here;
  const __nv_bfloat16* qrow = a.q + b * a.q_stride_b + (head_base + h) * a.q_stride_h;
#pragma unroll 1
  for (int blk = 0; blk < 4; ++blk) {
    uint4 v[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) v[k] = ldg_stream_if(qrow + 32 * (4 * part + blk) + 8 * k, live);
    q_block(v, h, 4 * part + blk, img, img + kQTermBytes + kQPeBytes);
  }
#pragma unroll
  for (int k = 0; k < 2; ++k)
    *reinterpret_cast<uint4*>(img + kQTermBytes + (h >> 3) * 1024 + sw128_offset(h & 7, 2 * part + k)) =
        ldg_stream_if(qrow + kLatent + 8 * (2 * part + k), live);
}


// ---------------------------------------------------------------------------
// CTA 0 softmax warps (4..11)
// ---------------------------------------------------------------------------
// Thread (warp w, lane l): token row 32 (w % 4) + l of S, heads 32 hf ..
// 32 hf + 31 (hf = (w - 4) / 4).  P'' goes into CTA 1's buffer j % 2 as token
// rows of 128 bytes (hi terms of heads 0..63, then lo terms), 128-byte
// swizzled atoms of 8 tokens: the MN-major A operand of CTA 1's PV MMAs.
__device__ void softmax_qk(uint8_t* sm, Misc& ms, uint32_t tmem, const Sched& sc, int head_base, int heads_here,
                           int warp, int lane, float c_log2, const DecodeArgs& a) {
  const int tid = threadIdx.x - 32 * kSoftmaxWarp0;  // 0..255
  const int q = warp & 3;                             // TMEM lane quadrant = token quarter
  const int hf = (warp - kSoftmaxWarp0) >> 2;         // heads 32 hf .. 32 hf + 31
  const int st = 32 * q + lane;                       // softmax token
  const uint32_t lane_base = static_cast<uint32_t>(32 * q) << 16;
  // CTA 1's P'' buffers, event records, piece record and their mbarriers
  const uint32_t rP = map_to_rank(smem_addr(sm + kOffP), 1);
  const uint32_t rAlpha = map_to_rank(smem_addr(&ms.info_alpha[0][0]), 1);
  const uint32_t rEvent = map_to_rank(smem_addr(&ms.info_event[0]), 1);
  const uint32_t rStatL = map_to_rank(smem_addr(&ms.stat_l[0]), 1);
  const uint32_t rStatR = map_to_rank(smem_addr(&ms.stat_r[0]), 1);
  const uint32_t rPFull = map_to_rank(smem_addr(&ms.mb_p_full[0][0]), 1);
  const uint32_t rInfoFull = map_to_rank(smem_addr(&ms.mb_info_full[0]), 1);
  const uint32_t rStatsFull = map_to_rank(smem_addr(&ms.mb_stats_full), 1);
  // this thread's four 16-byte pieces of its token row: hi chunks 2 hf, 2 hf + 1, lo chunks 4 + 2 hf, 5 + 2 hf
  const uint32_t prow = q * 4096 + (lane >> 3) * 1024;

  float l_part[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) l_part[j] = 0.f;
  int pieces = 0;
  Cursor cur;
  cursor_start(a, sc, cur);

  for (int tile = 0; tile < sc.count; ++tile, cursor_next(a, cur)) {
    const int b = tile & 1;
    const uint32_t par = static_cast<uint32_t>((tile >> 1) & 1);
    const bool first = cursor_first(cur);
    if (first) {
      // A new sequence.  Without Q images in the workspace (one split, so one
      // piece per pair) its Q operands are quantised here.
      if (!a.q_img) {
        q_operands(a, cur.b, head_base, heads_here, tid, sm + kOffQ);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&ms.mb_q_full);
      }
      if (tid < kNH) ms.R[tid] = 0.f;
      named_bar(kBarSoftmax, kSoftmaxThreads);  // R of the new sequence is visible
    }
    bool ok = warp_wait(&ms.mb_s_full[b], par, ms, a, kStatusSoftmaxWait, lane);
    fence_after_sync();
    float t[32];
    if (ok) {
      uint32_t sv[32];
      const uint32_t sb = tmem + lane_base + kColS + 192 * b + 32 * hf;
      tmem_ld32(sb, sv);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 32; ++j) t[j] = __uint_as_float(sv[j]);
      tmem_ld32(sb + 64, sv);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 32; ++j) t[j] += __uint_as_float(sv[j]);
      tmem_ld32(sb + 128, sv);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 32; ++j) t[j] += __uint_as_float(sv[j]);
      fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ms.mb_s_free[b]);
      const bool tvalid = st < cursor_valid(cur);
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        const float4 r4 = *reinterpret_cast<const float4*>(&ms.R[32 * hf + j]);
        const float rv[4] = {r4.x, r4.y, r4.z, r4.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) t[j + u] = tvalid ? fmaf(t[j + u], c_log2, -rv[u]) : -CUDART_INF_F;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) t[j] = -CUDART_INF_F;
    }
    // CTA 1's P'' buffer b and event record b are free once its PV of tile
    // j - 2 is complete
    if (ok && tile >= 2)
      ok = warp_wait_cluster(&ms.mb_p_free[b], static_cast<uint32_t>(((tile - 2) >> 1) & 1), ms, a,
                             kStatusSoftmaxPvWait, lane);
    // rescale event: a piece's first tile or a score above R + 8.5.  One
    // barrier ORs "event or failure"; only when it is raised does a second
    // one tell a failure (leave the loop) from an event.
    float tmaxv = -CUDART_INF_F;
#pragma unroll
    for (int j = 0; j < 32; ++j) tmaxv = fmaxf(tmaxv, t[j]);
    const bool need = bar_or(kBarSoftmax, kSoftmaxThreads, !ok || first || tmaxv > 8.5f);
    if (need && bar_or(kBarSoftmax, kSoftmaxThreads, !ok)) break;
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
        const float alpha = first ? 1.0f : ex2(-dshift);
        ms.red[1][tid] = alpha;   // factor of the sums and of O
        ms.red[0][tid] = dshift;  // per-head shift of t
        if (!first) st_cluster_f32(rAlpha + 4 * (b * kNH + tid), alpha);
      }
      named_bar(kBarSoftmax, kSoftmaxThreads);
#pragma unroll
      for (int j = 0; j < 32; ++j) t[j] -= ms.red[0][32 * hf + j];
      if (!first) {
#pragma unroll
        for (int j = 0; j < 32; ++j) l_part[j] *= ms.red[1][32 * hf + j];
      }
      // every thread has read red before the next event overwrites it
      named_bar(kBarSoftmax, kSoftmaxThreads);
    }
    if (tid == 0) {
      // the tile's event record: CTA 1 rescales O by alpha before this tile's PV
      st_cluster_u32(rEvent + 4 * b, (need && !first) ? 1u : 0u);
      mbar_arrive_remote(rInfoFull + 8 * b);
    }

    // ---- P'' = exp2(t) as e4m3 hi + residual, into CTA 1's buffer b ----
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
      const uint32_t base = rP + b * kPBuf + prow;
      const uint32_t row = lane & 7;
      st_cluster_v4(base + sw128_offset(row, 2 * hf), make_uint4(pw[0], pw[1], pw[2], pw[3]));
      st_cluster_v4(base + sw128_offset(row, 2 * hf + 1), make_uint4(pw[4], pw[5], pw[6], pw[7]));
      st_cluster_v4(base + sw128_offset(row, 4 + 2 * hf), make_uint4(pl[0], pl[1], pl[2], pl[3]));
      st_cluster_v4(base + sw128_offset(row, 5 + 2 * hf), make_uint4(pl[4], pl[5], pl[6], pl[7]));
    }
    asm volatile("fence.proxy.async.shared::cluster;\n" ::: "memory");
    __syncwarp();
    if (lane == 0) mbar_arrive_remote(rPFull + 8 * (4 * b + q));

    if (!cursor_last(cur)) continue;
    // ---------------- the piece's record for CTA 1 ----------------
    {
      const float s = warp_transpose_reduce<false>(l_part, lane);
      ms.red[q][32 * hf + lane] = s;
    }
#pragma unroll
    for (int j = 0; j < 32; ++j) l_part[j] = 0.f;
    const bool free_ok =
        pieces == 0 ||
        warp_wait_cluster(&ms.mb_stats_free, static_cast<uint32_t>((pieces - 1) & 1), ms, a, kStatusEpilogueWait, lane);
    named_bar(kBarSoftmax, kSoftmaxThreads);
    if (tid < kNH) {
      const float l = ms.red[0][tid] + ms.red[1][tid] + ms.red[2][tid] + ms.red[3][tid];
      st_cluster_f32(rStatL + 4 * tid, l);
      st_cluster_f32(rStatR + 4 * tid, ms.R[tid]);
    }
    if (bar_or(kBarSoftmax, kSoftmaxThreads, !free_ok)) break;
    if (tid == 0) mbar_arrive_remote(rStatsFull);
    ++pieces;
    named_bar(kBarSoftmax, kSoftmaxThreads);  // red is free again
  }
}

// ---------------------------------------------------------------------------
// CTA 1 MMA thread (warp 1, lane 0): PV(j) = 8 MMAs, M = 128 (hi and lo rows
// of 64 heads), N = 256 (a latent half), K = 32 tokens
// ---------------------------------------------------------------------------
__device__ void mma_pv(uint8_t* sm, Misc& ms, uint32_t tmem, const Sched& sc, int lane, const DecodeArgs& a) {
  if (lane != 0) return;
  const uint32_t id_pv = instr_desc(kFmtE4M3, kFmtE5M2, true, true, 128, 256);
  // A: P'' token rows of 128 bytes (M), 8-token atoms along K 1 KB apart.
  // B: V'' token rows of 128 latents per 4 KB chunk (N atoms 4 KB apart),
  // 8-token atoms along K 1 KB apart.
  const uint64_t dP = smem_desc(smem_addr(sm + kOffP), kPBuf, 1024, kSwizzle128B);
  const uint64_t dV = smem_desc(smem_addr(sm + kOffV), kVChunk, 1024, kSwizzle128B);
  Cursor cur;
  cursor_start(a, sc, cur);
  for (int j = 0; j < sc.count; ++j, cursor_next(a, cur)) {
    const int b = j & 1;
    const uint32_t par = static_cast<uint32_t>((j >> 1) & 1);
    const bool first = cursor_first(cur);
    if (!wait_phase(&ms.mb_o_ready[b], par, ms, a, kStatusIssuerPvWait)) break;
    bool ok = true;
#pragma unroll 1
    for (int k = 0; k < 4; ++k) {
      ok = wait_phase_cluster(&ms.mb_p_full[b][k], par, ms, a, kStatusIssuerPvWait) &&
           wait_phase(&ms.mb_v_full[k], static_cast<uint32_t>(j & 1), ms, a, kStatusIssuerPvWait);
      if (!ok) break;
      fence_proxy_async_smem();  // P'' came from the other CTA's generic stores
      fence_after_sync();
      const uint64_t pa = dP + ((b * kPBuf + k * 4096) >> 4);
      const uint32_t acc = (first && k == 0) ? 0u : 1u;  // the piece's first PV starts the accumulator
#pragma unroll
      for (int h = 0; h < 2; ++h) mma_f8f6f4_ss(tmem + 256 * h, pa, dV + ((k * kVSlot + h * 2 * kVChunk) >> 4), id_pv, acc);
      mma_commit(&ms.mb_pv_done[k]);
    }
    if (!ok) break;
    mma_commit(&ms.mb_tile_done[b]);             // the epilogue may rescale or read O
    mma_commit_multicast(&ms.mb_p_free[b], 1);  // CTA 0 may refill P'' buffer b
  }
}

// ---------------------------------------------------------------------------
// CTA 1 converters (warps 8..15)
// ---------------------------------------------------------------------------
// V''(j) one token quarter at a time into ring slot k, each once PV(j - 1) of
// that quarter is complete.  Warp lw converts 4 tokens of the quarter's
// 8-token atom lw / 2, rows {0, 2, 5, 7} (lw even) or {1, 3, 4, 6} (lw odd);
// lane l the 32-element groups 8h + c, h = 0, 1, with c % 4 = l % 4 (bits
// 0-1), c / 4 = bit 4, and the row chosen by bits 2-3.  Every 8-lane phase of
// a 16-byte access then meets 8 distinct bank groups, for the swizzled nibble
// loads (c ^ row) and the V'' stores (2 (c % 4) ^ row) alike.
__device__ void converter(uint8_t* sm, Misc& ms, const Sched& sc, int warp, int lane, const DecodeArgs& a) {
  const int lw = warp - kConvWarp0;
  const int c = (lane & 3) | ((lane >> 2) & 4);
  const int row = ((2 * ((lane >> 3) & 1)) | (lw & 1)) ^ (5 * ((lane >> 2) & 1));
  Cursor cur;
  cursor_start(a, sc, cur);
  for (int j = 0; j < sc.count; ++j, cursor_next(a, cur)) {
    const int s = j % kStages;
    if (!warp_wait(&ms.mb_sig[j & 3], static_cast<uint32_t>((j >> 2) & 1), ms, a, kStatusConverterWait, lane) ||
        !warp_wait(&ms.mb_stage_full[s], static_cast<uint32_t>((j / kStages) & 1), ms, a, kStatusConverterWait, lane))
      break;
    const int sigma = ms.sig[j & 3];
    const int nvalid = cursor_valid(cur);
    const uint8_t* nib = sm + kOffStage1 + s * kStageBytes;
    const uint8_t* scb = nib + kStageNib;
    bool ok = true;
#pragma unroll 1
    for (int k = 0; k < 4; ++k) {
      if (j > 0 && !warp_wait(&ms.mb_pv_done[k], static_cast<uint32_t>((j - 1) & 1), ms, a, kStatusConverterWait,
                              lane)) {
        ok = false;
        break;
      }
      const int t = 32 * k + 8 * (lw >> 1) + row;
      uint8_t* atom = sm + kOffV + k * kVSlot + (lw >> 1) * 1024;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint4 nb = *reinterpret_cast<const uint4*>(nib + h * kNibBlock + (t >> 3) * 1024 + sw128_offset(row, c));
        const int sbyte = scb[t * kScaleBytes + 8 * h + c];
        uint32_t lo, hi;
        e5m2_tables(sbyte - 127 - sigma, lo, hi);
        uint4 o0 = half_group_to_e5m2(nb.x, nb.y, lo, hi);
        uint4 o1 = half_group_to_e5m2(nb.z, nb.w, lo, hi);
        if (t >= nvalid) o0 = o1 = make_uint4(0u, 0u, 0u, 0u);
        uint8_t* dst = atom + (2 * h + (c >> 2)) * kVChunk;
        *reinterpret_cast<uint4*>(dst + sw128_offset(row, 2 * (c & 3))) = o0;
        *reinterpret_cast<uint4*>(dst + sw128_offset(row, 2 * (c & 3) + 1)) = o1;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ms.mb_v_full[k]);
    }
    if (!ok) break;
    __syncwarp();
    if (lane == 0) mbar_arrive(&ms.mb_stage_free[s]);
  }
}

// ---------------------------------------------------------------------------
// CTA 1 epilogue warps (4..7): O rescales and each piece's output
// ---------------------------------------------------------------------------
// Warp 4 + w owns TMEM lanes 32 w .. 32 w + 31 of O_hl: lanes 0..63 hold the
// hi-term sums of heads 0..63, lanes 64..127 the lo-term sums.  Before each
// tile's PV: if CTA 0 moved R (event record) or sigma moved, O_hl is scaled by
// alpha[head] * 2^(sigma_prev - sigma) once PV(j - 1) is complete.  At a
// piece's end: O = (hi + lo) * 2^sigma / l, the lo half passed through
// shared memory.
//
// Both waits for a PV are on tile_done[t % 2] (tile t's commit), not on
// pv_done[3]: a parity wait names the right phase only while the barrier is
// at most one phase past the one waited for, and these warps wait only on
// some tiles.  Slot t % 2 has tiles t - 2 and t + 2 on either side: tile t - 2
// is complete before CTA 0 sends tile t's event record (which it does after
// PV(t - 2)'s later p_free commit), and PV(t + 2) cannot start before these
// warps' o_ready for it.  pv_done[3], waited on only now and then, could
// already be a phase behind (PV(j - 1) in flight) and match tile j - 2.
__device__ void epilogue_pv(uint8_t* sm, Misc& ms, uint32_t tmem, const Sched& sc, int head_base, int heads_here,
                            int warp, int lane, const DecodeArgs& a) {
  const int w = warp - kEpiWarp0;
  const uint32_t lane_base = static_cast<uint32_t>(32 * w) << 16;
  const int head = (32 * w + lane) & (kNH - 1);
  const bool lo_row = w >= 2;
  float* stage = reinterpret_cast<float*>(sm + kOffEpi + (w & 1) * 4096);  // [32 columns][32 lanes]
  const uint32_t rStatsFree = map_to_rank(smem_addr(&ms.mb_stats_free), 0);
  int sigma_prev = 0, pieces = 0;
  Cursor cur;
  cursor_start(a, sc, cur);
  for (int j = 0; j < sc.count; ++j, cursor_next(a, cur)) {
    const int b = j & 1;
    const bool first = cursor_first(cur);
    // every exit is decided by all four warps at once (they share a named barrier)
    const bool ok0 =
        warp_wait_cluster(&ms.mb_info_full[b], static_cast<uint32_t>((j >> 1) & 1), ms, a, kStatusEpilogueWait,
                          lane) &&
        warp_wait(&ms.mb_sig[j & 3], static_cast<uint32_t>((j >> 2) & 1), ms, a, kStatusEpilogueWait, lane);
    if (bar_or(kBarEpi, kEpiThreads, !ok0)) break;
    const int sigma = ms.sig[j & 3];
    const bool ev = ms.info_event[b] != 0;
    if (!first && (ev || sigma != sigma_prev)) {
      const bool ok1 = warp_wait(&ms.mb_tile_done[(j - 1) & 1], static_cast<uint32_t>(((j - 1) >> 1) & 1), ms, a,
                                 kStatusEpilogueWait, lane);
      if (bar_or(kBarEpi, kEpiThreads, !ok1)) break;
      fence_after_sync();
      const float f = (ev ? ms.info_alpha[b][head] : 1.0f) * ex2(static_cast<float>(sigma_prev - sigma));
#pragma unroll 1
      for (int cb = 0; cb < 16; ++cb) {
        uint32_t vv[32];
        tmem_ld32(tmem + lane_base + 32 * cb, vv);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) vv[i] = __float_as_uint(__uint_as_float(vv[i]) * f);
        tmem_st32(tmem + lane_base + 32 * cb, vv);
      }
      tmem_st_wait();
    }
    fence_before_sync();
    __syncwarp();
    if (lane == 0) mbar_arrive(&ms.mb_o_ready[b]);
    sigma_prev = sigma;
    if (!cursor_last(cur)) continue;

    // ---------------- epilogue of the piece ----------------
    const bool ok =
        warp_wait(&ms.mb_tile_done[b], static_cast<uint32_t>((j >> 1) & 1), ms, a, kStatusEpilogueWait, lane) &&
        warp_wait_cluster(&ms.mb_stats_full, static_cast<uint32_t>(pieces & 1), ms, a, kStatusEpilogueWait, lane);
    if (bar_or(kBarEpi, kEpiThreads, !ok)) break;
    fence_after_sync();
    const float l = ms.stat_l[head], rr = ms.stat_r[head];
    named_bar(kBarEpi, kEpiThreads);  // the piece record is read
    if (threadIdx.x == 32 * kEpiWarp0) mbar_arrive_remote(rStatsFree);
    ++pieces;
    // the piece covers its whole sequence -> final output; otherwise a partial in its slot
    const int pair = blockIdx.x >> 1;
    const bool direct = a.balanced ? (cur.piece_begin == 0 && cur.piece_end == cursor_tiles(cur))
                                   : a.num_splits == 1;
    const int64_t slot = a.balanced ? static_cast<int64_t>(cur.b) + pair
                                    : static_cast<int64_t>(cur.b) * a.num_splits + pair;
    const float factor = l > 0.f ? exp2f(static_cast<float>(sigma)) / l : 0.f;
    if (!lo_row && !direct && head < heads_here)
      a.partial_lse[slot * a.num_heads + head_base + head] = (rr + __log2f(l)) * kLn2;
    if (a.balanced && threadIdx.x == 32 * kEpiWarp0 && cur.piece_begin == 0) {
      // this pair holds the sequence's first tile: record its pair span for the merge
      const int last_pair = cta_of_tile(cur.seq_pos + cursor_tiles(cur) - 1, sc, gridDim.x >> 1);
      a.seq_meta[cur.b] = make_int2(pair, last_pair);
    }
    const bool vec = !direct || ((reinterpret_cast<uintptr_t>(a.o) | static_cast<uintptr_t>(a.o_stride_b * 2) |
                                  static_cast<uintptr_t>(a.o_stride_h * 2)) & 15) == 0;
    const int hq = head_base + head;
    __nv_bfloat16* orow = direct ? a.o + cur.b * a.o_stride_b + hq * a.o_stride_h
                                 : a.partial_o + (slot * a.num_heads + hq) * kLatent;
#pragma unroll 1
    for (int cb = 0; cb < 16; ++cb) {
      uint32_t vv[32];
      tmem_ld32(tmem + lane_base + 32 * cb, vv);
      tmem_ld_wait();
      if (lo_row) {
#pragma unroll
        for (int i = 0; i < 32; ++i) stage[32 * i + lane] = __uint_as_float(vv[i]);
      }
      named_bar(kBarEpi, kEpiThreads);
      if (!lo_row && head < heads_here) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float x0 = (__uint_as_float(vv[2 * i]) + stage[32 * (2 * i) + lane]) * factor;
          const float x1 = (__uint_as_float(vv[2 * i + 1]) + stage[32 * (2 * i + 1) + lane]) * factor;
          pk[i] = static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(x0))) |
                  (static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(x1))) << 16);
        }
        __nv_bfloat16* dst = orow + 32 * cb;
        if (vec) {
#pragma unroll
          for (int i = 0; i < 4; ++i)
            reinterpret_cast<uint4*>(dst)[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) reinterpret_cast<uint32_t*>(dst)[i] = pk[i];
        }
      }
      named_bar(kBarEpi, kEpiThreads);  // the stage is rewritten by the next unit
    }
    fence_before_sync();
  }
}

__global__ void __launch_bounds__(kThreads, 1) mla_decode_fp4_kernel(const __grid_constant__ DecodeArgs a,
                                                                  const __grid_constant__ CacheMaps maps) {
  // the merge kernel (launched next as a programmatic dependent) may be
  // scheduled once every CTA of this grid runs; it waits for this grid to
  // complete before reading anything
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
  uint8_t* sm = smem_base();
  Misc& ms = *reinterpret_cast<Misc*>(sm);
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const bool qk_cta = cluster_ctarank() == 0;
  const int pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;
  const int head_base = blockIdx.z * kNH;
  const int heads_here = min(kNH, a.num_heads - head_base);

  // Both CTAs of a pair compute the same run, so they leave here together.
  Sched sc;
  if (a.balanced) {
    balanced_schedule<kThreads>(a, ms.sched, sc, pairs, pair);
    if (sc.count == 0) {
      // An empty run (fewer tiles than pairs) can sit inside the pair span of
      // the sequence at its position; its slot of that sequence carries no weight.
      if (!qk_cta && sc.pos0 < sc.total && tid < heads_here)
        a.partial_lse[(static_cast<int64_t>(sc.b0) + pair) * a.num_heads + head_base + tid] = -CUDART_INF_F;
      return;
    }
  } else {
    const int b = blockIdx.y, tiles = seq_tiles_of(a, b);
    const int per_split = (tiles + a.num_splits - 1) / a.num_splits;
    sc.b0 = b;
    sc.off0 = pair * per_split;
    sc.count = max(0, min(per_split, tiles - sc.off0));
    sc.pos0 = 0;
    sc.total = 0;
    sc.per_seq = sc.split_tiles = sc.seq_tiles = 0;
    if (sc.count == 0) {
      // nothing to attend to: zeros (one split) or a split that carries no weight
      if (!qk_cta) {
        if (a.num_splits == 1) {
          for (int i = tid; i < heads_here * (kLatent / 2); i += kThreads) {
            const int h = i / (kLatent / 2), d = (i % (kLatent / 2)) * 2;
            *reinterpret_cast<uint32_t*>(a.o + b * a.o_stride_b + (head_base + h) * a.o_stride_h + d) = 0u;
          }
        } else if (tid < heads_here) {
          a.partial_lse[(static_cast<int64_t>(b) * a.num_splits + pair) * a.num_heads + head_base + tid] =
              -CUDART_INF_F;
        }
      }
      return;
    }
  }

  // ---------------- setup: barriers, TMEM, the pair ----------------
  if (tid == 0) {
#pragma unroll
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&ms.mb_stage_full[i], 1);
      mbar_init(&ms.mb_stage_free[i], qk_cta ? 1 : kConvWarps + 1);
      mbar_init(&ms.mb_sfa[i], 1);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      mbar_init(&ms.mb_kpe_full[i], 1);
      mbar_init(&ms.mb_kpe_free[i], 1);
      mbar_init(&ms.mb_s_full[i], 1);
      mbar_init(&ms.mb_s_free[i], kSoftmaxWarps);
      mbar_init(&ms.mb_p_free[i], 1);
      mbar_init(&ms.mb_info_full[i], 1);
      mbar_init(&ms.mb_o_ready[i], kEpiWarps);
      mbar_init(&ms.mb_tile_done[i], 1);
#pragma unroll
      for (int k = 0; k < 4; ++k) mbar_init(&ms.mb_p_full[i][k], 2);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      mbar_init(&ms.mb_sig[i], 1);
      mbar_init(&ms.mb_v_full[i], kConvWarps);
      mbar_init(&ms.mb_pv_done[i], 1);
    }
    mbar_init(&ms.mb_q_full, a.q_img ? 1 : kSoftmaxWarps);
    mbar_init(&ms.mb_q_free, 1);
    mbar_init(&ms.mb_stats_free, 1);
    mbar_init(&ms.mb_stats_full, 1);
    mbar_init(&ms.mb_drain, 1);
    ms.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kWarpMMA) tmem_alloc(&ms.tmem_base, kTmemCols);
  fence_before_sync();
  __syncthreads();
  cluster_sync();  // the peer's barriers exist before any remote arrive or store
  fence_after_sync();
  const uint32_t tmem = ms.tmem_base;

  if (warp == kWarpTMA) {
    if (lane == 0) producer(sm, ms, sc, a, maps, qk_cta);
  } else if (warp == kWarpMMA) {
    if (qk_cta) mma_qk(sm, ms, tmem, sc, lane, a);
    else mma_pv(sm, ms, tmem, sc, lane, a);
    __syncwarp();
    if (lane == 0) mma_commit(&ms.mb_drain);  // arrives once every MMA issued has completed
    __syncwarp();
  } else if (warp == kWarpKpe) {
    if (qk_cta && lane == 0) kpe_producer(sm, ms, sc, a, maps);
  } else if (warp == kWarpScale) {
    if (qk_cta) scale_warp_qk(sm, ms, sc, lane, a);
    else scale_warp_pv(sm, ms, sc, lane, a);
  } else if (qk_cta) {
    if (warp < kSoftmaxWarp0 + kSoftmaxWarps)
      softmax_qk(sm, ms, tmem, sc, head_base, heads_here, warp, lane, a.sm_scale * kLog2e, a);
  } else if (warp < kEpiWarp0 + kEpiWarps) {
    epilogue_pv(sm, ms, tmem, sc, head_base, heads_here, warp, lane, a);
  } else {
    converter(sm, ms, sc, warp, lane, a);
  }

  fence_before_sync();
  __syncthreads();  // every TMEM access of this CTA is done
  if (warp == kWarpMMA) {
    if (lane == 0 && !drain_wait(&ms.mb_drain, 0)) record_status(a, kStatusDrain);
    __syncwarp();
    fence_after_sync();
    tmem_dealloc(tmem, kTmemCols);
  }
  // neither CTA leaves while the other may still store into its shared
  // memory or arrive on its barriers
  cluster_sync();
}

// Q operand images of every (sequence, head block): one CTA of 1024 threads
// each, thread (h, bl) quantising the 32-element block bl of head h (and the
// 16-byte chunk bl < 8 of its q_pe).  It lets the decode kernel launched
// after it start at once; that kernel waits for this grid before reading
// the images.
__global__ void __launch_bounds__(1024) q_prep_fp4_kernel(const __grid_constant__ DecodeArgs a) {
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
  const int b = blockIdx.y, head_base = blockIdx.x * kNH;
  const int h = threadIdx.x >> 4, bl = threadIdx.x & 15;
  const bool live = h < a.num_heads - head_base;
  uint8_t* img = const_cast<uint8_t*>(a.q_img) + (static_cast<int64_t>(b) * gridDim.x + blockIdx.x) * kQImageBytes;
  const __nv_bfloat16* qrow = a.q + b * a.q_stride_b + (head_base + h) * a.q_stride_h;
  uint4 v[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) v[k] = ldg_stream_if(qrow + 32 * bl + 8 * k, live);
  const uint4 pe = ldg_stream_if(qrow + kLatent + 8 * (bl & 7), live && bl < 8);
  q_block(v, h, bl, img, img + kQTermBytes + kQPeBytes);
  if (bl < 8) *reinterpret_cast<uint4*>(img + kQTermBytes + (h >> 3) * 1024 + sw128_offset(h & 7, bl)) = pe;
}

}  // namespace

cudaError_t launch_q_prep_fp4(const DecodeArgs& a, cudaStream_t stream) {
  const dim3 grid((a.num_heads + kNH - 1) / kNH, a.batch);
  q_prep_fp4_kernel<<<grid, 1024, 0, stream>>>(a);
  return cudaGetLastError();
}

// One cluster of two CTAs per pair: grid.x = 2 x pairs (balanced) or 2 x
// splits (split mode).  After the Q prep kernel, the decode is its
// programmatic dependent (everything before the Q images, the first cache
// loads included, overlaps it).
cudaError_t launch_decode_fp4(const DecodeArgs& a, const CacheMaps& maps, cudaStream_t stream) {
  cudaError_t e = cudaFuncSetAttribute(mla_decode_fp4_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
  if (e != cudaSuccess) return e;
  const int head_blocks = (a.num_heads + kNH - 1) / kNH;
  const dim3 grid = a.balanced ? dim3(2 * a.num_splits, 1, head_blocks) : dim3(2 * a.num_splits, a.batch, head_blocks);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = a.q_img ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, mla_decode_fp4_kernel, a, maps);
}

}  // namespace kimi
