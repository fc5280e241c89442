// The layer-input step after the tensor-parallel all-reduce, in one kernel:
// the ranks' partial hidden states summed (read straight from each rank's
// buffer: peer pointers over NVLink, or local buffers), the residual added and
// written back, RMSNorm with its weight, MXFP4 quantisation.
//
// Reference (paths inside ianye23301/kimi): the one-shot fused all-reduce +
// residual + RMSNorm `allreduce_fusion_kernel_1stage_nloop`
// (patches/aiter-1stage-nloop-ar-rmsnorm.patch:12-253) and the MXFP4
// quant-only step after it (patches/aiter-mxfp4-quant-only.patch:29-125;
// checked against the fused norm+quant in tests/test_ar_fusion_correctness.py:15-151):
//   combined = bf16(sum_r x_r + residual)            -> residual_out
//   normed   = bf16(combined * rsqrt(mean(combined^2) + eps))
//   out      = bf16(normed * weight)                 -> MXFP4 (unshuffled scales)
//
// One CTA per row; thread g owns elements 32 g .. 32 g + 31 -- exactly one
// MXFP4 group -- so the only cross-thread step is the sum of squares: the
// thread's 32 squares in order, a warp butterfly (lane 0's value kept), the
// warps in order.  Every float32 step is the oracle's, so the results are
// bit-exact.  The kernel is one pass over the inputs (bound by HBM or, for
// peer inputs, by NVLink).  A warp reads its 32 groups (2 KB of each input) as
// four fully coalesced 16-byte loads per lane, so every 32-byte sector is
// requested once (which matters for peer reads, where nothing merges partial
// requests), then hands each lane its own group's 64 bytes through a swizzled
// 2 KB shared-memory stage.
//
// The caller orders the kernel after every rank's partial is complete and
// keeps each partial unchanged until every rank's kernel has read it (for
// example with a stream-ordered barrier on both sides); the kernel itself
// waits for nothing.
#include <cuda_runtime.h>

#include "kernels.cuh"
#include "mxfp4.cuh"

namespace kimi {
namespace {

__device__ __forceinline__ void bf16x8_to_f32(const uint4 v, float* x) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    x[2 * j] = __uint_as_float(w[j] << 16);
    x[2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
  }
}

__device__ __forceinline__ float round_bf16(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// The warp's 128 uint4 of one input, loaded coalesced (lane l holds slots
// 32 p + l), are handed back as lane l's own group (slots 4 l .. 4 l + 3).
// Slot s lives at s ^ ((s >> 3) & 3): both the stores (8 consecutive slots per
// quarter warp) and the loads (stride 4 slots) then hit 8 distinct 16-byte
// bank groups per quarter warp.
__device__ __forceinline__ void warp_regroup(uint4 (&v)[4], uint4* stage, int lane) {
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const int s = 32 * p + lane;
    stage[s ^ ((s >> 3) & 3)] = v[p];
  }
  __syncwarp();
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const int s = 4 * lane + p;
    v[p] = stage[s ^ ((s >> 3) & 3)];
  }
  __syncwarp();
}

// Where one row's results go: `n` copies of residual_out / nibbles / scales
// (the local buffers, or every rank's for the two-shot form), all written
// with the same values.
struct RowDest {
  __nv_bfloat16* residual_out[kArMaxInputs];
  uint8_t* nibbles[kArMaxInputs];
  uint8_t* scales[kArMaxInputs];
  int n;
};

// Row `row` of a: the inputs summed in rank order, the residual added, the
// new residual, RMSNorm and MXFP4 of the row stored to every destination of
// `d`.  One CTA of ((hidden / 32 + 31) / 32) * 32 threads.
template <bool LEGACY>
__device__ __forceinline__ void norm_quant_row(const ArNormArgs& a, int row, const RowDest& d) {
  __shared__ float warp_sum[32];
  __shared__ float rstd;
  __shared__ uint4 stage[8][128];  // one 2 KB regroup stage per warp (at most 256 threads)
  const int g = threadIdx.x, lane = g & 31, warp = g >> 5;
  const int groups = a.hidden / 32;
  const bool live = g < groups;
  const int64_t off = static_cast<int64_t>(row) * a.hidden + 32 * g;
  // the warp's span: groups 32 warp .. 32 warp + warp_groups - 1 (every warp
  // has at least one, the launch rounds the groups up to whole warps)
  const int warp_groups = min(32, groups - 32 * warp);
  const int64_t span = (static_cast<int64_t>(row) * a.hidden + 1024 * warp) / 8;  // in uint4

  // every rank's slots and the residual's are loaded first (all in flight
  // together), then regrouped, summed in rank order, the residual added
  uint4 raw[kArMaxInputs][4], rres[4], wraw[4];
#pragma unroll
  for (int r = 0; r < kArMaxInputs; ++r)
#pragma unroll
    for (int p = 0; p < 4; ++p)
      raw[r][p] = r < a.num_inputs && 32 * p + lane < 4 * warp_groups
                      ? reinterpret_cast<const uint4*>(a.inputs[r])[span + 32 * p + lane]
                      : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
  for (int p = 0; p < 4; ++p)
    rres[p] = 32 * p + lane < 4 * warp_groups ? reinterpret_cast<const uint4*>(a.residual)[span + 32 * p + lane]
                                              : make_uint4(0u, 0u, 0u, 0u);
  if (live) {  // the weight is read by every row: left to the caches, 64 bytes per lane
#pragma unroll
    for (int p = 0; p < 4; ++p) wraw[p] = reinterpret_cast<const uint4*>(a.weight + 32 * g)[p];
  }
  uint4* st = stage[warp];
#pragma unroll
  for (int r = 0; r < kArMaxInputs; ++r)
    if (r < a.num_inputs) warp_regroup(raw[r], st, lane);  // uniform over the block
  warp_regroup(rres, st, lane);

  float c[32];
  float sq = 0.f;
  if (live) {
    float acc[32], t[8];
#pragma unroll
    for (int p = 0; p < 4; ++p) bf16x8_to_f32(raw[0][p], acc + 8 * p);
#pragma unroll
    for (int r = 1; r < kArMaxInputs; ++r) {
      if (r < a.num_inputs) {
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          bf16x8_to_f32(raw[r][p], t);
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[8 * p + j] = __fadd_rn(acc[8 * p + j], t[j]);
        }
      }
    }
    uint32_t packed[16];
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      bf16x8_to_f32(rres[p], t);
#pragma unroll
      for (int j = 0; j < 8; ++j) c[8 * p + j] = round_bf16(__fadd_rn(acc[8 * p + j], t[j]));
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const __nv_bfloat162 pr = __floats2bfloat162_rn(c[2 * j], c[2 * j + 1]);
      packed[j] = *reinterpret_cast<const uint32_t*>(&pr);
    }
#pragma unroll 1
    for (int k = 0; k < d.n; ++k) {
      uint4* ro = reinterpret_cast<uint4*>(d.residual_out[k] + off);
#pragma unroll
      for (int p = 0; p < 4; ++p)
        ro[p] = make_uint4(packed[4 * p], packed[4 * p + 1], packed[4 * p + 2], packed[4 * p + 3]);
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) sq = __fadd_rn(sq, __fmul_rn(c[i], c[i]));
  }
  // warp butterfly (lane 0's value), then the warps in order
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) sq = __fadd_rn(sq, __shfl_xor_sync(0xffffffffu, sq, o));
  if (lane == 0) warp_sum[warp] = sq;
  __syncthreads();
  if (g == 0) {
    float total = 0.f;
    for (int w = 0; w < (blockDim.x >> 5); ++w) total = __fadd_rn(total, warp_sum[w]);
    const float var = __fdiv_rn(total, static_cast<float>(a.hidden));
    rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, a.eps)));
  }
  __syncthreads();
  if (!live) return;
  const float r = rstd;
  float out[32];
  float wt[8];
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    bf16x8_to_f32(wraw[p], wt);
#pragma unroll
    for (int j = 0; j < 8; ++j) out[8 * p + j] = round_bf16(__fmul_rn(round_bf16(__fmul_rn(c[8 * p + j], r)), wt[j]));
  }
  uint32_t nib[4];
  uint8_t sb;
  quantize_group32<LEGACY>(out, nib, sb);
#pragma unroll 1
  for (int k = 0; k < d.n; ++k) {
    *reinterpret_cast<uint4*>(d.nibbles[k] + static_cast<int64_t>(row) * (a.hidden / 2) + 16 * g) =
        make_uint4(nib[0], nib[1], nib[2], nib[3]);
    d.scales[k][static_cast<int64_t>(row) * groups + g] = sb;
  }
}

template <bool LEGACY>
__global__ void __launch_bounds__(256) ar_norm_quant_kernel(const __grid_constant__ ArNormArgs a) {
  RowDest d;
  d.residual_out[0] = a.residual_out;
  d.nibbles[0] = a.nibbles;
  d.scales[0] = a.scales;
  d.n = 1;
  norm_quant_row<LEGACY>(a, blockIdx.x, d);
}

// ---------------------------------------------------------------------------
// Two-shot form over peer memory
// ---------------------------------------------------------------------------
// Rank r computes rows [r R / N, (r + 1) R / N) of the R rows -- each row
// reading all N ranks' partials, as above -- and stores each row's results
// into every rank's output buffers (plain peer stores).  Per call each rank
// reads 1 / N of every partial and writes its rows N times, instead of every
// rank reading all N partials whole.
//
// Two flag barriers over the ranks' flag words (int32 [2][N] per rank, slot
// [phase][source rank]; a rank writes the call's epoch -- its own call
// counter (counter[1]) plus one, the same on every rank since all make the
// same calls -- into every rank's slot, and waits until its own N slots of
// the phase hold it; the counter lives on the device, so a captured call
// replays correctly):
//   * entry: a rank's partial is complete when its call starts (stream
//     order); nobody reads a partial before all N ranks have entered;
//   * exit: the last CTA of a rank to finish its rows (a counter in the
//     rank's memory) announces that the rank's stores are out and its reads
//     done, then waits for all ranks: when the call completes, every rank's
//     rows have landed here and no rank still reads this rank's partial.
// Epochs only grow, so the flags are never reset.  Every wait is bounded in
// time; a wait that runs out sets kStatusPeerWait in the status word (after
// an entry give-up the CTA neither reads nor stores a row).  The ranks' flags
// may then be out of step: the exchange is to be set up anew.
// One system-scope fence per signal and per wait, made by one thread: a
// fence.sc.sys costs microseconds here, so the CTA's stores are first
// ordered before thread 0 by the CTA barrier (a release is cumulative over
// what precedes it in causality order), thread 0 fences once and writes the
// flags with relaxed stores; a waiting thread polls with relaxed loads and
// fences once it has seen the value (the acquire pattern).
__device__ __forceinline__ void st_relaxed_sys(int* p, int v) {
  asm volatile("st.relaxed.sys.global.b32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_relaxed_sys(const int* p) {
  int v;
  asm volatile("ld.relaxed.sys.global.b32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;\n" ::: "memory"); }
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
  return t;
}

// Thread 0 (after a CTA barrier): this rank's slot of `phase` in every rank's
// flag words := the epoch.
__device__ __forceinline__ void signal_all_ranks(const ArTwoShotArgs& t, int phase, int epoch) {
  fence_acq_rel_sys();
  for (int r = 0; r < t.world; ++r) st_relaxed_sys(t.flags[r] + phase * kArMaxInputs + t.rank, epoch);
}

// Threads 0 .. world - 1 each wait for one rank's slot of `phase` to reach
// the epoch (epochs are compared as the difference, so they may wrap); the
// CTA's verdict is the AND over them.
__device__ __forceinline__ bool wait_all_ranks(const ArTwoShotArgs& t, int phase, int epoch) {
  __shared__ int failed;
  if (threadIdx.x == 0) failed = 0;
  __syncthreads();
  if (static_cast<int>(threadIdx.x) < t.world) {
    const int* slot = t.flags[t.rank] + phase * kArMaxInputs + threadIdx.x;
    if (ld_relaxed_sys(slot) - epoch < 0) {
      const uint64_t t0 = global_ns();
      while (ld_relaxed_sys(slot) - epoch < 0) {
        if (global_ns() - t0 >= t.timeout_ns) {
          atomicExch(&failed, 1);
          break;
        }
        __nanosleep(32);
      }
    }
    fence_acq_rel_sys();
  }
  __syncthreads();
  const bool ok = failed == 0;
  if (!ok && threadIdx.x == 0 && t.status) atomicOr(t.status, kStatusPeerWait);
  return ok;
}

template <bool LEGACY>
__global__ void __launch_bounds__(256) ar_two_shot_kernel(const __grid_constant__ ArTwoShotArgs t) {
  const int begin = static_cast<int>(static_cast<int64_t>(t.base.rows) * t.rank / t.world);
  const int end = static_cast<int>(static_cast<int64_t>(t.base.rows) * (t.rank + 1) / t.world);
  // entry: CTA 0 announces this rank (its partial is complete: stream order),
  // every CTA waits for all ranks.  A CTA whose wait gave up skips its row but
  // still counts itself below, so the counter stays in step.
  // the call's number: one past the previous call's (the counter word is
  // advanced by this call's last CTA, after every CTA has read it here)
  const int epoch = *reinterpret_cast<volatile int*>(t.counter + 1) + 1;
  if (blockIdx.x == 0 && threadIdx.x == 0) signal_all_ranks(t, 0, epoch);
  const bool entered = wait_all_ranks(t, 0, epoch);
  const int row = begin + static_cast<int>(blockIdx.x);
  if (entered && row < end) {
    RowDest d;
#pragma unroll
    for (int k = 0; k < kArMaxInputs; ++k) {
      d.residual_out[k] = t.residual_out[k];
      d.nibbles[k] = t.nibbles[k];
      d.scales[k] = t.scales[k];
    }
    d.n = t.world;
    norm_quant_row<LEGACY>(t.base, row, d);
  }
  // exit: the CTA's stores are ordered before thread 0 by the barrier; the
  // rank's last CTA announces the rank (one system fence) and waits for all
  __syncthreads();
  __shared__ int last;
  if (threadIdx.x == 0) {
    int done;
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;\n" : "=r"(done) : "l"(t.counter) : "memory");
    last = done == static_cast<int>(gridDim.x) - 1;
    if (last) {
      t.counter[0] = 0;      // the next call is stream-ordered after this one
      t.counter[1] = epoch;  // every CTA of this call has read the previous number
      signal_all_ranks(t, 1, epoch);
    }
  }
  __syncthreads();
  if (last) wait_all_ranks(t, 1, epoch);
}

}  // namespace

cudaError_t launch_ar_two_shot(const ArTwoShotArgs& t, cudaStream_t stream) {
  const int threads = ((t.base.hidden / 32) + 31) / 32 * 32;
  const int mine = static_cast<int>(static_cast<int64_t>(t.base.rows) * (t.rank + 1) / t.world -
                                    static_cast<int64_t>(t.base.rows) * t.rank / t.world);
  const int grid = mine > 0 ? mine : 1;  // a rank without rows still takes part in both barriers
  if (t.base.legacy_rule)
    ar_two_shot_kernel<true><<<grid, threads, 0, stream>>>(t);
  else
    ar_two_shot_kernel<false><<<grid, threads, 0, stream>>>(t);
  return cudaGetLastError();
}

cudaError_t launch_ar_norm_quant(const ArNormArgs& a, cudaStream_t stream) {
  const int threads = ((a.hidden / 32) + 31) / 32 * 32;
  if (a.legacy_rule)
    ar_norm_quant_kernel<true><<<a.rows, threads, 0, stream>>>(a);
  else
    ar_norm_quant_kernel<false><<<a.rows, threads, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace kimi
