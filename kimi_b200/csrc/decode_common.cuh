// Device helpers shared by the tensor-core decode kernels: named barriers,
// guarded loads, the e2m1 -> e5m2 byte-permute conversion, the e4m3 hi/lo
// split of P, and the tile schedule (split mode and the balanced schedule)
// with the cursors every warp role walks.
#pragma once

#include <cstdint>

#include <cuda_runtime.h>

#include "kernels.cuh"
#include "sm100.cuh"

namespace kimi {
namespace dec {

using namespace sm100;

__device__ __forceinline__ void named_bar(int id, int count) {
  asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(count) : "memory");
}

// End of setup, reached by every role from its own code path.
// Barrier over `count` threads that also ORs a predicate across them.
__device__ __forceinline__ bool bar_or(int id, int count, bool pred) {
  uint32_t out;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}\n"
      : "=r"(out)
      : "r"(pred ? 1u : 0u), "r"(id), "r"(count)
      : "memory");
  return out != 0;
}

__device__ __forceinline__ void mbar_arrive(uint64_t* mbar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_addr(mbar)) : "memory");
}

// Guarded loads: the predicate sits on the load itself and the destination
// keeps its preset value when it is false.  (A load followed by a select on
// the guard would make the select, and so the thread, wait for the data.)
__device__ __forceinline__ uint4 ldg_stream_if(const void* p, bool pred) {
  uint4 v = make_uint4(0u, 0u, 0u, 0u);
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.u32 p, %5, 0;\n\t"
      "@p ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n\t}\n"
      : "+r"(v.x), "+r"(v.y), "+r"(v.z), "+r"(v.w)
      : "l"(p), "r"(pred ? 1u : 0u));
  return v;
}

__device__ __forceinline__ uint32_t ldg_u8_if(const uint8_t* p, bool pred) {
  uint32_t v = 0u;
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.u32 p, %2, 0;\n\t"
      "@p ld.global.nc.u8 %0, [%1];\n\t}\n"
      : "+r"(v)
      : "l"(p), "r"(pred ? 1u : 0u));
  return v;
}

__device__ __forceinline__ int ldg_s32_or(const int32_t* p, bool pred, int fallback) {
  int v = fallback;
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.u32 p, %2, 0;\n\t"
      "@p ld.global.nc.s32 %0, [%1];\n\t}\n"
      : "+r"(v)
      : "l"(p), "r"(pred ? 1u : 0u));
  return v;
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}

// e2m1 -> e5m2 without conversion instructions.  For an e2m1 magnitude code
// c = (e << 1) | m (c >= 2 normal: 2^(e-1) (1 + m/2); c = 1: 0.5), the e5m2
// byte of value * 2^k is (0x38 + 4k) + 2c for c >= 2, 0x38 + 4k for c = 1 and
// 0 for c = 0.  A group of 32 elements shares k, so the eight magnitude bytes
// form a two-register PRMT table built once per group; the e2m1 sign (bit 3)
// becomes the e5m2 sign (bit 7).  Exact for k in [-13, 13]; below -14 the
// group is flushed to zero (it is then below 2^-14 of the reference).
__device__ __forceinline__ void e5m2_tables(int k, uint32_t& lut_lo, uint32_t& lut_hi) {
  if (k < -14) {
    lut_lo = lut_hi = 0u;
    return;
  }
  lut_lo = 0x3E3C3800u + 0x04040400u * static_cast<uint32_t>(k);
  lut_hi = 0x46444240u + 0x04040404u * static_cast<uint32_t>(k);
}

// prmt.b32 (default mode): byte n of the result is byte (sel_n & 7) of {a, b};
// when sel_n & 8 it is that byte's sign bit replicated over all eight bits.
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;\n" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// Eight e2m1 values (one u32 of packed nibbles, element 2j in the low nibble
// of byte j) -> eight e5m2 bytes in element order: nine instructions.
__device__ __forceinline__ void e2m1x8_to_e5m2(uint32_t w, uint32_t lut_lo, uint32_t lut_hi, uint32_t& o0,
                                               uint32_t& o1) {
  const uint32_t wm = w & 0x77777777u;                 // magnitude codes (selector bit 3 clear)
  const uint32_t m0 = prmt(lut_lo, lut_hi, wm);        // elements 0..3 (low four selector nibbles)
  const uint32_t m1 = prmt(lut_lo, lut_hi, wm >> 16);  // elements 4..7
  // sign of element 2j is bit 3 of byte j (bit 7 of byte j of w << 4), of
  // element 2j + 1 bit 7 of byte j: replicate them into sign masks
  const uint32_t w4 = w << 4;
  const uint32_t s0 = prmt(w4, w, 0xD9C8u);
  const uint32_t s1 = prmt(w4, w, 0xFBEAu);
  o0 = m0 | (s0 & 0x80808080u);
  o1 = m1 | (s1 & 0x80808080u);
}

// Eight nibble bytes (16 elements) with shift k -> 16 e5m2 bytes.
__device__ __forceinline__ uint4 half_group_to_e5m2(uint32_t w0, uint32_t w1, uint32_t lut_lo, uint32_t lut_hi) {
  uint4 o;
  e2m1x8_to_e5m2(w0, lut_lo, lut_hi, o.x, o.y);
  e2m1x8_to_e5m2(w1, lut_lo, lut_hi, o.z, o.w);
  return o;
}

// (a0, a1) += (b0, b1) as one packed instruction: two round-to-nearest fp32
// adds, the same results as two scalar adds.
__device__ __forceinline__ void add_f32x2(float& a0, float& a1, float b0, float b1) {
  uint64_t a = (static_cast<uint64_t>(__float_as_uint(a1)) << 32) | __float_as_uint(a0);
  const uint64_t b = (static_cast<uint64_t>(__float_as_uint(b1)) << 32) | __float_as_uint(b0);
  asm("add.rn.f32x2 %0, %0, %1;\n" : "+l"(a) : "l"(b));
  a0 = __uint_as_float(static_cast<uint32_t>(a));
  a1 = __uint_as_float(static_cast<uint32_t>(a >> 32));
}

// (a0, a1) = (a0, a1) * c + (d0, d1) as one packed instruction: two fused
// round-to-nearest multiply-adds, the same results as two fmaf calls.
__device__ __forceinline__ void fma_f32x2(float& a0, float& a1, float c, float d0, float d1) {
  uint64_t a = (static_cast<uint64_t>(__float_as_uint(a1)) << 32) | __float_as_uint(a0);
  const uint64_t cc = (static_cast<uint64_t>(__float_as_uint(c)) << 32) | __float_as_uint(c);
  const uint64_t d = (static_cast<uint64_t>(__float_as_uint(d1)) << 32) | __float_as_uint(d0);
  asm("fma.rn.f32x2 %0, %0, %1, %2;\n" : "+l"(a) : "l"(cc), "l"(d));
  a0 = __uint_as_float(static_cast<uint32_t>(a));
  a1 = __uint_as_float(static_cast<uint32_t>(a >> 32));
}

// p (two floats) -> e4m3 hi and e4m3 residual, through f16 (exact residual).
__device__ __forceinline__ void split_e4m3x2(float p0, float p1, uint16_t& hi, uint16_t& lo) {
  uint32_t h;
  asm("cvt.rn.f16x2.f32 %0, %2, %1;\n" : "=r"(h) : "f"(p0), "f"(p1));
  uint16_t h8;
  asm("cvt.rn.satfinite.e4m3x2.f16x2 %0, %1;\n" : "=h"(h8) : "r"(h));
  uint32_t back;
  asm("{\n\t.reg .b16 t;\n\tmov.b16 t, %1;\n\tcvt.rn.f16x2.e4m3x2 %0, t;\n\t}\n" : "=r"(back) : "h"(h8));
  uint32_t res;
  asm("sub.rn.f16x2 %0, %1, %2;\n" : "=r"(res) : "r"(h), "r"(back));
  uint16_t l8;
  asm("cvt.rn.satfinite.e4m3x2.f16x2 %0, %1;\n" : "=h"(l8) : "r"(res));
  hi = h8;
  lo = l8;
}

// ---------------------------------------------------------------------------
// Tile schedule and cursors
// ---------------------------------------------------------------------------
// A CTA's run of tiles: `count` tiles starting at tile off0 of sequence b0
// (global position pos0 of the batch's tile list in balanced mode).
struct Sched {
  int b0, off0, count;
  long long pos0, total;
};

// Position in the run.  A piece is the part of one sequence inside the run:
// tiles [piece_begin, piece_end) of sequence b; `left` tiles of the run follow it.
struct Cursor {
  int b, tile, piece_begin, piece_end, left;
  int page_lo, n_pages, n_tok;
  long long seq_pos;  // global position of tile 0 of sequence b (balanced mode)
};

__device__ __forceinline__ int seq_tiles_of(const DecodeArgs& a, int b) {
  const int n = a.kv_indptr[b + 1] - a.kv_indptr[b];
  return n > 0 ? (n + 1) >> 1 : 0;
}

__device__ __forceinline__ int cursor_tiles(const Cursor& c) { return (c.n_pages + 1) >> 1; }

__device__ __forceinline__ void cursor_load_seq(const DecodeArgs& a, Cursor& c) {
  c.page_lo = a.kv_indptr[c.b];
  c.n_pages = max(a.kv_indptr[c.b + 1] - c.page_lo, 0);
  const int last =
      c.n_pages == 0 ? 0 : min(max(a.kv_last_page_len ? a.kv_last_page_len[c.b] : kPageSize, 1), kPageSize);
  c.n_tok = c.n_pages == 0 ? 0 : (c.n_pages - 1) * kPageSize + last;
}

__device__ __forceinline__ void cursor_start(const DecodeArgs& a, const Sched& s, Cursor& c) {
  c.b = s.b0;
  cursor_load_seq(a, c);
  c.tile = c.piece_begin = s.off0;
  c.piece_end = min(cursor_tiles(c), s.off0 + s.count);
  c.left = s.count - (c.piece_end - s.off0);
  c.seq_pos = s.pos0 - s.off0;
}

// Step to the next tile of the run (past its end the cursor stays in the last piece).
__device__ __forceinline__ void cursor_next(const DecodeArgs& a, Cursor& c) {
  if (++c.tile < c.piece_end || c.left <= 0) return;
  c.seq_pos += cursor_tiles(c);
  do {
    ++c.b;
    cursor_load_seq(a, c);
  } while (cursor_tiles(c) == 0 && c.b + 1 < a.batch);
  c.tile = c.piece_begin = 0;
  c.piece_end = min(cursor_tiles(c), c.left);
  c.left -= c.piece_end;
}

__device__ __forceinline__ bool cursor_first(const Cursor& c) { return c.tile == c.piece_begin; }
__device__ __forceinline__ bool cursor_last(const Cursor& c) { return c.tile + 1 == c.piece_end; }
__device__ __forceinline__ int cursor_valid(const Cursor& c) {
  return max(0, min(kPageSize * 2, c.n_tok - c.tile * kPageSize * 2));
}

// CTA of a global tile position in balanced mode: the largest c with
// c T / G <= x.
__device__ __forceinline__ int cta_of_tile(long long x, const Sched& s, int ctas) {
  return static_cast<int>(((x + 1) * ctas - 1) / s.total);
}

// Block-scan scratch of balanced_schedule (in the kernel's shared memory).
struct SchedScratch {
  long long pos0;   // global position of the CTA's first tile
  long long total;  // tiles of the whole batch
  int b0, off0, count;
  int scan_warp[32];
};

// Balanced mode: locate run `c` of `ctas` runs with a block-wide scan of the
// tiles per sequence (all threads of the CTA call this).  Uniform batches
// take the same schedule: measured at 64 x 8192 tokens (64 heads) and at
// 128 x 4096 (8 heads), runs over all SMs were faster than whole-sequence
// splits over batch x floor(SMs / batch) CTAs, by 0.7% and 8.5%.
template <int kThreads>
__device__ void balanced_schedule(const DecodeArgs& a, SchedScratch& ms, Sched& s, int ctas, int c) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per = (a.batch + kThreads - 1) / kThreads;
  const int lo = min(a.batch, tid * per), hi = min(a.batch, lo + per);
  int mine = 0;
  for (int b = lo; b < hi; ++b) mine += seq_tiles_of(a, b);
  int incl = mine;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, d);
    if (lane >= d) incl += v;
  }
  if (lane == 31) ms.scan_warp[warp] = incl;
  __syncthreads();
  int before = 0, total = 0;
  for (int w2 = 0; w2 < kThreads / 32; ++w2) {
    const int v = ms.scan_warp[w2];
    if (w2 < warp) before += v;
    total += v;
  }
  const int excl = before + incl - mine;
  const long long start = static_cast<long long>(c) * total / ctas;
  const long long end = static_cast<long long>(c + 1) * total / ctas;
  // (also for an empty run: the sequence at its position names its merge slot)
  if (start < total && excl <= start && start < excl + mine) {
    long long acc = excl;
    for (int b = lo; b < hi; ++b) {
      const int t = seq_tiles_of(a, b);
      if (start < acc + t) {
        ms.b0 = b;
        ms.off0 = static_cast<int>(start - acc);
        break;
      }
      acc += t;
    }
  }
  if (tid == 0) {
    ms.count = static_cast<int>(end - start);
    ms.pos0 = start;
    ms.total = total;
  }
  __syncthreads();
  s.count = ms.count;
  s.b0 = ms.pos0 < total ? ms.b0 : 0;
  s.off0 = ms.pos0 < total ? ms.off0 : 0;
  s.pos0 = ms.pos0;
  s.total = ms.total;
  __syncthreads();  // the scan scratch is reused
}

// Transpose-reduce (max or sum) of N per-lane values over the warp (N a
// power of two, at most 32): lane l ends with the reduction of element l % N
// across all 32 lanes.  The exchange steps halve the values held per lane
// (each keeps one half and combines it with the partner's same half); with
// N < 32 a butterfly over the remaining lane bits finishes the reduction.
template <bool kMax, int N = 32>
__device__ __forceinline__ float warp_transpose_reduce(float (&v)[N], int lane) {
  static_assert(N >= 1 && N <= 32 && (N & (N - 1)) == 0, "N is a power of two up to 32");
#pragma unroll
  for (int width = N / 2; width >= 1; width >>= 1) {
    const bool upper = (lane & width) != 0;
#pragma unroll
    for (int j = 0; j < width; ++j) {
      const float send = upper ? v[j] : v[j + width];
      const float keep = upper ? v[j + width] : v[j];
      const float got = __shfl_xor_sync(0xffffffffu, send, width);
      v[j] = kMax ? fmaxf(keep, got) : keep + got;
    }
  }
  float r = v[0];
#pragma unroll
  for (int width = N; width < 32; width <<= 1) {
    const float got = __shfl_xor_sync(0xffffffffu, r, width);
    r = kMax ? fmaxf(r, got) : r + got;
  }
  return r;
}

}  // namespace dec
}  // namespace kimi
