// Thin wrappers over the sm_100a PTX used by the tensor-core decode kernel:
// tcgen05 (TMEM allocation, MMA issue/commit, TMEM loads), mbarriers with
// bounded waits, proxy fences, and the UMMA shared-memory / instruction
// descriptors.
//
// Shared-memory operands use the SWIZZLE_NONE canonical layouts: an operand
// is a grid of "core matrices" of 8 rows x 16 bytes (128 contiguous bytes,
// rows 16 bytes apart).  For a K-major operand the rows are M (or N) and the
// 16 bytes run along K; for an MN-major operand the rows are K and the 16
// bytes run along M (or N).  The descriptor's two byte offsets give the
// distance between core matrices adjacent in the leading and in the strided
// direction:
//   K-major : LBO = next 16 bytes of K,          SBO = next 8 rows of M/N
//   MN-major: LBO = next 8 rows of K,            SBO = next 16 bytes of M/N
#pragma once

#include <cstdint>
#include <cuda_fp16.h>

namespace kimi {
namespace sm100 {

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// Descriptors
// ---------------------------------------------------------------------------

enum : uint32_t { kSwizzleNone = 0, kSwizzle128B = 2, kSwizzle64B = 4, kSwizzle32B = 6 };

// Shared-memory matrix descriptor (sm100 version bits, base offset 0).
// Swizzled operands must start their swizzle atoms on an atom-size boundary
// (1024 B for 128B swizzle, 512 B for 64B); a K-major start address may
// advance inside the atom's first row (K steps of 32 B).
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                              uint32_t layout = kSwizzleNone) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1u) << 46;  // descriptor version for tcgen05
  d |= static_cast<uint64_t>(layout & 7u) << 61;
  return d;
}

// Byte offset of 16-byte chunk `chunk` of row `row` inside a 128B-swizzled
// atom (8 rows x 128 B): chunk index XOR (row mod 8).
__host__ __device__ constexpr uint32_t sw128_offset(uint32_t row, uint32_t chunk) {
  return (row & 7u) * 128u + ((chunk ^ (row & 7u)) & 7u) * 16u;
}
// Same inside a 64B-swizzled atom (8 rows x 64 B): chunk index XOR ((row / 2) mod 4).
__host__ __device__ constexpr uint32_t sw64_offset(uint32_t row, uint32_t chunk) {
  return (row & 7u) * 64u + ((chunk ^ ((row >> 1) & 3u)) & 3u) * 16u;
}

enum : uint32_t {
  kFmtF16 = 0, kFmtBF16 = 1,          // kind::f16 operand formats
  kFmtE4M3 = 0, kFmtE5M2 = 1,         // kind::f8f6f4 operand formats
};

// Instruction descriptor (dense, fp32 accumulator).
__host__ __device__ constexpr uint32_t instr_desc(uint32_t a_fmt, uint32_t b_fmt, bool a_mn_major, bool b_mn_major,
                                                  uint32_t m, uint32_t n) {
  return (1u << 4)                        // D format: f32
         | (a_fmt << 7) | (b_fmt << 10)   // A / B formats
         | ((a_mn_major ? 1u : 0u) << 15) | ((b_mn_major ? 1u : 0u) << 16)
         | ((n >> 3) << 17) | ((m >> 4) << 24);
}

// ---------------------------------------------------------------------------
// TMEM
// ---------------------------------------------------------------------------

// Allocate `ncols` TMEM columns (power of two >= 32); the base address is
// written to shared memory at `dst`.  Executed by one full warp.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_addr(dst)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
}

// Generic-proxy shared-memory writes -> visible to the async proxy (tensor core).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp receives
// lane (32 * (warp % 4) + i), columns [col, col + 32).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }

// ---------------------------------------------------------------------------
// MMA issue (one thread) and completion tracking
// ---------------------------------------------------------------------------

__device__ __forceinline__ void mma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}

// A operand from TMEM (lane = row m, 32-bit column = two consecutive 16-bit K elements).
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void mma_f8f6f4_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}

// Block-scaled e2m1 x e2m1 MMA (kind::mxf4, one e8m0 scale per 32 K elements,
// K = 64 per instruction), both operands K-major packed nibbles in shared
// memory (element 2j in the low nibble of byte j, as in the MXFP4 cache).
// The scale factors sit in TMEM: for an operand row r (of A's M or B's N),
// scale block k4 (four consecutive 32-element groups, K = 128) occupies one
// 32-bit column per 32 rows, column c0 + r / 32 of lane r % 32 holding the
// four e8m0 bytes of groups 4 k4 .. 4 k4 + 3 of row r, copied identically
// into all four 32-lane quarters.  `sfa` / `sfb` are the TMEM addresses of
// that block's first column with the byte of the instruction's first group
// (0 or 2) in bits 30-31; the same byte index goes into the descriptor.
__device__ __forceinline__ void mma_mxf4_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t sfa, uint32_t sfb, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4.block_scale.block32 [%0], %1, %2, %3, [%5], [%6], p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa), "r"(sfb));
}

// Instruction descriptor of kind::mxf4 (e2m1 operands, e8m0 scales, M = 128,
// K = 64, fp32 accumulator): scale byte index of A in bits 29-30, of B in 4-5.
__host__ __device__ constexpr uint32_t instr_desc_mxf4(uint32_t n, uint32_t a_sf_byte, uint32_t b_sf_byte) {
  return (b_sf_byte << 4) | (1u << 7) | (1u << 10) | ((n >> 3) << 17) | (1u << 23) | ((128u >> 4) << 24) |
         (a_sf_byte << 29);
}

// Arrive (once) on an mbarrier when all previously issued tcgen05.mma of this
// thread have completed.
__device__ __forceinline__ void mma_commit(uint64_t* mbar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(
                   smem_addr(mbar))
               : "memory");
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint64_t* mbar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_addr(mbar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* mbar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_addr(mbar)), "r"(bytes)
               : "memory");
}

// ---------------------------------------------------------------------------
// TMA (tensor maps encoded on the host; no cluster multicast)
// ---------------------------------------------------------------------------

// 2-D tiled load of one box at element coordinates (x, y) into shared memory;
// the box's bytes count towards the mbarrier's transaction count.  Box
// elements outside the tensor are filled with zeros.
__device__ __forceinline__ void tma_load_2d(void* dst, const void* tensor_map, int x, int y, uint64_t* mbar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n" ::
          "r"(smem_addr(dst)),
      "l"(tensor_map), "r"(x), "r"(y), "r"(smem_addr(mbar))
      : "memory");
}

// 3-D tiled load of one box at element coordinates (x, y, z); otherwise as
// tma_load_2d.
__device__ __forceinline__ void tma_load_3d(void* dst, const void* tensor_map, int x, int y, int z, uint64_t* mbar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];\n" ::"r"(smem_addr(dst)),
      "l"(tensor_map), "r"(x), "r"(y), "r"(z), "r"(smem_addr(mbar))
      : "memory");
}

// Untiled bulk copy global -> shared of `bytes` (a multiple of 16; both
// addresses 16-byte aligned); the bytes count towards the mbarrier's
// transaction count.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* mbar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                   smem_addr(dst)),
               "l"(src), "r"(bytes), "r"(smem_addr(mbar))
               : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const void* tensor_map) {
  asm volatile("prefetch.tensormap [%0];\n" ::"l"(tensor_map) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* mbar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_addr(mbar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint: a thread whose phase is not complete
// sleeps (issuing nothing) until the phase completes or about `ns`
// nanoseconds pass, instead of spinning through quick polls.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* mbar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_addr(mbar)), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}

// Each unsuccessful poll of the bounded waits below sleeps up to this long.
constexpr uint32_t kWaitSleepNs = 20000;

// Wait for the phase with the given parity to complete, giving up after
// `max_polls` unsuccessful polls (each sleeping up to kWaitSleepNs).  Returns
// false on give-up.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* mbar, uint32_t parity, uint32_t max_polls) {
  for (uint32_t i = 0; i < max_polls; ++i)
    if (mbar_try_wait_sleep(mbar, parity, kWaitSleepNs)) return true;
  return false;
}

// As mbar_wait_bounded, but also gives up as soon as *abort (a shared-memory
// word another thread sets when one of its own waits gave up) is non-zero.
__device__ __forceinline__ bool mbar_wait_or_abort(uint64_t* mbar, uint32_t parity, uint32_t max_polls,
                                                   const volatile int* abort) {
  for (uint32_t i = 0; i < max_polls; ++i) {
    if (mbar_try_wait_sleep(mbar, parity, kWaitSleepNs)) return true;
    if (*abort) return false;
  }
  return false;
}

// Nanoseconds of the GPU's global timer.
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
  return t;
}

// Wait for the phase with the given parity to complete for at most about
// `timeout_ns` nanoseconds of global time (each poll sleeping up to
// min(kWaitSleepNs, timeout_ns); the clock is read from the second poll on,
// so a wait that the first poll ends costs no timer read), giving up early
// once *abort is non-zero.  Returns false on give-up.
__device__ __forceinline__ bool mbar_wait_timed(uint64_t* mbar, uint32_t parity, uint64_t timeout_ns,
                                                const volatile int* abort) {
  const uint32_t hint = timeout_ns < kWaitSleepNs ? static_cast<uint32_t>(timeout_ns) : kWaitSleepNs;
  if (mbar_try_wait_sleep(mbar, parity, hint)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    if (mbar_try_wait_sleep(mbar, parity, hint)) return true;
    if (abort && *abort) return false;
    if (globaltimer_ns() - t0 >= timeout_ns) return false;
  }
}

// ---------------------------------------------------------------------------
// Per-warpgroup register budgets (all four warps of a warpgroup execute these)
// ---------------------------------------------------------------------------
template <uint32_t kRegs>
__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;\n" ::"n"(kRegs));
}
template <uint32_t kRegs>
__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;\n" ::"n"(kRegs));
}

// ---------------------------------------------------------------------------
// Conversions
// ---------------------------------------------------------------------------

// Two e2m1 values (one byte: element 2j low nibble, 2j+1 high nibble) ->
// f16x2 (low half = low nibble), exact.
__device__ __forceinline__ uint32_t cvt_e2m1x2_f16x2(uint32_t byte) {
  uint32_t out;
  asm("{\n\t.reg .b8 b;\n\t"
      "cvt.u8.u32 b, %1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b;\n\t}\n"
      : "=r"(out)
      : "r"(byte));
  return out;
}

// Two floats -> two e2m1 codes in one byte (round to nearest even,
// saturating to +-6); `lo` lands in the low nibble.
__device__ __forceinline__ uint32_t cvt_f32x2_e2m1x2(float lo, float hi) {
  uint32_t out;
  asm("{\n\t.reg .b8 t;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 t, %2, %1;\n\t"
      "cvt.u32.u8 %0, t;\n\t}\n"
      : "=r"(out)
      : "f"(lo), "f"(hi));
  return out;
}

// Two floats -> e4m3x2 (round to nearest even, saturating to +-448); `lo`
// lands in the low byte.
__device__ __forceinline__ uint16_t cvt_f32x2_e4m3x2(float lo, float hi) {
  uint16_t out;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %2, %1;\n" : "=h"(out) : "f"(lo), "f"(hi));
  return out;
}

// e4m3x2 (low byte = first value) -> two floats, exact.
__device__ __forceinline__ float2 e4m3x2_to_float2(uint16_t v) {
  uint32_t h2;
  asm("{\n\t.reg .b16 t;\n\tmov.b16 t, %1;\n\tcvt.rn.f16x2.e4m3x2 %0, t;\n\t}\n" : "=r"(h2) : "h"(v));
  const float lo = __half2float(__ushort_as_half(static_cast<unsigned short>(h2 & 0xFFFFu)));
  const float hi = __half2float(__ushort_as_half(static_cast<unsigned short>(h2 >> 16)));
  return make_float2(lo, hi);
}

}  // namespace sm100
}  // namespace kimi
