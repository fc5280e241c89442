// MXFP4 KV-append (quantise + paged cache write) and the plain row quantiser.
//
// One thread quantises one 32-element group (64 bytes of bf16 in, 16 bytes of
// nibbles + 1 scale byte out): 16 threads cover a 512-dim latent row, so a
// 256-thread block writes 16 tokens.  Loads and stores are 16-byte vectors;
// the whole kernel is a single HBM pass (1024 B read + 400 B written per
// token), bound by HBM bandwidth.
#include <cuda_runtime.h>

#include "kernels.cuh"
#include "mxfp4.cuh"

namespace kimi {

namespace {

__device__ __forceinline__ void load_group32(const __nv_bfloat16* src, float (&x)[32]) {
  const uint4* p = reinterpret_cast<const uint4*>(src);
#pragma unroll
  for (int v = 0; v < 4; ++v) {
    uint4 w = __ldg(p + v);
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      x[v * 8 + 2 * j] = __uint_as_float(ws[j] << 16);
      x[v * 8 + 2 * j + 1] = __uint_as_float(ws[j] & 0xFFFF0000u);
    }
  }
}

template <bool LEGACY>
__global__ void __launch_bounds__(256) kv_append_kernel(KvAppendArgs a) {
  const int tok = blockIdx.x * 16 + (threadIdx.x >> 4);
  const int grp = threadIdx.x & 15;
  if (tok >= a.num_tokens) return;
  const int64_t slot = a.slot_mapping[tok];
  if (slot < 0 || slot >= a.num_pages * kPageSize) return;

  const __nv_bfloat16* src = a.kv_c + tok * a.kv_c_stride + grp * 32;
  float x[32];
  load_group32(src, x);
  uint32_t packed[4];
  uint8_t sb;
  quantize_group32<LEGACY>(x, packed, sb);

  uint8_t* row = a.kv_buffer + slot * kTokenBytes;
  *reinterpret_cast<uint4*>(row + grp * 16) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
  a.kv_scales[slot * kScaleBytes + grp] = sb;
  if (grp < 8) {  // 64 bf16 of RoPE = 8 x 16 bytes, copied verbatim
    const uint4* pe = reinterpret_cast<const uint4*>(a.k_pe + tok * a.k_pe_stride);
    *reinterpret_cast<uint4*>(row + kNibbleBytes + grp * 16) = __ldg(pe + grp);
  }
}

template <bool LEGACY>
__global__ void __launch_bounds__(256) quantize_rows_kernel(QuantizeArgs a) {
  const int64_t gid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t groups_per_row = a.cols / 32;
  if (gid >= a.rows * groups_per_row) return;
  const int64_t r = gid / groups_per_row;
  const int64_t g = gid % groups_per_row;
  float x[32];
  load_group32(a.x + r * a.x_stride + g * 32, x);
  uint32_t packed[4];
  uint8_t sb;
  quantize_group32<LEGACY>(x, packed, sb);
  *reinterpret_cast<uint4*>(a.nibbles + r * (a.cols / 2) + g * 16) =
      make_uint4(packed[0], packed[1], packed[2], packed[3]);
  a.scales[r * groups_per_row + g] = sb;
}

}  // namespace

cudaError_t launch_kv_append(const KvAppendArgs& a, cudaStream_t stream) {
  if (a.num_tokens == 0) return cudaSuccess;
  const dim3 grid((a.num_tokens + 15) / 16);
  if (a.legacy_rule)
    kv_append_kernel<true><<<grid, 256, 0, stream>>>(a);
  else
    kv_append_kernel<false><<<grid, 256, 0, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_quantize_rows(const QuantizeArgs& a, cudaStream_t stream) {
  const int64_t total = a.rows * (a.cols / 32);
  if (total == 0) return cudaSuccess;
  const dim3 grid(static_cast<unsigned>((total + 255) / 256));
  if (a.legacy_rule)
    quantize_rows_kernel<true><<<grid, 256, 0, stream>>>(a);
  else
    quantize_rows_kernel<false><<<grid, 256, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace kimi
