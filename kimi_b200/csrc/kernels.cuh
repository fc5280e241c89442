// Internal (C++) launch interfaces shared by the kernels and the C ABI layer.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace kimi {

constexpr int kLatent = 512;      // kv_lora_rank
constexpr int kRope = 64;         // qk_rope_head_dim
constexpr int kQkDim = 576;
constexpr int kPageSize = 64;
constexpr int kNibbleBytes = 256;
constexpr int kRopeBytes = 128;
constexpr int kTokenBytes = 384;  // nibbles + RoPE per token in kv_buffer
constexpr int kScaleBytes = 16;
constexpr int kPageBytes = kPageSize * kTokenBytes;        // 24576
constexpr int kPageScaleBytes = kPageSize * kScaleBytes;   // 1024
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

struct KvAppendArgs {
  const __nv_bfloat16* kv_c;
  int64_t kv_c_stride;
  const __nv_bfloat16* k_pe;
  int64_t k_pe_stride;
  const int64_t* slot_mapping;
  uint8_t* kv_buffer;
  uint8_t* kv_scales;
  int64_t num_pages;
  int num_tokens;
  int legacy_rule;
};

struct QuantizeArgs {
  const __nv_bfloat16* x;
  int64_t rows;
  int64_t cols;
  int64_t x_stride;
  uint8_t* nibbles;
  uint8_t* scales;
  int legacy_rule;
};

// Split-K decode: stage 1 writes per-(sequence, split, head) partial outputs
// normalised by the split's own softmax sum plus the natural-log
// log-sum-exp; with one split it writes the final bf16 output directly.
struct DecodeArgs {
  const __nv_bfloat16* q;
  int64_t q_stride_b;
  int64_t q_stride_h;
  const uint8_t* kv_buffer;
  const uint8_t* kv_scales;
  int64_t num_pages;
  const int32_t* kv_indptr;
  const int32_t* kv_indices;
  const int32_t* kv_last_page_len;  // may be null (full pages)
  __nv_bfloat16* o;
  int64_t o_stride_b;
  int64_t o_stride_h;
  float* partial_o;    // [batch, splits, heads, 512]
  float* partial_lse;  // [batch, splits, heads]
  int* status;         // optional device word: bits set when a bounded wait gave up
  int batch;
  int num_heads;
  int num_splits;
  float sm_scale;
};

struct ReduceArgs {
  const float* partial_o;
  const float* partial_lse;
  __nv_bfloat16* o;
  int64_t o_stride_b;
  int64_t o_stride_h;
  int batch;
  int num_heads;
  int num_splits;
};

cudaError_t launch_kv_append(const KvAppendArgs& a, cudaStream_t stream);
cudaError_t launch_quantize_rows(const QuantizeArgs& a, cudaStream_t stream);
cudaError_t launch_decode_mma(const DecodeArgs& a, cudaStream_t stream);
cudaError_t launch_decode_tc(const DecodeArgs& a, cudaStream_t stream);
cudaError_t launch_reduce(const ReduceArgs& a, cudaStream_t stream);

}  // namespace kimi
