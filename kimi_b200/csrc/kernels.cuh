// Internal (C++) launch interfaces shared by the kernels and the C ABI layer.
#pragma once

#include <cstdint>
#include <cuda.h>
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
// Heads per CTA of the fp4 decode: 64, or 16 for a call with at most 16
// heads (a tensor-parallel shard: 8 heads of Kimi-K2 or 16 of DeepSeek-V3 at
// TP8), whose MMAs and softmax then work on 16 head columns instead of 64.
__host__ __device__ constexpr int decode_heads_per_cta(int num_heads) { return num_heads <= 16 ? 16 : 64; }

// Q operands of the fp4 kernel for one (sequence, head block of nh heads), as
// the shared-memory images its QK^T MMAs read: three block-scaled e2m1 terms
// (2 K blocks x 3 nh rows x 128 B, 128-byte swizzle), q_pe (nh rows x 128 B,
// same swizzle), then the terms' e8m0 scales as [3 nh rows][16 blocks].
__host__ __device__ constexpr int q_term_bytes(int nh) { return 2 * 3 * nh * 128; }
__host__ __device__ constexpr int q_pe_bytes(int nh) { return nh * 128; }
__host__ __device__ constexpr int q_scale_bytes(int nh) { return 3 * nh * 16; }
__host__ __device__ constexpr int q_image_bytes(int nh) { return q_term_bytes(nh) + q_pe_bytes(nh) + q_scale_bytes(nh); }
constexpr int kQImageBytes = q_image_bytes(64);       // 60416 (64-head blocks)
constexpr int kQImageBytesSmall = q_image_bytes(16);  // 15104 (16-head blocks)
static_assert(kQImageBytes == 60416 && kQImageBytesSmall == 15104, "Q image sizes");

// Bits of the decode's device status word (DecodeArgs::status): which wait
// gave up, or a page id outside the cache.
enum : int {
  kStatusSoftmaxWait = 1,
  kStatusSoftmaxPvWait = 2,
  kStatusEpilogueWait = 4,
  kStatusIssuerWait = 16,
  kStatusIssuerPvWait = 32,
  kStatusConverterWait = 64,
  kStatusDrain = 128,
  kStatusProducerWait = 256,
  kStatusBadPage = 512,
  kStatusPeerWait = 1024,
  kStatusQAbsorbWait = 2048,
  kStatusVupWait = 4096,
  kStatusScaleWait = 8,
};
// Default bound of a device wait when the caller passes 0 (2 s).
constexpr unsigned long long kDefaultTimeoutNs = 2000000000ull;
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

// The decode prologue: q absorption by W_UK, RoPE of q_pe / k_pe, KV append.
struct QAbsorbArgs {
  const __nv_bfloat16* q_nope;  // [T, H, 128]
  int64_t q_nope_stride_t, q_nope_stride_h;
  const __nv_bfloat16* q_pe;    // [T, H, 64]
  int64_t q_pe_stride_t, q_pe_stride_h;
  const __nv_bfloat16* w_uk;    // [H, 128, 512] contiguous
  const __nv_bfloat16* kv_c;    // [T, 512]
  int64_t kv_c_stride;
  const __nv_bfloat16* k_pe;    // [T, 64], before RoPE
  int64_t k_pe_stride;
  const int64_t* positions;     // [T]
  const float* cos;             // [max_position, 32]
  const float* sin;             // [max_position, 32]
  int64_t max_position;
  const int64_t* slot_mapping;  // [T]
  uint8_t* kv_buffer;
  uint8_t* kv_scales;
  int64_t num_pages;
  __nv_bfloat16* q_out;         // [T, H, 576]
  int64_t q_out_stride_t, q_out_stride_h;
  int num_tokens;
  int num_heads;
  int is_neox;
  int legacy_rule;
  int* status;  // optional device word (kStatusQAbsorbWait)
};

// Sum of the ranks' partial rows + residual, RMSNorm, MXFP4 (one CTA per row).
constexpr int kArMaxInputs = 8;
struct ArNormArgs {
  const __nv_bfloat16* inputs[kArMaxInputs];  // [rows, hidden] each, rank order
  int num_inputs;
  const __nv_bfloat16* residual;              // [rows, hidden]
  __nv_bfloat16* residual_out;                // [rows, hidden] (may alias residual)
  const __nv_bfloat16* weight;                // [hidden]
  float eps;
  uint8_t* nibbles;                           // [rows, hidden / 2]
  uint8_t* scales;                            // [rows, hidden / 32]
  int rows;
  int hidden;
  int legacy_rule;
};

// Two-shot all-reduce + RMSNorm + MXFP4 over peer memory (ar_norm_quant.cu):
// `base` holds every rank's partial in inputs[] (rank order), this rank's
// residual, the weight, eps, rows, hidden and the rounding rule; its
// residual_out / nibbles / scales are unused.
struct ArTwoShotArgs {
  ArNormArgs base;
  __nv_bfloat16* residual_out[kArMaxInputs];  // every rank's [rows, hidden]
  uint8_t* nibbles[kArMaxInputs];             // every rank's [rows, hidden / 2]
  uint8_t* scales[kArMaxInputs];              // every rank's [rows, hidden / 32]
  int* flags[kArMaxInputs];                   // every rank's flag words [2][kArMaxInputs]
  int* counter;                               // this rank's [CTA count (0 between calls), call number]
  int* status;                                // optional device word (kStatusPeerWait)
  unsigned long long timeout_ns;              // bound of each barrier wait
  int world;
  int rank;
};

struct VUpOProjArgs {
  const __nv_bfloat16* o;  // [num_heads, num_tokens, 512], element strides below
  int64_t o_stride_h;
  int64_t o_stride_t;
  const __nv_bfloat16* w_uv;  // [num_heads, 512, 128]
  const __nv_bfloat16* w_o;   // [hidden, num_heads * 128]
  __nv_bfloat16* x;           // [num_tokens, num_heads * 128] scratch
  __nv_bfloat16* out;         // [num_tokens, hidden], row stride out_stride
  int64_t out_stride;
  int num_tokens;
  int num_heads;
  int hidden;
  int* status;  // optional device word (kStatusVupWait)
};

// TMA maps of the V up-projection + o_proj operands, all bf16 with 128-byte
// swizzle: o as [H][T][512] (box 64 x 128 tokens x 1 head), W_UV as
// [H * 512][128] (box 64 x 64 rows), x as [T][H * 128] (box 64 x 128 tokens),
// W_o as [hidden][H * 128] (box 64 x 64 rows).
// Tokens per phase-1 CTA of the V up-projection (the o map's box height).
constexpr int kVUpRows = 64;

struct VUpOProjMaps {
  CUtensorMap o;
  CUtensorMap w_uv;
  CUtensorMap x;
  CUtensorMap w_o;
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

// Split-K decode.  Stage 1 covers each sequence's 128-token tiles with one or
// more pieces; a piece that holds a whole sequence writes the final bf16
// output, any other writes a partial output (normalised by its own softmax
// sum) and its natural-log log-sum-exp to a workspace slot.
// The grid's x index is (CTA or split) * head blocks + head block: the CTAs of
// one tile range for the different 64-head blocks are neighbours.
//   * split mode (balanced = 0): grid (num_splits x head blocks, batch); CTA
//     (s, b) takes the s-th of num_splits equal tile ranges of sequence b, slot
//     b * num_splits + s; with one split the CTA writes the output directly.
//   * balanced mode (balanced = 1): grid (ctas x head blocks, 1); CTA c takes
//     tiles [c T / ctas, (c + 1) T / ctas) of all T tiles of the batch laid end
//     to end, slot b + c for its piece of sequence b (unique: along the tile
//     list both b and c only grow), and the CTA holding a sequence's first tile
//     records (first CTA, last CTA) of that sequence in seq_meta for the merge.
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
  __nv_bfloat16* partial_o;  // [slots, heads, 512] bf16 (the merge restores fp32 sums)
  float* partial_lse;  // [batch, splits, heads]
  int* status;         // optional device word: kStatus* bits (a wait that gave up, a bad page id)
  int2* seq_meta;      // balanced mode: [batch] (first CTA, last CTA) of each sequence's tiles
  const uint8_t* q_img;  // fp4 kernel: [batch][head blocks] Q operand images (kQImageBytes each), or null
  int batch;
  int num_heads;
  int num_splits;      // split mode: splits per sequence; balanced mode: CTAs per head block
  int balanced;        // 1: balanced mode
  float sm_scale;
  unsigned long long timeout_ns;  // bound of each device wait (the drain's excepted)
};

// TMA maps of the cache for the fp4 tensor-core kernel: kv_buffer as a
// [num_pages * 64, 384] byte matrix (box 128 x 64 rows, 128-byte swizzle) and
// kv_scales as [num_pages * 64, 16] (box 16 x 64 rows).
struct CacheMaps {
  CUtensorMap kv;
  CUtensorMap sc;
};

struct ReduceArgs {
  const void* partial_o;      // [slots, heads, 512], bf16 (this library's decode) or fp32
  int partial_bf16;
  const float* partial_lse;
  __nv_bfloat16* o;
  int64_t o_stride_b;
  int64_t o_stride_h;
  int batch;
  int num_heads;
  int num_splits;             // split mode: slots b * num_splits + s; balanced mode: CTAs (spans lie in [0, num_splits))
  const int2* seq_meta;       // balanced mode (non-null): slots b + c, c in [meta.x, meta.y]
  const int32_t* kv_indptr;   // balanced mode: sequences without pages get zeros
  int programmatic;           // launched as a programmatic dependent of the decode kernel (waits for it)
};

cudaError_t launch_kv_append(const KvAppendArgs& a, cudaStream_t stream);
cudaError_t launch_q_absorb(const QAbsorbArgs& a, cudaStream_t stream);
cudaError_t launch_ar_norm_quant(const ArNormArgs& a, cudaStream_t stream);
cudaError_t launch_ar_two_shot(const ArTwoShotArgs& t, cudaStream_t stream);
cudaError_t launch_v_up_o_proj(const VUpOProjArgs& a, const VUpOProjMaps& maps, cudaStream_t stream);
cudaError_t launch_quantize_rows(const QuantizeArgs& a, cudaStream_t stream);
cudaError_t launch_decode_fp4(const DecodeArgs& a, const CacheMaps& maps, cudaStream_t stream);
// Writes a.q_img (one CTA per sequence and head block); the fp4 kernel launched after it reads the images.
cudaError_t launch_q_prep_fp4(const DecodeArgs& a, cudaStream_t stream);
cudaError_t launch_reduce(const ReduceArgs& a, cudaStream_t stream);

}  // namespace kimi
