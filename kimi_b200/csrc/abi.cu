// C ABI of the library (declared in include/kimi_mla.h): host-side argument
// checks, workspace layout, split-count choice, and kernel launches.  No
// allocation, no host synchronisation.
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>

#include <cuda.h>
#include <cuda_runtime.h>

#include "../../include/kimi_mla.h"
#include "kernels.cuh"

namespace {

using kimi::kLatent;

static_assert(kimi::kStatusSoftmaxWait == KIMI_DEVICE_SOFTMAX_WAIT && kimi::kStatusSoftmaxPvWait == KIMI_DEVICE_SOFTMAX_PV_WAIT &&
                  kimi::kStatusEpilogueWait == KIMI_DEVICE_EPILOGUE_WAIT && kimi::kStatusIssuerWait == KIMI_DEVICE_ISSUER_WAIT &&
                  kimi::kStatusIssuerPvWait == KIMI_DEVICE_ISSUER_PV_WAIT &&
                  kimi::kStatusConverterWait == KIMI_DEVICE_CONVERTER_WAIT && kimi::kStatusDrain == KIMI_DEVICE_DRAIN_WAIT &&
                  kimi::kStatusProducerWait == KIMI_DEVICE_PRODUCER_WAIT && kimi::kStatusBadPage == KIMI_DEVICE_BAD_PAGE &&
                  kimi::kStatusScaleWait == KIMI_DEVICE_SCALE_WAIT && kimi::kStatusPeerWait == KIMI_DEVICE_PEER_WAIT &&
                  kimi::kStatusQAbsorbWait == KIMI_DEVICE_QABSORB_WAIT && kimi::kStatusVupWait == KIMI_DEVICE_VUP_WAIT,
              "device status bits of the kernels and the header agree");

inline bool aligned(const void* p, uintptr_t n) { return (reinterpret_cast<uintptr_t>(p) % n) == 0; }

inline int cuda_status(cudaError_t e) {
  return e == cudaSuccess ? KIMI_OK : KIMI_ERR_CUDA_BASE + static_cast<int>(e);
}

int device_sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

// cuTensorMapEncodeTiled, from the driver through the runtime (no link
// against libcuda).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// TMA maps of the paged cache for the fp4 kernel: kv_buffer as a
// [num_pages * 64, 384] byte matrix read in boxes of 128 bytes x 64 rows
// (128-byte swizzle: the MMA operand layout), kv_scales as [num_pages * 64,
// 16] in boxes of 16 x 64.  Reads past either end yield zeros.  The last
// encoding is kept (it depends only on the two base pointers and the page
// count).
bool encode_cache_maps(const void* kv_buffer, const void* kv_scales, int64_t num_pages, CUtensorMap& kv_map,
                       CUtensorMap& sc_map) {
  struct Last {
    const void* kv = nullptr;
    const void* sc = nullptr;
    int64_t pages = -1;
    CUtensorMap kv_map, sc_map;
  };
  static thread_local Last last;
  if (last.kv == kv_buffer && last.sc == kv_scales && last.pages == num_pages) {
    kv_map = last.kv_map;
    sc_map = last.sc_map;
    return true;
  }
  const EncodeTiledFn enc = encode_tiled();
  if (!enc) return false;
  const cuuint64_t rows = static_cast<cuuint64_t>(num_pages > 0 ? num_pages : 1) * kimi::kPageSize;
  const cuuint32_t unit[2] = {1, 1};
  {
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(kimi::kTokenBytes), rows};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(kimi::kTokenBytes)};
    const cuuint32_t box[2] = {128, static_cast<cuuint32_t>(kimi::kPageSize)};
    if (enc(&kv_map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(kv_buffer), dims, strides, box, unit,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return false;
  }
  {
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(kimi::kScaleBytes), rows};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(kimi::kScaleBytes)};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(kimi::kScaleBytes), static_cast<cuuint32_t>(kimi::kPageSize)};
    if (enc(&sc_map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(kv_scales), dims, strides, box, unit,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return false;
  }
  last.kv = kv_buffer;
  last.sc = kv_scales;
  last.pages = num_pages;
  last.kv_map = kv_map;
  last.sc_map = sc_map;
  return true;
}

// A bf16 tensor map with 128-byte swizzle over `rank` dimensions (innermost
// first; strides in bytes for dimensions 1 ..), boxes of 64 elements (128 B)
// innermost.  Reads outside the tensor yield zeros.
bool encode_bf16_map(CUtensorMap& m, const void* base, cuuint32_t rank, const cuuint64_t* dims,
                     const cuuint64_t* strides, const cuuint32_t* box) {
  const EncodeTiledFn enc = encode_tiled();
  const cuuint32_t unit[3] = {1, 1, 1};
  return enc && enc(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), dims, strides, box, unit,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// How one call is laid out on the GPU.
//  * requested splits S > 0: split mode, every sequence cut into S equal tile
//    ranges (the reference's num_kv_splits), S = 1 writing the output directly;
//  * requested 0 (auto): balanced mode, one CTA per SM and head block (64
//    heads, or 16 for calls with at most 16 heads),
//    each a run over the batch's tiles laid end to end (see DecodeArgs in
//    kernels.cuh).
struct Plan {
  bool balanced;
  int ctas;  // balanced: CTAs per head block; split mode: splits per sequence
};

Plan resolve_plan(int32_t /*batch*/, int32_t num_heads, int32_t requested) {
  const int nh = kimi::decode_heads_per_cta(num_heads);
  const int head_blocks = (num_heads + nh - 1) / nh;
  if (requested > 0) return {false, requested > KIMI_MLA_MAX_SPLITS ? KIMI_MLA_MAX_SPLITS : requested};
  const int c = device_sm_count() / head_blocks;  // one CTA per SM and head block
  return {true, c < 1 ? 1 : c};
}

inline size_t round256(size_t n) { return (n + 255) & ~static_cast<size_t>(255); }

// Workspace: partial outputs [slots, heads, 512] bf16 (each normalised by its own
// softmax sum, so bf16 costs one rounding like the output's), log-sum-exps [slots,
// heads] fp32, then (balanced mode) [batch] int2 CTA spans, then the Q
// operand images [batch][head blocks] of q_image_bytes(nh) (nh heads per block:
// 64, or 16 for calls with at most 16 heads).  Split mode has
// batch * S slots (none for S = 1, and no workspace at all: the decode kernel
// then quantises Q itself, one piece per CTA), balanced mode batch + ctas.
struct Layout {
  size_t slots, po_bytes, lse_bytes, meta_bytes, qimg_bytes;
  size_t total() const { return po_bytes + lse_bytes + meta_bytes + qimg_bytes; }
};

Layout workspace_layout(int64_t batch, int64_t heads, const Plan& plan) {
  Layout l{};
  if (!plan.balanced && plan.ctas <= 1) return l;
  l.slots = plan.balanced ? static_cast<size_t>(batch + plan.ctas) : static_cast<size_t>(batch) * plan.ctas;
  l.po_bytes = round256(l.slots * heads * kLatent * sizeof(__nv_bfloat16));
  l.lse_bytes = round256(l.slots * heads * sizeof(float));
  l.meta_bytes = plan.balanced ? round256(static_cast<size_t>(batch) * 2 * sizeof(int32_t)) : 0;
  const int nh = kimi::decode_heads_per_cta(static_cast<int>(heads));
  l.qimg_bytes = round256(static_cast<size_t>(batch) * ((heads + nh - 1) / nh) * kimi::q_image_bytes(nh));
  return l;
}

}  // namespace

extern "C" {

int kimi_abi_version(void) { return KIMI_ABI_VERSION; }

const char* kimi_status_string(int status) {
  switch (status) {
    case KIMI_OK: return "ok";
    case KIMI_ERR_NULL_POINTER: return "null pointer argument";
    case KIMI_ERR_BAD_SHAPE: return "unsupported or inconsistent shape";
    case KIMI_ERR_BAD_STRIDE: return "unsupported stride";
    case KIMI_ERR_MISALIGNED: return "pointer or stride not aligned as required";
    case KIMI_ERR_WORKSPACE_TOO_SMALL: return "workspace too small";
    case KIMI_ERR_UNSUPPORTED: return "unsupported option";
    case KIMI_ERR_STATIC_WORKSPACE_LIMIT:
      return "split-K partials exceed the library's 32 MiB static workspace (use kimi_mla_decode with a caller workspace)";
    default: break;
  }
  if (status > 0 && status < KIMI_ERR_CUDA_BASE) {
    if (status & KIMI_DEVICE_PEER_WAIT)
      return "a peer rank did not reach the all-reduce barrier in time (the call's output is not valid)";
    if (status & KIMI_DEVICE_BAD_PAGE)
      return (status & ~KIMI_DEVICE_BAD_PAGE) ? "a device wait gave up; a page id was outside the cache"
                                              : "a page id was outside the cache (its tokens were read as zeros)";
    return "a device wait gave up (the call's output is not valid)";
  }
  if (status >= KIMI_ERR_CUDA_BASE) return cudaGetErrorString(static_cast<cudaError_t>(status - KIMI_ERR_CUDA_BASE));
  return "unknown status";
}

int32_t kimi_mla_decode_num_splits(int32_t batch, int32_t num_heads, int32_t num_kv_splits) {
  if (batch < 0 || num_heads < 1 || num_heads > KIMI_MLA_MAX_HEADS || num_kv_splits < 0) return 0;
  return resolve_plan(batch, num_heads, num_kv_splits).ctas;
}

size_t kimi_mla_decode_workspace_size(int32_t batch, int32_t num_heads, int32_t num_kv_splits) {
  if (batch < 0 || num_heads < 1 || num_heads > KIMI_MLA_MAX_HEADS || num_kv_splits < 0) return 0;
  return workspace_layout(batch, num_heads, resolve_plan(batch, num_heads, num_kv_splits)).total();
}

}  // extern "C"

namespace {

// Checked arguments of one decode call, ready to launch.
struct Prepared {
  Plan plan;
  kimi::DecodeArgs args;
  kimi::CacheMaps maps;
};

int prepare(const KimiMlaDecodeParams* p, void* workspace, size_t workspace_bytes, Prepared& out) {
  if (!p) return KIMI_ERR_NULL_POINTER;
  if (p->batch < 0 || p->num_heads < 1 || p->num_heads > KIMI_MLA_MAX_HEADS || p->num_kv_splits < 0 ||
      p->num_kv_splits > KIMI_MLA_MAX_SPLITS || p->num_pages < 0)
    return KIMI_ERR_BAD_SHAPE;
  if (p->logit_cap != 0.0f) return KIMI_ERR_UNSUPPORTED;
  if (!std::isfinite(p->sm_scale)) return KIMI_ERR_BAD_SHAPE;
  if (p->batch == 0) return KIMI_OK;
  if (!p->q || !p->kv_buffer || !p->kv_scales || !p->kv_indptr || !p->kv_indices || !p->o)
    return KIMI_ERR_NULL_POINTER;
  if (p->q_stride_b % 8 || p->q_stride_h % 8 || p->o_stride_b % 4 || p->o_stride_h % 4)
    return KIMI_ERR_BAD_STRIDE;
  if (!aligned(p->q, 16) || !aligned(p->kv_buffer, 16) || !aligned(p->kv_scales, 16) || !aligned(p->o, 8) ||
      !aligned(p->status, 4))
    return KIMI_ERR_MISALIGNED;
  const Plan plan = resolve_plan(p->batch, p->num_heads, p->num_kv_splits);
  const Layout lay = workspace_layout(p->batch, p->num_heads, plan);
  const size_t need = lay.total();
  if (need > 0) {
    if (!workspace || workspace_bytes < need) return KIMI_ERR_WORKSPACE_TOO_SMALL;
    if (!aligned(workspace, 256)) return KIMI_ERR_MISALIGNED;
  }
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  kimi::DecodeArgs& a = out.args;
  a.q = static_cast<const __nv_bfloat16*>(p->q);
  a.q_stride_b = p->q_stride_b;
  a.q_stride_h = p->q_stride_h;
  a.kv_buffer = static_cast<const uint8_t*>(p->kv_buffer);
  a.kv_scales = static_cast<const uint8_t*>(p->kv_scales);
  a.num_pages = p->num_pages;
  a.kv_indptr = p->kv_indptr;
  a.kv_indices = p->kv_indices;
  a.kv_last_page_len = p->kv_last_page_len;
  a.o = static_cast<__nv_bfloat16*>(p->o);
  a.o_stride_b = p->o_stride_b;
  a.o_stride_h = p->o_stride_h;
  a.partial_o = need ? reinterpret_cast<__nv_bfloat16*>(ws) : nullptr;
  a.partial_lse = need ? reinterpret_cast<float*>(ws + lay.po_bytes) : nullptr;
  a.seq_meta = plan.balanced ? reinterpret_cast<int2*>(ws + lay.po_bytes + lay.lse_bytes) : nullptr;
  a.q_img = lay.qimg_bytes ? ws + lay.po_bytes + lay.lse_bytes + lay.meta_bytes : nullptr;
  a.batch = p->batch;
  a.num_heads = p->num_heads;
  a.num_splits = plan.ctas;
  a.balanced = plan.balanced ? 1 : 0;
  a.sm_scale = p->sm_scale;
  a.status = p->status;
  a.timeout_ns = p->timeout_ns ? p->timeout_ns : kimi::kDefaultTimeoutNs;
  if (!encode_cache_maps(p->kv_buffer, p->kv_scales, p->num_pages, out.maps.kv, out.maps.sc))
    return KIMI_ERR_UNSUPPORTED;
  out.plan = plan;
  return KIMI_OK;
}

int launch_stage1(const Prepared& pr, cudaStream_t s) {
  if (pr.args.q_img) {
    const int st = cuda_status(kimi::launch_q_prep_fp4(pr.args, s));
    if (st != KIMI_OK) return st;
  }
  return cuda_status(kimi::launch_decode_fp4(pr.args, pr.maps, s));
}

// `after_stage1`: launched right after this call's stage-1 kernel on the same
// stream, which lets it start as its programmatic dependent.
int launch_merge(const Prepared& pr, cudaStream_t s, bool after_stage1) {
  if (!pr.plan.balanced && pr.plan.ctas == 1) return KIMI_OK;  // stage 1 wrote the output
  const kimi::DecodeArgs& a = pr.args;
  kimi::ReduceArgs r;
  r.partial_o = a.partial_o;
  r.partial_bf16 = 1;
  r.partial_lse = a.partial_lse;
  r.o = a.o;
  r.o_stride_b = a.o_stride_b;
  r.o_stride_h = a.o_stride_h;
  r.batch = a.batch;
  r.num_heads = a.num_heads;
  r.num_splits = pr.plan.ctas;
  r.seq_meta = a.seq_meta;
  r.kv_indptr = a.kv_indptr;
  r.programmatic = after_stage1 ? 1 : 0;
  return cuda_status(kimi::launch_reduce(r, s));
}

}  // namespace

extern "C" {

int kimi_mla_decode(const KimiMlaDecodeParams* p, void* workspace, size_t workspace_bytes, void* stream) {
  Prepared pr;
  int st = prepare(p, workspace, workspace_bytes, pr);
  if (st != KIMI_OK || p->batch == 0) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  st = launch_stage1(pr, s);
  return st != KIMI_OK ? st : launch_merge(pr, s, true);
}

int kimi_mla_decode_partial(const KimiMlaDecodeParams* p, void* workspace, size_t workspace_bytes, void* stream) {
  Prepared pr;
  const int st = prepare(p, workspace, workspace_bytes, pr);
  if (st != KIMI_OK || p->batch == 0) return st;
  return launch_stage1(pr, static_cast<cudaStream_t>(stream));
}

int kimi_mla_decode_merge(const KimiMlaDecodeParams* p, void* workspace, size_t workspace_bytes, void* stream) {
  Prepared pr;
  const int st = prepare(p, workspace, workspace_bytes, pr);
  if (st != KIMI_OK || p->batch == 0) return st;
  return launch_merge(pr, static_cast<cudaStream_t>(stream), false);
}

int kimi_mla_reduce(const KimiMlaReduceParams* p, void* stream) {
  if (!p) return KIMI_ERR_NULL_POINTER;
  if (p->batch < 0 || p->num_heads < 1 || p->num_heads > KIMI_MLA_MAX_HEADS || p->num_splits < 1 ||
      p->num_splits > KIMI_MLA_MAX_SPLITS)
    return KIMI_ERR_BAD_SHAPE;
  if (p->batch == 0) return KIMI_OK;
  if (!p->partial_o || !p->partial_lse || !p->o) return KIMI_ERR_NULL_POINTER;
  if (p->o_stride_b % 4 || p->o_stride_h % 4) return KIMI_ERR_BAD_STRIDE;
  if (!aligned(p->partial_o, 16) || !aligned(p->partial_lse, 4) || !aligned(p->o, 8)) return KIMI_ERR_MISALIGNED;
  kimi::ReduceArgs r;
  r.partial_o = p->partial_o;
  r.partial_bf16 = 0;
  r.partial_lse = p->partial_lse;
  r.o = static_cast<__nv_bfloat16*>(p->o);
  r.o_stride_b = p->o_stride_b;
  r.o_stride_h = p->o_stride_h;
  r.batch = p->batch;
  r.num_heads = p->num_heads;
  r.num_splits = p->num_splits;
  r.seq_meta = nullptr;
  r.kv_indptr = nullptr;
  r.programmatic = 0;
  return cuda_status(kimi::launch_reduce(r, static_cast<cudaStream_t>(stream)));
}

int kimi_mxfp4_kv_append(const KimiKvAppendParams* p, void* stream) {
  if (!p) return KIMI_ERR_NULL_POINTER;
  if (p->num_tokens < 0 || p->num_pages < 0) return KIMI_ERR_BAD_SHAPE;
  if (p->legacy_rule != 0 && p->legacy_rule != 1) return KIMI_ERR_UNSUPPORTED;
  if (p->num_tokens == 0) return KIMI_OK;
  if (!p->kv_c || !p->k_pe || !p->slot_mapping || !p->kv_buffer || !p->kv_scales) return KIMI_ERR_NULL_POINTER;
  if (p->kv_c_stride % 8 || p->k_pe_stride % 8 || p->kv_c_stride < kLatent || p->k_pe_stride < 64)
    return KIMI_ERR_BAD_STRIDE;
  if (!aligned(p->kv_c, 16) || !aligned(p->k_pe, 16) || !aligned(p->kv_buffer, 16) || !aligned(p->slot_mapping, 8))
    return KIMI_ERR_MISALIGNED;
  kimi::KvAppendArgs a;
  a.kv_c = static_cast<const __nv_bfloat16*>(p->kv_c);
  a.kv_c_stride = p->kv_c_stride;
  a.k_pe = static_cast<const __nv_bfloat16*>(p->k_pe);
  a.k_pe_stride = p->k_pe_stride;
  a.slot_mapping = p->slot_mapping;
  a.kv_buffer = static_cast<uint8_t*>(p->kv_buffer);
  a.kv_scales = static_cast<uint8_t*>(p->kv_scales);
  a.num_pages = p->num_pages;
  a.num_tokens = p->num_tokens;
  a.legacy_rule = p->legacy_rule;
  return cuda_status(kimi::launch_kv_append(a, static_cast<cudaStream_t>(stream)));
}

int kimi_mla_q_absorb_rope_append(const KimiQAbsorbParams* p, void* stream) {
  if (!p) return KIMI_ERR_NULL_POINTER;
  if (p->num_tokens < 0 || p->num_heads < 1 || p->num_heads > KIMI_MLA_MAX_HEADS || p->num_pages < 0 ||
      p->max_position < 1)
    return KIMI_ERR_BAD_SHAPE;
  if ((p->is_neox != 0 && p->is_neox != 1) || (p->legacy_rule != 0 && p->legacy_rule != 1))
    return KIMI_ERR_UNSUPPORTED;
  if (p->num_tokens == 0) return KIMI_OK;
  if (!p->q_nope || !p->q_pe || !p->w_uk || !p->kv_c || !p->k_pe || !p->positions || !p->cos_cache ||
      !p->sin_cache || !p->slot_mapping || !p->kv_buffer || !p->kv_scales || !p->q_out)
    return KIMI_ERR_NULL_POINTER;
  const int64_t strides[] = {p->q_nope_stride_t, p->q_nope_stride_h, p->q_pe_stride_t, p->q_pe_stride_h,
                             p->kv_c_stride,     p->k_pe_stride,     p->q_out_stride_t, p->q_out_stride_h};
  for (int64_t st : strides)
    if (st % 8 || st < 0) return KIMI_ERR_BAD_STRIDE;
  if (p->kv_c_stride < kLatent || p->k_pe_stride < 64) return KIMI_ERR_BAD_STRIDE;
  if (!aligned(p->q_nope, 16) || !aligned(p->q_pe, 16) || !aligned(p->w_uk, 16) || !aligned(p->kv_c, 16) ||
      !aligned(p->k_pe, 2) || !aligned(p->kv_buffer, 16) || !aligned(p->q_out, 16) ||
      !aligned(p->positions, 8) || !aligned(p->slot_mapping, 8) || !aligned(p->cos_cache, 16) ||
      !aligned(p->sin_cache, 16))
    return KIMI_ERR_MISALIGNED;
  kimi::QAbsorbArgs a;
  a.q_nope = static_cast<const __nv_bfloat16*>(p->q_nope);
  a.q_nope_stride_t = p->q_nope_stride_t;
  a.q_nope_stride_h = p->q_nope_stride_h;
  a.q_pe = static_cast<const __nv_bfloat16*>(p->q_pe);
  a.q_pe_stride_t = p->q_pe_stride_t;
  a.q_pe_stride_h = p->q_pe_stride_h;
  a.w_uk = static_cast<const __nv_bfloat16*>(p->w_uk);
  a.kv_c = static_cast<const __nv_bfloat16*>(p->kv_c);
  a.kv_c_stride = p->kv_c_stride;
  a.k_pe = static_cast<const __nv_bfloat16*>(p->k_pe);
  a.k_pe_stride = p->k_pe_stride;
  a.positions = p->positions;
  a.cos = p->cos_cache;
  a.sin = p->sin_cache;
  a.max_position = p->max_position;
  a.slot_mapping = p->slot_mapping;
  a.kv_buffer = static_cast<uint8_t*>(p->kv_buffer);
  a.kv_scales = static_cast<uint8_t*>(p->kv_scales);
  a.num_pages = p->num_pages;
  a.q_out = static_cast<__nv_bfloat16*>(p->q_out);
  a.q_out_stride_t = p->q_out_stride_t;
  a.q_out_stride_h = p->q_out_stride_h;
  a.num_tokens = p->num_tokens;
  a.num_heads = p->num_heads;
  a.is_neox = p->is_neox;
  a.legacy_rule = p->legacy_rule;
  if (p->status && !aligned(p->status, 4)) return KIMI_ERR_MISALIGNED;
  a.status = p->status;
  return cuda_status(kimi::launch_q_absorb(a, static_cast<cudaStream_t>(stream)));
}

int kimi_ar_rmsnorm_mxfp4(const KimiArRmsNormParams* p, void* stream) {
  if (!p) return KIMI_ERR_NULL_POINTER;
  if (p->rows < 0 || p->hidden < 32 || p->hidden % 32 || p->hidden > 8192 || p->num_inputs < 1 ||
      p->num_inputs > KIMI_AR_MAX_INPUTS || !std::isfinite(p->eps) || p->eps < 0.f)
    return KIMI_ERR_BAD_SHAPE;
  if (p->legacy_rule != 0 && p->legacy_rule != 1) return KIMI_ERR_UNSUPPORTED;
  if (p->rows == 0) return KIMI_OK;
  if (!p->residual || !p->residual_out || !p->weight || !p->nibbles || !p->scales) return KIMI_ERR_NULL_POINTER;
  kimi::ArNormArgs a;
  for (int i = 0; i < p->num_inputs; ++i) {
    if (!p->inputs[i]) return KIMI_ERR_NULL_POINTER;
    if (!aligned(p->inputs[i], 16)) return KIMI_ERR_MISALIGNED;
    a.inputs[i] = static_cast<const __nv_bfloat16*>(p->inputs[i]);
  }
  for (int i = p->num_inputs; i < kimi::kArMaxInputs; ++i) a.inputs[i] = nullptr;
  if (!aligned(p->residual, 16) || !aligned(p->residual_out, 16) || !aligned(p->weight, 16) ||
      !aligned(p->nibbles, 16))
    return KIMI_ERR_MISALIGNED;
  a.num_inputs = p->num_inputs;
  a.residual = static_cast<const __nv_bfloat16*>(p->residual);
  a.residual_out = static_cast<__nv_bfloat16*>(p->residual_out);
  a.weight = static_cast<const __nv_bfloat16*>(p->weight);
  a.eps = p->eps;
  a.nibbles = static_cast<uint8_t*>(p->nibbles);
  a.scales = static_cast<uint8_t*>(p->scales);
  a.rows = p->rows;
  a.hidden = p->hidden;
  a.legacy_rule = p->legacy_rule;
  return cuda_status(kimi::launch_ar_norm_quant(a, static_cast<cudaStream_t>(stream)));
}

int kimi_ar_rmsnorm_mxfp4_two_shot(const KimiArTwoShotParams* p, void* stream) {
  if (!p) return KIMI_ERR_NULL_POINTER;
  if (p->rows < 0 || p->hidden < 32 || p->hidden % 32 || p->hidden > 8192 || p->world < 1 ||
      p->world > KIMI_AR_MAX_INPUTS || p->rank < 0 || p->rank >= p->world || !std::isfinite(p->eps) || p->eps < 0.f)
    return KIMI_ERR_BAD_SHAPE;
  if (p->legacy_rule != 0 && p->legacy_rule != 1) return KIMI_ERR_UNSUPPORTED;
  if (!p->counter || !p->residual || !p->weight) return KIMI_ERR_NULL_POINTER;
  if (!aligned(p->counter, 4) || !aligned(p->residual, 16) || !aligned(p->weight, 16) ||
      (p->status && !aligned(p->status, 4)))
    return KIMI_ERR_MISALIGNED;
  kimi::ArTwoShotArgs t{};
  for (int r = 0; r < kimi::kArMaxInputs; ++r) {
    if (r >= p->world) break;
    if (!p->inputs[r] || !p->residual_out[r] || !p->nibbles[r] || !p->scales[r] || !p->flags[r])
      return KIMI_ERR_NULL_POINTER;
    if (!aligned(p->inputs[r], 16) || !aligned(p->residual_out[r], 16) || !aligned(p->nibbles[r], 16) ||
        !aligned(p->flags[r], 4))
      return KIMI_ERR_MISALIGNED;
    t.base.inputs[r] = static_cast<const __nv_bfloat16*>(p->inputs[r]);
    t.residual_out[r] = static_cast<__nv_bfloat16*>(p->residual_out[r]);
    t.nibbles[r] = static_cast<uint8_t*>(p->nibbles[r]);
    t.scales[r] = static_cast<uint8_t*>(p->scales[r]);
    t.flags[r] = p->flags[r];
  }
  t.base.num_inputs = p->world;
  t.base.residual = static_cast<const __nv_bfloat16*>(p->residual);
  t.base.weight = static_cast<const __nv_bfloat16*>(p->weight);
  t.base.eps = p->eps;
  t.base.rows = p->rows;
  t.base.hidden = p->hidden;
  t.base.legacy_rule = p->legacy_rule;
  t.counter = p->counter;
  t.status = p->status;
  t.timeout_ns = p->timeout_ns ? p->timeout_ns : kimi::kDefaultTimeoutNs;
  t.world = p->world;
  t.rank = p->rank;
  // zero rows still take part in both barriers (every rank makes the same calls)
  return cuda_status(kimi::launch_ar_two_shot(t, static_cast<cudaStream_t>(stream)));
}

int kimi_mla_v_up_o_proj(const KimiVUpOProjParams* p, void* stream) {
  if (!p) return KIMI_ERR_NULL_POINTER;
  if (p->num_tokens < 0 || p->num_heads < 1 || p->num_heads > 8 || p->hidden < 64 || p->hidden % 64)
    return KIMI_ERR_BAD_SHAPE;
  if (p->num_tokens == 0) return KIMI_OK;
  if (!p->o || !p->w_uv || !p->w_o || !p->x || !p->out) return KIMI_ERR_NULL_POINTER;
  if (p->o_stride_t % 8 || p->o_stride_h % 8 || p->o_stride_t < 512 || p->o_stride_h < 0 ||
      (p->num_heads > 1 && p->o_stride_h == 0) || p->out_stride % 8 || p->out_stride < p->hidden)
    return KIMI_ERR_BAD_STRIDE;
  if (!aligned(p->o, 16) || !aligned(p->w_uv, 16) || !aligned(p->w_o, 16) || !aligned(p->x, 16) ||
      !aligned(p->out, 16))
    return KIMI_ERR_MISALIGNED;
  kimi::VUpOProjArgs a;
  a.o = static_cast<const __nv_bfloat16*>(p->o);
  a.o_stride_h = p->o_stride_h;
  a.o_stride_t = p->o_stride_t;
  a.w_uv = static_cast<const __nv_bfloat16*>(p->w_uv);
  a.w_o = static_cast<const __nv_bfloat16*>(p->w_o);
  a.x = static_cast<__nv_bfloat16*>(p->x);
  a.out = static_cast<__nv_bfloat16*>(p->out);
  a.out_stride = p->out_stride;
  a.num_tokens = p->num_tokens;
  a.num_heads = p->num_heads;
  a.hidden = p->hidden;
  if (p->status && !aligned(p->status, 4)) return KIMI_ERR_MISALIGNED;
  a.status = p->status;
  const cuuint64_t T = static_cast<cuuint64_t>(p->num_tokens), H = static_cast<cuuint64_t>(p->num_heads);
  const cuuint64_t K = 128 * H, stride_t = 2 * static_cast<cuuint64_t>(p->o_stride_t);
  // a single head's stride is never used: give it the extent of the tokens
  const cuuint64_t stride_h = p->num_heads > 1 ? 2 * static_cast<cuuint64_t>(p->o_stride_h) : T * stride_t;
  kimi::VUpOProjMaps maps;
  {
    const cuuint64_t dims[3] = {512, T, H}, strides[2] = {stride_t, stride_h};
    const cuuint32_t box[3] = {64, static_cast<cuuint32_t>(kimi::kVUpRows), 1};
    if (!encode_bf16_map(maps.o, p->o, 3, dims, strides, box)) return KIMI_ERR_BAD_STRIDE;
  }
  {
    const cuuint64_t dims[2] = {128, 512 * H}, strides[1] = {256};
    const cuuint32_t box[2] = {64, 64};
    if (!encode_bf16_map(maps.w_uv, p->w_uv, 2, dims, strides, box)) return KIMI_ERR_UNSUPPORTED;
  }
  {
    const cuuint64_t dims[2] = {K, T}, strides[1] = {2 * K};
    const cuuint32_t box[2] = {64, 128};
    if (!encode_bf16_map(maps.x, p->x, 2, dims, strides, box)) return KIMI_ERR_UNSUPPORTED;
  }
  {
    const cuuint64_t dims[2] = {K, static_cast<cuuint64_t>(p->hidden)}, strides[1] = {2 * K};
    const cuuint32_t box[2] = {64, 64};
    if (!encode_bf16_map(maps.w_o, p->w_o, 2, dims, strides, box)) return KIMI_ERR_UNSUPPORTED;
  }
  return cuda_status(kimi::launch_v_up_o_proj(a, maps, static_cast<cudaStream_t>(stream)));
}

int kimi_device_status(int32_t* device_word, int32_t clear, void* stream) {
  if (!device_word) return KIMI_ERR_NULL_POINTER;
  if (!aligned(device_word, 4)) return KIMI_ERR_MISALIGNED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int32_t host = 0;
  cudaError_t e = cudaMemcpyAsync(&host, device_word, sizeof(host), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e == cudaSuccess && clear) e = cudaMemsetAsync(device_word, 0, sizeof(int32_t), s);
  if (e != cudaSuccess) return cuda_status(e);
  return host & 0x1FFF;
}

int kimi_mxfp4_quantize(const void* x, int64_t rows, int64_t cols, int64_t x_stride, void* nibbles, void* scales,
                        int32_t legacy_rule, void* stream) {
  if (rows < 0 || cols < 0 || cols % 32) return KIMI_ERR_BAD_SHAPE;
  if (legacy_rule != 0 && legacy_rule != 1) return KIMI_ERR_UNSUPPORTED;
  if (rows == 0 || cols == 0) return KIMI_OK;
  if (!x || !nibbles || !scales) return KIMI_ERR_NULL_POINTER;
  if (x_stride % 8 || x_stride < cols) return KIMI_ERR_BAD_STRIDE;
  if (!aligned(x, 16) || !aligned(nibbles, 16)) return KIMI_ERR_MISALIGNED;
  kimi::QuantizeArgs a;
  a.x = static_cast<const __nv_bfloat16*>(x);
  a.rows = rows;
  a.cols = cols;
  a.x_stride = x_stride;
  a.nibbles = static_cast<uint8_t*>(nibbles);
  a.scales = static_cast<uint8_t*>(scales);
  a.legacy_rule = legacy_rule;
  return cuda_status(kimi::launch_quantize_rows(a, static_cast<cudaStream_t>(stream)));
}

}  // extern "C"
