/*
 * kimi_mla.h -- C ABI of the B200 (sm_100a) MXFP4 absorbed-MLA decode path.
 *
 * Plain C: device pointers, sizes, element strides and a cudaStream_t passed
 * as `void*`.  No C++ or torch types cross this boundary.  Every entry point
 * is asynchronous on the given stream, allocates nothing, never synchronises
 * the host and returns a status code:
 *
 *      0                  success (KIMI_OK)
 *      negative           bad arguments, detected on the host before launch
 *      1 .. 0xFFFF        a device status word read back by kimi_device_status
 *                         (KIMI_DEVICE_* bits: a bounded device wait gave up,
 *                         a page id lay outside the cache, or a peer rank did
 *                         not reach an all-reduce barrier in time)
 *      >= 0x10000         a CUDA runtime error from the launch (the cudaError_t
 *                         value plus KIMI_ERR_CUDA_BASE)
 *
 * Reference interfaces replaced (paths inside the ianye23301/kimi tree):
 *
 *   kimi_mla_decode            aiter `mla_decode_fwd(q, kv_buffer, o, qo_indptr,
 *                              kv_indptr, kv_indices, kv_last_page_len,
 *                              max_seqlen_q, page_size, nhead_kv, sm_scale,
 *                              logit_cap, num_kv_splits, ...)` as called at
 *                              scripts/submission.py:115-133 and
 *                              patches/atom-optimizations.patch:741-748, and
 *                              the archive's `mla_decode_mxfp4`
 *                              (archive/mla-mxfp4-dead-end/mla_decode_mxfp4_v5.py:313-376).
 *                              Writes `o` in place; `o` may be the heads-first
 *                              permuted view (patches/atom-optimizations.patch:261-289).
 *   kimi_mla_decode_workspace_size
 *                              the caller-owned split-K buffer of the reference
 *                              (`attn_logits`, tests/test_triton_mla_decode.py:137-140,
 *                              patches/atom-optimizations.patch:192-197).
 *   kimi_mla_reduce            the split-K log-sum-exp merge `_mla_reduce`
 *                              (archive/mla-mxfp4-dead-end/mla_decode_mxfp4_v5.py:264-306),
 *                              aiter's stage-2 `_fwd_kernel_stage2_asm`.
 *   kimi_mxfp4_kv_append       the KV-append cache writer
 *                              `fused_qk_rope_concat_and_cache_mla(..., slot_mapping, ...)`
 *                              (patches/atom-optimizations.patch:615-634) with the
 *                              MXFP4 quantiser `_mxfp4_quant_inline`
 *                              (archive/mla-mxfp4-dead-end/mla_decode_mxfp4_v5.py:18-75)
 *                              or, with legacy_rule = 1, `_quantize_mxfp4_torch`
 *                              (same file, :421-438).
 *   kimi_mxfp4_quantize        row quantiser with the same two rules (aiter
 *                              `dynamic_mxfp4_quant`, archive/mla-mxfp4-dead-end/mla_decode_mxfp4.py:139-156).
 *
 * Cache layout (one KV head, page size 64):
 *   kv_buffer  uint8 [num_pages, 64, 384]: per token 256 bytes of e2m1 nibbles
 *              of the 512-dim latent (element 2j in the low nibble of byte j)
 *              followed by the 64-dim RoPE part as 128 bytes of bf16.
 *   kv_scales  uint8 [num_pages, 64, 16]: per token 16 e8m0 scale bytes, one
 *              per 32 latent elements; value = e2m1 * 2^(scale - 127).
 * Both arrays are contiguous and 16-byte aligned.
 */
#ifndef KIMI_MLA_H_
#define KIMI_MLA_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define KIMI_API __attribute__((visibility("default")))
#else
#define KIMI_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define KIMI_MLA_KV_LORA_RANK 512
#define KIMI_MLA_ROPE_DIM 64
#define KIMI_MLA_QK_DIM 576
#define KIMI_MLA_PAGE_SIZE 64
#define KIMI_MLA_TOKEN_BYTES 384
#define KIMI_MLA_SCALE_BYTES 16
#define KIMI_MLA_MAX_SPLITS 64
#define KIMI_MLA_MAX_HEADS 128
#define KIMI_MLA_STATIC_WORKSPACE_BYTES 33554432u /* 32 MiB, see kimi_mla_decode_static_workspace */
#define KIMI_ABI_VERSION 201

/* Bits the decode kernels OR into the caller's device status word
 * (KimiMlaDecodeParams.status).  Every device-side wait of the decode is
 * bounded in time (KimiMlaDecodeParams.timeout_ns); a wait that runs out
 * ends the CTA's work cleanly, leaves that CTA's part of the output unwritten
 * and sets one of the wait bits.  The reference raises a Python exception
 * instead (patches/atom-optimizations.patch:125-128). */
#define KIMI_DEVICE_SOFTMAX_WAIT    0x001
#define KIMI_DEVICE_SOFTMAX_PV_WAIT 0x002
#define KIMI_DEVICE_EPILOGUE_WAIT   0x004
#define KIMI_DEVICE_SCALE_WAIT      0x008
#define KIMI_DEVICE_ISSUER_WAIT     0x010
#define KIMI_DEVICE_ISSUER_PV_WAIT  0x020
#define KIMI_DEVICE_CONVERTER_WAIT  0x040
#define KIMI_DEVICE_DRAIN_WAIT      0x080
#define KIMI_DEVICE_PRODUCER_WAIT   0x100
/* A kv_indices entry outside [0, num_pages) (negative included): nothing
 * is read from outside the cache; that page reads as zeros (zero keys and
 * values, so its 64 tokens still take part in the softmax with score 0 and
 * add nothing to the output), the rest of the sequence is decoded as usual,
 * and this bit is set.  The reference indexes the cache tensor with the id
 * and raises an index error (or reads another page for a negative id). */
#define KIMI_DEVICE_BAD_PAGE        0x200
/* The two-shot all-reduce (kimi_ar_rmsnorm_mxfp4_two_shot): a rank did not
 * reach the entry or exit barrier within the call's timeout_ns. */
#define KIMI_DEVICE_PEER_WAIT       0x400
/* The decode prologue (kimi_mla_q_absorb_rope_append) and the V up-projection
 * + o_proj (kimi_mla_v_up_o_proj): a wait gave up.  Their waits keep a fixed
 * bound of about 2 s (their give-up paths do not wait for the copies and
 * MMAs already issued, so no shorter caller-set bound is offered). */
#define KIMI_DEVICE_QABSORB_WAIT    0x800
#define KIMI_DEVICE_VUP_WAIT        0x1000

enum {
  KIMI_OK = 0,
  KIMI_ERR_NULL_POINTER = -1,
  KIMI_ERR_BAD_SHAPE = -2,
  KIMI_ERR_BAD_STRIDE = -3,
  KIMI_ERR_MISALIGNED = -4,
  KIMI_ERR_WORKSPACE_TOO_SMALL = -5,
  KIMI_ERR_UNSUPPORTED = -6,
  KIMI_ERR_STATIC_WORKSPACE_LIMIT = -7,
  KIMI_ERR_CUDA_BASE = 0x10000 /* above every combination of KIMI_DEVICE_* bits */
};

/* Arguments of one decode call.  Element strides are in elements of the
 * pointed-to type; the innermost dimension of q and o is contiguous. */
typedef struct KimiMlaDecodeParams {
  const void* q;              /* bf16 [batch, num_heads, 576] */
  int64_t q_stride_b;
  int64_t q_stride_h;
  const void* kv_buffer;      /* uint8 [num_pages, 64, 384] */
  const void* kv_scales;      /* uint8 [num_pages, 64, 16]  */
  int64_t num_pages;
  const int32_t* kv_indptr;   /* [batch + 1] page-table offsets */
  const int32_t* kv_indices;  /* [kv_indptr[batch]] page ids    */
  const int32_t* kv_last_page_len; /* [batch] tokens in the last page (1..64); NULL = full pages */
  void* o;                    /* bf16 [batch, num_heads, 512], any (b, h) strides */
  int64_t o_stride_b;
  int64_t o_stride_h;
  int32_t batch;
  int32_t num_heads;          /* 1..128 */
  int32_t num_kv_splits;      /* 1..64 equal splits per sequence, or 0 = balanced schedule (below) */
  float sm_scale;
  float logit_cap;            /* must be 0 (no logit soft-capping on this path) */
  int32_t* status;            /* optional device word (4-byte aligned): KIMI_DEVICE_* bits are ORed
                                 into it; never cleared by the library.  NULL = not reported. */
  uint64_t timeout_ns;        /* bound of each device-side wait in nanoseconds; 0 = 2 s */
} KimiMlaDecodeParams;

/* Bytes of caller-owned workspace one kimi_mla_decode call needs (split-K
 * partial outputs and log-sum-exps, and the quantised Q operands).
 * num_kv_splits as in the params.  Returns 0 for invalid sizes.
 *
 * num_kv_splits = S > 0 cuts every sequence into S equal ranges of 128-token
 * tiles, as the reference's num_kv_splits does (S = 1 needs no workspace).
 * num_kv_splits = 0 selects the balanced schedule: the batch's tiles are laid
 * end to end and split evenly over one CTA per SM per head block, so
 * ragged batches and batches smaller than the SM count keep every SM busy;
 * sequences that one CTA covers are written directly, the others merged.
 * A head block is 64 heads, or 16 when num_heads <= 16 (a tensor-parallel
 * shard such as 8 heads per GPU).
 * The workspace holds slots x heads x 1028 bytes of partials (bf16 rows and
 * fp32 log-sum-exps; slots = batch x S, or batch + CTAs when balanced), 8
 * bytes per sequence when balanced, and Q operands per sequence and head
 * block (60416 bytes for a 64-head block, 15104 for a 16-head block), each
 * part rounded up to 256 bytes. */
KIMI_API size_t kimi_mla_decode_workspace_size(int32_t batch, int32_t num_heads, int32_t num_kv_splits);

/* S for num_kv_splits = S > 0 (capped at 64); for 0, the balanced schedule's
 * CTAs per head block on the current device. */
KIMI_API int32_t kimi_mla_decode_num_splits(int32_t batch, int32_t num_heads, int32_t num_kv_splits);

/* Absorbed-MLA decode, one query token per sequence, one KV head. */
KIMI_API int kimi_mla_decode(const KimiMlaDecodeParams* params, void* workspace, size_t workspace_bytes,
                    void* stream);

/* The two launches of kimi_mla_decode, for callers that schedule them apart
 * (the archive wrapper `mla_decode_mxfp4` likewise launches its stage-1
 * kernel `_mla_decode_split_kv` and then `_mla_reduce`,
 * archive/mla-mxfp4-dead-end/mla_decode_mxfp4_v5.py:313-376).  Same params
 * and workspace in both calls, in stream order: kimi_mla_decode_partial runs
 * the split-K attention (it alone writes the output when no merge is needed),
 * kimi_mla_decode_merge the log-sum-exp merge of its partials (nothing when
 * there are none). */
KIMI_API int kimi_mla_decode_partial(const KimiMlaDecodeParams* params, void* workspace, size_t workspace_bytes,
                                     void* stream);
KIMI_API int kimi_mla_decode_merge(const KimiMlaDecodeParams* params, void* workspace, size_t workspace_bytes,
                                   void* stream);

/* Same decode as kimi_mla_decode, for callers that cannot allocate device
 * memory.  No counterpart in the reference: aiter and the archive kernels
 * always take (or allocate) their split-K buffers.  Callers such as a
 * foreign-language binding holding only the pointers an engine handed it, or
 * an engine that reserved all free HBM up front, have no way to obtain the
 * workspace kimi_mla_decode needs; this call takes it from a 32 MiB array
 * compiled into the library instead (KIMI_MLA_STATIC_WORKSPACE_BYTES, held on
 * every GPU that loads the library until exit) and allocates nothing.
 *  - Returns KIMI_ERR_STATIC_WORKSPACE_LIMIT, launching nothing, when
 *    kimi_mla_decode_workspace_size() for these sizes exceeds 32 MiB.
 *  - All calls on a device share the array and it keeps the last call's
 *    contents; calls that overlap on the GPU race, so order them on one
 *    stream.  Nothing in it needs clearing between calls.
 *  - The first call on a device looks up the array's device address
 *    (cudaGetSymbolAddress, with that device current); make that first call
 *    before any stream capture begins. */
KIMI_API int kimi_mla_decode_static_workspace(const KimiMlaDecodeParams* params, void* stream);

/* Split-K merge.  partial_o float32 [batch, num_splits, num_heads, 512]
 * (each split normalised by its own softmax sum), partial_lse float32
 * [batch, num_splits, num_heads] (natural-log log-sum-exp of the split's
 * scaled scores; -inf for an empty split).  Writes bf16 o through strides. */
typedef struct KimiMlaReduceParams {
  const float* partial_o;
  const float* partial_lse;
  void* o;
  int64_t o_stride_b;
  int64_t o_stride_h;
  int32_t batch;
  int32_t num_heads;
  int32_t num_splits;
} KimiMlaReduceParams;

KIMI_API int kimi_mla_reduce(const KimiMlaReduceParams* params, void* stream);

/* Quantise kv_c (bf16 [num_tokens, 512]) to MXFP4 and write it, with k_pe
 * (bf16 [num_tokens, 64]) copied verbatim, into the paged cache at flat slots
 * slot_mapping[i] = page * 64 + row.  A negative slot skips its token; a slot
 * >= num_pages * 64 is an error the kernel skips (the host cannot see device
 * slot values without a sync).  legacy_rule: 0 = the in-kernel Triton rule,
 * 1 = the reference's legacy torch rule. */
typedef struct KimiKvAppendParams {
  const void* kv_c;           /* bf16 [num_tokens, 512] */
  int64_t kv_c_stride;
  const void* k_pe;           /* bf16 [num_tokens, 64] */
  int64_t k_pe_stride;
  const int64_t* slot_mapping; /* [num_tokens] */
  void* kv_buffer;            /* uint8 [num_pages, 64, 384] */
  void* kv_scales;            /* uint8 [num_pages, 64, 16]  */
  int64_t num_pages;
  int32_t num_tokens;
  int32_t legacy_rule;
} KimiKvAppendParams;

KIMI_API int kimi_mxfp4_kv_append(const KimiKvAppendParams* params, void* stream);

/* The decode step before attention, fused into one launch.  Replaces the
 * reference's k_up_proj BMM + RoPE + cache write (`MLAAttention.fused_kv_bmm`
 * and `fused_qk_rope_concat_and_cache_mla`, patches/atom-optimizations.patch:468-639):
 *   q_out[t, h, :512] = q_nope[t, h, :] @ w_uk[h]          (q absorbed into the latent)
 *   q_out[t, h, 512:] = rope(q_pe[t, h, :], positions[t])
 *   cache[slot_mapping[t]] = MXFP4(kv_c[t]) ++ rope(k_pe[t], positions[t])
 * RoPE: 32 frequency pairs (x[i], x[i+32]) when is_neox, else (x[2i], x[2i+1]);
 * (a, b) -> (a cos - b sin, b cos + a sin) with cos / sin float32
 * [max_position, 32] indexed by the position.  A token whose slot is negative
 * or out of range, or whose position is out of range, is not written to the
 * cache; an out-of-range position also zeroes its q_out RoPE part.  Element
 * strides: q_nope / q_pe / q_out per token and per head, kv_c / k_pe per
 * token, all multiples of 8; w_uk is contiguous [num_heads, 128, 512]. */
typedef struct KimiQAbsorbParams {
  const void* q_nope;          /* bf16 [num_tokens, num_heads, 128] */
  int64_t q_nope_stride_t, q_nope_stride_h;
  const void* q_pe;            /* bf16 [num_tokens, num_heads, 64] */
  int64_t q_pe_stride_t, q_pe_stride_h;
  const void* w_uk;            /* bf16 [num_heads, 128, 512] */
  const void* kv_c;            /* bf16 [num_tokens, 512] */
  int64_t kv_c_stride;
  const void* k_pe;            /* bf16 [num_tokens, 64], before RoPE */
  int64_t k_pe_stride;
  const int64_t* positions;    /* [num_tokens] */
  const float* cos_cache;      /* [max_position, 32] */
  const float* sin_cache;      /* [max_position, 32] */
  int64_t max_position;
  const int64_t* slot_mapping; /* [num_tokens] */
  void* kv_buffer;             /* uint8 [num_pages, 64, 384] */
  void* kv_scales;             /* uint8 [num_pages, 64, 16]  */
  int64_t num_pages;
  void* q_out;                 /* bf16 [num_tokens, num_heads, 576] */
  int64_t q_out_stride_t, q_out_stride_h;
  int32_t num_tokens;
  int32_t num_heads;
  int32_t is_neox;
  int32_t legacy_rule;
  int32_t* status;             /* optional device word: KIMI_DEVICE_QABSORB_WAIT when a wait gave up
                                  (each wait keeps a fixed ~2 s bound); NULL = not reported */
} KimiQAbsorbParams;

KIMI_API int kimi_mla_q_absorb_rope_append(const KimiQAbsorbParams* params, void* stream);

/* The layer-input step after the tensor-parallel all-reduce, in one kernel.
 * Replaces the fused one-shot all-reduce + residual + RMSNorm
 * (`allreduce_fusion_kernel_1stage_nloop`, patches/aiter-1stage-nloop-ar-rmsnorm.patch:12-253)
 * and the MXFP4 quant-only step after it (patches/aiter-mxfp4-quant-only.patch:29-125):
 *   residual_out = bf16(inputs[0] + ... + inputs[n-1] + residual)   (float32 sum, rank order)
 *   out          = bf16(bf16(residual_out * rsqrt(mean(residual_out^2) + eps)) * weight)
 *   nibbles / scales = MXFP4(out), scales unshuffled [rows, hidden / 32].
 * inputs[] are the ranks' partial outputs, each bf16 [rows, hidden]
 * contiguous: device pointers this GPU can read (its own buffer and peer
 * buffers mapped over NVLink).  The caller orders the call after every
 * partial is written and keeps the partials unchanged until every rank's call
 * has finished (the call itself waits for nothing).  hidden: a multiple of 32,
 * at most 8192.  residual_out may alias residual. */
#define KIMI_AR_MAX_INPUTS 8
typedef struct KimiArRmsNormParams {
  const void* inputs[KIMI_AR_MAX_INPUTS]; /* bf16 [rows, hidden] each */
  int32_t num_inputs;
  const void* residual;        /* bf16 [rows, hidden] */
  void* residual_out;          /* bf16 [rows, hidden] */
  const void* weight;          /* bf16 [hidden] */
  float eps;
  void* nibbles;               /* uint8 [rows, hidden / 2] */
  void* scales;                /* uint8 [rows, hidden / 32] */
  int32_t rows;
  int32_t hidden;
  int32_t legacy_rule;
} KimiArRmsNormParams;

KIMI_API int kimi_ar_rmsnorm_mxfp4(const KimiArRmsNormParams* params, void* stream);

/* The same step as a two-shot exchange over peer memory, with its own device
 * barriers (the same reference interface as kimi_ar_rmsnorm_mxfp4).  Every
 * rank of `world` calls it with the same rows, hidden, eps and weight values;
 * rank r computes rows [r rows / world, (r + 1) rows / world) from all
 * ranks' partials and stores those rows' residual_out, nibbles and scales into
 * every rank's buffers, so that when the call completes each rank holds all
 * rows.  The call waits on the device for the other ranks twice (at entry, so
 * that no partial is read before its rank has written it; at exit, so that no
 * rank reuses its partial while another still reads it): no host barrier is
 * needed around it.  Each wait is bounded by timeout_ns (0 = 2 s); a wait
 * that runs out sets KIMI_DEVICE_PEER_WAIT in *status and leaves the rows of
 * that call undefined.
 * Pointer arrays are indexed by rank; all of them are device pointers this
 * GPU can read and write (its own buffers and peer buffers mapped over
 * NVLink, for example with CUDA IPC).  flags: every rank's int32
 * [2 * KIMI_AR_MAX_INPUTS], zero before the first call; counter: this rank's
 * int32 [2], zero before the first call: [0] counts the call's CTAs (each call
 * leaves it zero), [1] numbers the calls (each call reads it, uses the next
 * number as the barriers' epoch and leaves it there), so a call captured in a
 * CUDA graph may be replayed.  Every rank makes the same sequence of calls.
 * No TMA or bulk copy touches peer memory: plain loads and stores only. */
typedef struct KimiArTwoShotParams {
  const void* inputs[KIMI_AR_MAX_INPUTS];  /* every rank's partial, bf16 [rows, hidden] */
  void* residual_out[KIMI_AR_MAX_INPUTS];  /* every rank's bf16 [rows, hidden] */
  void* nibbles[KIMI_AR_MAX_INPUTS];       /* every rank's uint8 [rows, hidden / 2] */
  void* scales[KIMI_AR_MAX_INPUTS];        /* every rank's uint8 [rows, hidden / 32] */
  int32_t* flags[KIMI_AR_MAX_INPUTS];      /* every rank's int32 [2 * KIMI_AR_MAX_INPUTS] */
  int32_t* counter;                        /* this rank's int32 [2] (CTA count, call number) */
  const void* residual;                    /* this rank's bf16 [rows, hidden] (equal on every rank) */
  const void* weight;                      /* bf16 [hidden] */
  float eps;
  int32_t rows;
  int32_t hidden;
  int32_t legacy_rule;
  int32_t world;                           /* 1 .. KIMI_AR_MAX_INPUTS */
  int32_t rank;
  int32_t* status;                         /* optional device word (KIMI_DEVICE_PEER_WAIT) */
  uint64_t timeout_ns;
} KimiArTwoShotParams;

KIMI_API int kimi_ar_rmsnorm_mxfp4_two_shot(const KimiArTwoShotParams* params, void* stream);

/* The decode step after attention: V up-projection of the heads-first latent
 * output, then o_proj.  Replaces `MLAAttention._v_up_proj_and_o_proj(o,
 * heads_first=True)` (patches/atom-optimizations.patch:131-143, called at
 * :297-302 on the decode's heads-first output; tests/test_mla_heads_first_e2e.py:50-59):
 *   x[t, h * 128 + v] = bf16(sum_l o[h, t, l] * w_uv[h, l, v])   (fp32 accumulation)
 *   out[t, :]         = bf16(x[t, :] @ w_o^T)                      (fp32 accumulation)
 * o: bf16 [num_heads, num_tokens, 512] with element strides o_stride_h /
 * o_stride_t (latent dimension contiguous), w_uv bf16 [num_heads, 512, 128]
 * contiguous, w_o bf16 [hidden, num_heads * 128] contiguous (the o_proj
 * Linear weight), x a bf16 [num_tokens, num_heads * 128] contiguous scratch
 * (the BMM result, also readable afterwards), out bf16 [num_tokens, hidden]
 * with row stride out_stride.  num_heads 1..8, hidden a multiple of 64.
 * Two launches on `stream`, the second a programmatic dependent of the first. */
typedef struct KimiVUpOProjParams {
  const void* o;
  int64_t o_stride_h;
  int64_t o_stride_t;
  const void* w_uv;
  const void* w_o;
  void* x;
  void* out;
  int64_t out_stride;
  int32_t num_tokens;
  int32_t num_heads;
  int32_t hidden;
  int32_t* status;             /* optional device word: KIMI_DEVICE_VUP_WAIT when a wait gave up
                                  (each wait keeps a fixed ~2 s bound); NULL = not reported */
} KimiVUpOProjParams;

KIMI_API int kimi_mla_v_up_o_proj(const KimiVUpOProjParams* params, void* stream);

/* Row quantiser: x bf16 [rows, cols] (row stride x_stride elements, cols a
 * multiple of 32) -> nibbles uint8 [rows, cols/2] and scales uint8
 * [rows, cols/32], both contiguous. */
KIMI_API int kimi_mxfp4_quantize(const void* x, int64_t rows, int64_t cols, int64_t x_stride,
                        void* nibbles, void* scales, int32_t legacy_rule, void* stream);

/* Reads a device status word written by the decode kernels (copies 4 bytes
 * to the host after the work queued on `stream` so far, so it waits for that
 * work) and returns it: 0 when no bit is set, else the KIMI_DEVICE_* bits (a
 * positive status below KIMI_ERR_CUDA_BASE), or a CUDA error status.  When
 * `clear` is non-zero the word is reset to 0 afterwards. */
KIMI_API int kimi_device_status(int32_t* device_word, int32_t clear, void* stream);

/* Human-readable text for a status code (static storage). */
KIMI_API const char* kimi_status_string(int status);

/* ABI version of this header (major * 100 + minor). */
KIMI_API int kimi_abi_version(void);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* KIMI_MLA_H_ */
