"""Paged absorbed-MLA decode over the MXFP4 latent cache, in float32 numpy.

TEST INFRASTRUCTURE ONLY (the oracle): imported by tests, smoke() and the
bench CPU baseline, never by the product package.

Restates the reference's torch path, composed for this project's cache
layout (512-dim MXFP4 latent + 64-dim bf16 RoPE part):

1. dequantise the latent (``_dequant_mxfp4_torch``,
   archive/mla-mxfp4-dead-end/mla_decode_mxfp4_v5.py:381-400) and append the
   bf16 RoPE part -> a float32 ``[T, 576]`` cache;
2. gather each sequence's tokens through the page table and run
   ``reference_mla_decode`` (tests/test_triton_mla_decode.py:12-62):
   ``scores = (q_nope @ k_nope.T + q_pe @ k_pe.T) * sm_scale``,
   ``softmax``, ``o = attn @ v`` with ``v = k_nope``; an empty sequence
   leaves its output row at zero (:34-35).

The split-K pieces restate the stage-1 epilogue and the stage-2 merge of the
archive kernel (v5.py:249-261 and v5.py:264-306) in the natural-exp form
(the archive's kernels used ``exp2`` on scores that were never multiplied by
log2(e); the merge below is the mathematically intended one).
"""
from __future__ import annotations

import numpy as np

from . import mxfp4

KV_LORA_RANK = 512
ROPE_DIM = 64
QK_DIM = KV_LORA_RANK + ROPE_DIM
PAGE_SIZE = 64
NIBBLE_BYTES = KV_LORA_RANK // 2          # 256
ROPE_BYTES = ROPE_DIM * 2                 # 128
TOKEN_BYTES = NIBBLE_BYTES + ROPE_BYTES   # 384 bytes per token in kv_buffer
SCALE_BYTES = KV_LORA_RANK // mxfp4.GROUP  # 16 e8m0 bytes per token in kv_scales


# --------------------------------------------------------------------------
# Cache packing (this project's layout; the reference's own MXFP4 layout is
# [T, 288] nibbles + [T, 18] scales for an all-576 latent, v5.py:406-407)
# --------------------------------------------------------------------------
def empty_cache(num_pages: int, page_size: int = PAGE_SIZE):
    kv_buffer = np.zeros((num_pages, page_size, TOKEN_BYTES), dtype=np.uint8)
    kv_scales = np.zeros((num_pages, page_size, SCALE_BYTES), dtype=np.uint8)
    return kv_buffer, kv_scales


def kv_append(kv_buffer, kv_scales, kv_c_bits, k_pe_bits, slot_mapping, legacy_rule=False):
    """Quantise ``kv_c`` (bf16 bits [n, 512]) and store it with ``k_pe``
    (bf16 bits [n, 64]) at flat slots ``slot_mapping`` (page * page_size + row).

    Negative slots are skipped (the padding convention of the reference's
    cache writers, patches/atom-optimizations.patch:615-634 pass
    ``slot_mapping`` through unchanged).  Returns the updated arrays.
    """
    kv_c_bits = np.asarray(kv_c_bits, dtype=np.uint16)
    k_pe_bits = np.asarray(k_pe_bits, dtype=np.uint16)
    quant = mxfp4.quantize_legacy if legacy_rule else mxfp4.quantize_inline
    nib, sc = quant(kv_c_bits)
    page_size = kv_buffer.shape[1]
    flat_buf = kv_buffer.reshape(-1, TOKEN_BYTES)
    flat_sc = kv_scales.reshape(-1, SCALE_BYTES)
    rope_bytes = np.ascontiguousarray(k_pe_bits).view(np.uint8).reshape(-1, ROPE_BYTES)
    for i, slot in enumerate(np.asarray(slot_mapping, dtype=np.int64)):
        if slot < 0:
            continue
        flat_buf[slot, :NIBBLE_BYTES] = nib[i]
        flat_buf[slot, NIBBLE_BYTES:] = rope_bytes[i]
        flat_sc[slot] = sc[i]
    del page_size
    return kv_buffer, kv_scales


def dequantize_cache(kv_buffer, kv_scales) -> np.ndarray:
    """Whole paged cache -> float32 [num_pages * page_size, 576]."""
    flat_buf = np.asarray(kv_buffer, dtype=np.uint8).reshape(-1, TOKEN_BYTES)
    flat_sc = np.asarray(kv_scales, dtype=np.uint8).reshape(-1, SCALE_BYTES)
    latent = mxfp4.dequantize(flat_buf[:, :NIBBLE_BYTES], flat_sc, KV_LORA_RANK)
    rope_bits = np.ascontiguousarray(flat_buf[:, NIBBLE_BYTES:]).view(np.uint16)
    rope = mxfp4.bf16_bits_to_f32(rope_bits)
    return np.concatenate([latent, rope], axis=1)


def token_rows(kv_indptr, kv_indices, kv_last_page_len, page_size: int = PAGE_SIZE):
    """Per-sequence flat token ids from the page table (scripts/submission.py:101-106:
    pages ``kv_indices[kv_indptr[b]:kv_indptr[b+1]]``, the last page holding
    ``kv_last_page_len[b]`` tokens)."""
    kv_indptr = np.asarray(kv_indptr, dtype=np.int64)
    kv_indices = np.asarray(kv_indices, dtype=np.int64)
    last = np.asarray(kv_last_page_len, dtype=np.int64)
    rows = []
    for b in range(len(kv_indptr) - 1):
        pages = kv_indices[kv_indptr[b]:kv_indptr[b + 1]]
        if len(pages) == 0:
            rows.append(np.zeros(0, dtype=np.int64))
            continue
        r = (pages[:, None] * page_size + np.arange(page_size)[None, :]).reshape(-1)
        n_tok = (len(pages) - 1) * page_size + int(last[b])
        rows.append(r[:n_tok])
    return rows


# --------------------------------------------------------------------------
# Decode
# --------------------------------------------------------------------------
def reference_mla_decode(q: np.ndarray, kv_cache: np.ndarray, kv_indptr, kv_indices,
                         kv_lora_rank: int, sm_scale: float) -> np.ndarray:
    """tests/test_triton_mla_decode.py:12-62 in numpy float32.

    ``q`` float32 [B, H, 576]; ``kv_cache`` float32 [T, 576];
    ``kv_indptr`` / ``kv_indices`` index tokens.  Returns float32 [B, H, 512].
    """
    b_sz, h, _ = q.shape
    o = np.zeros((b_sz, h, kv_lora_rank), dtype=np.float32)
    for b in range(b_sz):
        start, end = int(kv_indptr[b]), int(kv_indptr[b + 1])
        if end == start:
            continue
        kv = kv_cache[np.asarray(kv_indices[start:end], dtype=np.int64)]
        q_nope = q[b, :, :kv_lora_rank].astype(np.float32)
        q_pe = q[b, :, kv_lora_rank:].astype(np.float32)
        k_nope = kv[:, :kv_lora_rank]
        k_pe = kv[:, kv_lora_rank:]
        scores = (q_nope @ k_nope.T + q_pe @ k_pe.T) * np.float32(sm_scale)
        scores = scores - scores.max(axis=-1, keepdims=True)
        p = np.exp(scores)
        p /= p.sum(axis=-1, keepdims=True)
        o[b] = p @ k_nope
    return o


def mla_decode(q_bits, kv_buffer, kv_scales, kv_indptr, kv_indices, kv_last_page_len,
               sm_scale: float, page_size: int = PAGE_SIZE) -> np.ndarray:
    """Paged MXFP4 decode: ``q_bits`` bf16 bits [B, H, 576] -> float32 [B, H, 512]."""
    q = mxfp4.bf16_bits_to_f32(q_bits)
    rows = token_rows(kv_indptr, kv_indices, kv_last_page_len, page_size)
    # Dequantise only the touched tokens (same values as dequantising the whole cache).
    all_rows = np.concatenate(rows) if rows else np.zeros(0, dtype=np.int64)
    flat_buf = np.asarray(kv_buffer, dtype=np.uint8).reshape(-1, TOKEN_BYTES)
    flat_sc = np.asarray(kv_scales, dtype=np.uint8).reshape(-1, SCALE_BYTES)
    sub_cache = dequantize_cache(flat_buf[all_rows], flat_sc[all_rows])
    tok_indptr = np.zeros(len(rows) + 1, dtype=np.int64)
    tok_indptr[1:] = np.cumsum([len(r) for r in rows])
    tok_indices = np.arange(len(all_rows), dtype=np.int64)
    return reference_mla_decode(q, sub_cache, tok_indptr, tok_indices, KV_LORA_RANK, sm_scale)


# --------------------------------------------------------------------------
# Split-K pieces (stage-1 epilogue and stage-2 merge)
# --------------------------------------------------------------------------
def split_partials(q: np.ndarray, kv: np.ndarray, bounds, sm_scale: float):
    """One sequence: float32 q [H, 576], kv [T, 576] and split token bounds
    [(s0, e0), ...] -> (partial_o [S, H, 512], lse [S, H]) with ``partial_o``
    normalised per split and ``lse`` the natural log-sum-exp of the split's
    scaled scores (v5.py:249-261).  An empty split has lse = -inf, o = 0."""
    h = q.shape[0]
    n_s = len(bounds)
    po = np.zeros((n_s, h, KV_LORA_RANK), dtype=np.float32)
    lse = np.full((n_s, h), -np.inf, dtype=np.float32)
    for s, (a, b) in enumerate(bounds):
        if b <= a:
            continue
        k = kv[a:b]
        sc = (q[:, :KV_LORA_RANK] @ k[:, :KV_LORA_RANK].T
              + q[:, KV_LORA_RANK:] @ k[:, KV_LORA_RANK:].T) * np.float32(sm_scale)
        m = sc.max(axis=-1, keepdims=True)
        p = np.exp(sc - m)
        l = p.sum(axis=-1, keepdims=True)
        po[s] = (p @ k[:, :KV_LORA_RANK]) / l
        lse[s] = (m + np.log(l))[:, 0]
    return po, lse


def lse_merge(partial_o: np.ndarray, lse: np.ndarray) -> np.ndarray:
    """Merge split partials (v5.py:264-306): weights ``exp(lse_s - max_s lse)``,
    normalised weighted sum.  partial_o [S, H, L], lse [S, H] -> [H, L].
    All-empty heads (every lse = -inf) give zeros."""
    m = lse.max(axis=0)
    safe_m = np.where(np.isfinite(m), m, 0.0).astype(np.float32)
    w = np.where(np.isfinite(lse), np.exp(lse - safe_m[None, :]), 0.0).astype(np.float32)
    tot = w.sum(axis=0)
    acc = (w[:, :, None] * partial_o).sum(axis=0)
    out = np.where(tot[:, None] > 0, acc / np.where(tot > 0, tot, 1.0)[:, None], 0.0)
    return out.astype(np.float32)
