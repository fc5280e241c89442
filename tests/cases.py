"""Seeded decode cases for the tests: inputs built on the CPU with the oracle's
quantiser, so every GPU result is compared against numbers that never went
through the code under test."""
from __future__ import annotations

import math

import numpy as np

from oracle import mla as omla
from oracle import mxfp4 as omx

PAGE = omla.PAGE_SIZE


def bf16_randn(rng: np.random.Generator, shape, scale: float = 1.0) -> np.ndarray:
    return omx.f32_to_bf16_bits(rng.standard_normal(shape, dtype=np.float32) * np.float32(scale))


def page_table(seq_lens, rng: np.random.Generator, shuffle: bool = True, spare_pages: int = 1):
    n_pages = [math.ceil(l / PAGE) for l in seq_lens]
    total = sum(n_pages) + spare_pages
    perm = rng.permutation(total) if shuffle else np.arange(total)
    indptr = np.zeros(len(seq_lens) + 1, np.int32)
    indptr[1:] = np.cumsum(n_pages)
    indices = perm[:indptr[-1]].astype(np.int32)
    last = np.array([l - (n - 1) * PAGE if n else 0 for l, n in zip(seq_lens, n_pages)], np.int32)
    return total, indptr, indices, last


def make_case(seq_lens, heads: int, seed: int, shuffle: bool = True, sm_scale: float | None = None,
              kv_scale: float = 1.0, legacy_rule: bool = False) -> dict:
    rng = np.random.default_rng(seed)
    total_pages, indptr, indices, last = page_table(seq_lens, rng, shuffle)
    q_bits = bf16_randn(rng, (len(seq_lens), heads, omla.QK_DIM))
    kv_c = bf16_randn(rng, (total_pages * PAGE, omla.KV_LORA_RANK), kv_scale)
    k_pe = bf16_randn(rng, (total_pages * PAGE, omla.ROPE_DIM))
    kv_buffer, kv_scales = omla.empty_cache(total_pages)
    omla.kv_append(kv_buffer, kv_scales, kv_c, k_pe, np.arange(total_pages * PAGE), legacy_rule=legacy_rule)
    return dict(q_bits=q_bits, kv_buffer=kv_buffer, kv_scales=kv_scales, kv_indptr=indptr,
                kv_indices=indices, kv_last_page_len=last,
                sm_scale=(1.0 / math.sqrt(192.0)) if sm_scale is None else sm_scale,
                seq_lens=list(seq_lens), heads=heads)


def oracle_out(case: dict) -> np.ndarray:
    return omla.mla_decode(case["q_bits"], case["kv_buffer"], case["kv_scales"], case["kv_indptr"],
                           case["kv_indices"], case["kv_last_page_len"], case["sm_scale"])


def compare(out: np.ndarray, ref: np.ndarray):
    """(cosine similarity, max abs error) of a bf16 result against the fp32 oracle."""
    a = out.astype(np.float64).reshape(-1)
    b = ref.astype(np.float64).reshape(-1)
    denom = np.linalg.norm(a) * np.linalg.norm(b)
    cos = 1.0 if denom == 0 and np.abs(a - b).max(initial=0) == 0 else float(a @ b / max(denom, 1e-300))
    return cos, float(np.abs(a - b).max(initial=0.0))


# Acceptance thresholds for the decode output (bf16 against the fp32 reference path).
COS_MIN = 0.9995
MAX_ABS = 2e-2
