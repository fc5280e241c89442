"""The decode step before attention: q absorption by W_UK, RoPE, KV append.

TEST INFRASTRUCTURE ONLY (the oracle): imported by tests, never by the
product package.

Restates what the reference's decode prologue computes in
``MLAAttention._forward_decode`` / ``fused_kv_bmm``
(patches/atom-optimizations.patch:468-639, the fused
``fused_fp4_bmm_rope_cat_and_cache_mla`` and the unfused
``_q_proj_and_k_up_proj`` + ``fused_qk_rope_concat_and_cache_mla`` path it
replaces):

* ``q_out[t, h, :512] = q_nope[t, h, :] @ W_UK[h]`` (the k_up_proj BMM that
  absorbs W_UK into q; ``q_nope`` is transposed to heads-major for it,
  patch:306);
* ``q_out[t, h, 512:] = rope(q_pe[t, h, :], positions[t])``;
* the cache gets ``kv_c[t]`` quantised to MXFP4 and ``rope(k_pe[t],
  positions[t])`` at ``slot_mapping[t]`` (``is_nope_first=True``: latent
  first, RoPE part second, patch:632).

The rotary embedding is the one the serving engine passes in
(``self.rotary_emb.cos_cache / sin_cache``, ``is_neox_style``; the source of
that class is a third-party dependency not present in the reference tree).
Its published convention, restated here: with ``c = cos[pos, i]`` and
``s = sin[pos, i]`` for the i-th of the 32 frequency pairs,
``(a, b) -> (a c - b s, b c + a s)``, where the pair is ``(x[i], x[i + 32])``
in the neox style and ``(x[2 i], x[2 i + 1])`` otherwise.  Every product and
sum is rounded to float32 on its own (no fused multiply-add), and the result
to bf16 once.
"""
from __future__ import annotations

import numpy as np

from . import mla, mxfp4

NOPE_DIM = 128  # qk_nope_head_dim of the Kimi-K2 / DeepSeek-V3 attention


def rope_pairs(is_neox: bool):
    """Index arrays (first, second) of the 32 rotated pairs of a 64-dim row."""
    i = np.arange(32)
    return (i, i + 32) if is_neox else (2 * i, 2 * i + 1)


def rope_bf16(x_bits: np.ndarray, positions: np.ndarray, cos: np.ndarray, sin: np.ndarray,
              is_neox: bool) -> np.ndarray:
    """bf16 bits [..., 64] rotated at ``positions`` (broadcast over the
    leading dims of x after the first) -> bf16 bits of the same shape."""
    x = mxfp4.bf16_bits_to_f32(x_bits)
    c = np.asarray(cos, np.float32)[positions]  # [T, 32]
    s = np.asarray(sin, np.float32)[positions]
    extra = x.ndim - 2
    c = c.reshape(c.shape[:1] + (1,) * extra + c.shape[1:])
    s = s.reshape(s.shape[:1] + (1,) * extra + s.shape[1:])
    ia, ib = rope_pairs(is_neox)
    a, b = x[..., ia], x[..., ib]
    out = np.empty_like(x)
    out[..., ia] = (a * c).astype(np.float32) - (b * s).astype(np.float32)
    out[..., ib] = (b * c).astype(np.float32) + (a * s).astype(np.float32)
    return mxfp4.f32_to_bf16_bits(out.astype(np.float32))


def q_absorb(q_nope_bits: np.ndarray, w_uk_bits: np.ndarray) -> np.ndarray:
    """q_nope bf16 bits [T, H, 128] x W_UK bf16 bits [H, 128, 512] -> float32
    [T, H, 512] (exact products, float64 sums)."""
    q = mxfp4.bf16_bits_to_f32(q_nope_bits).astype(np.float64)
    w = mxfp4.bf16_bits_to_f32(w_uk_bits).astype(np.float64)
    return np.einsum("thk,hkn->thn", q, w).astype(np.float32)


def absorb_rope_append(q_nope_bits, q_pe_bits, w_uk_bits, kv_c_bits, k_pe_bits, positions, cos, sin,
                       kv_buffer, kv_scales, slot_mapping, is_neox: bool, legacy_rule: bool = False):
    """The whole step.  Returns (q_absorbed float32 [T, H, 512], q_pe_rot bf16
    bits [T, H, 64], kv_buffer, kv_scales) with the cache arrays updated."""
    positions = np.asarray(positions, np.int64)
    q_abs = q_absorb(q_nope_bits, w_uk_bits)
    q_rot = rope_bf16(q_pe_bits, positions, cos, sin, is_neox)
    k_rot = rope_bf16(k_pe_bits, positions, cos, sin, is_neox)
    kv_buffer, kv_scales = mla.kv_append(kv_buffer, kv_scales, kv_c_bits, k_rot, slot_mapping, legacy_rule)
    return q_abs, q_rot, kv_buffer, kv_scales
