"""CPU checks of the decode-prologue oracle (oracle/q_absorb.py): the RoPE
restatement against a float64 complex rotation in both pairings, the W_UK
absorption against a per-head loop, and the cache it writes against the
plain append of the rotated k_pe."""
import numpy as np

from oracle import mla as omla
from oracle import mxfp4 as omx
from oracle import q_absorb as oqa
from tests.cases import bf16_randn


def _tables(max_position=64):
    freqs = 1.0 / (10000.0 ** (np.arange(32) / 32.0))
    ang = np.arange(max_position)[:, None] * freqs[None, :]
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def test_rope_is_a_rotation_of_each_pair():
    rng = np.random.default_rng(1)
    cos, sin = _tables()
    x = bf16_randn(rng, (16, 3, 64))
    pos = rng.integers(0, 64, 16)
    xf = omx.bf16_bits_to_f32(x).astype(np.float64)
    for neox in (False, True):
        ia, ib = oqa.rope_pairs(neox)
        z = (xf[..., ia] + 1j * xf[..., ib]) * np.exp(1j * np.arctan2(sin[pos], cos[pos]).astype(np.float64))[:, None, :]
        got = omx.bf16_bits_to_f32(oqa.rope_bf16(x, pos, cos, sin, neox)).astype(np.float64)
        np.testing.assert_allclose(got[..., ia], z.real, rtol=1e-2, atol=2e-2)
        np.testing.assert_allclose(got[..., ib], z.imag, rtol=1e-2, atol=2e-2)
    # the two pairings differ (they rotate different element pairs)
    assert not np.array_equal(oqa.rope_bf16(x, pos, cos, sin, True), oqa.rope_bf16(x, pos, cos, sin, False))
    # position 0 is the identity
    z0 = np.zeros(16, np.int64)
    np.testing.assert_array_equal(oqa.rope_bf16(x, z0, cos, sin, True), x)


def test_absorb_matches_per_head_products():
    rng = np.random.default_rng(2)
    q = bf16_randn(rng, (5, 3, 128))
    w = bf16_randn(rng, (3, 128, 512), scale=0.1)
    got = oqa.q_absorb(q, w)
    qf, wf = omx.bf16_bits_to_f32(q).astype(np.float64), omx.bf16_bits_to_f32(w).astype(np.float64)
    for h in range(3):
        np.testing.assert_allclose(got[:, h], (qf[:, h] @ wf[h]).astype(np.float32), rtol=1e-6, atol=1e-5)


def test_cache_gets_rotated_k_pe():
    rng = np.random.default_rng(3)
    cos, sin = _tables()
    T = 10
    kv_c, k_pe = bf16_randn(rng, (T, 512)), bf16_randn(rng, (T, 64))
    pos, slots = rng.integers(0, 64, T), rng.permutation(128)[:T]
    kvb, kvs = omla.empty_cache(2)
    _, _, kvb, kvs = oqa.absorb_rope_append(bf16_randn(rng, (T, 2, 128)), bf16_randn(rng, (T, 2, 64)),
                                            bf16_randn(rng, (2, 128, 512)), kv_c, k_pe, pos, cos, sin, kvb, kvs,
                                            slots, is_neox=False)
    ref_b, ref_s = omla.empty_cache(2)
    ref_b, ref_s = omla.kv_append(ref_b, ref_s, kv_c, oqa.rope_bf16(k_pe, pos, cos, sin, False), slots)
    np.testing.assert_array_equal(kvb, ref_b)
    np.testing.assert_array_equal(kvs, ref_s)
    rot = kvb.reshape(-1, omla.TOKEN_BYTES)[slots, omla.NIBBLE_BYTES:].view(np.uint16)
    assert not np.array_equal(rot, k_pe)  # rotated, not copied
