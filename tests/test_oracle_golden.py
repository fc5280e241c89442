"""Pin the CPU oracle against the golden vectors produced by the reference's
own code (tests/golden/make_golden.py).  CPU only."""
import os

import numpy as np
import pytest

from oracle import mla, mxfp4


def _load(golden_dir, name):
    return np.load(os.path.join(golden_dir, name))


def test_inline_quantiser_matches_reference_triton_rule(golden_dir):
    g = _load(golden_dir, "quant_golden.npz")
    nib, sc = mxfp4.quantize_inline(g["x_bits"])
    assert np.array_equal(sc, g["inline_scales"])
    assert np.array_equal(nib, g["inline_nibbles"])
    # every e2m1 magnitude code is exercised by the fixture
    assert set(np.unique(g["inline_nibbles"] & 7).tolist()) == set(range(8))


def test_legacy_quantiser_matches_reference_torch_rule(golden_dir):
    g = _load(golden_dir, "quant_golden.npz")
    nib, sc = mxfp4.quantize_legacy(g["x_bits"])
    assert np.array_equal(sc, g["legacy_scales"])
    assert np.array_equal(nib, g["legacy_nibbles"])


def test_dequant_matches_reference(golden_dir):
    g = _load(golden_dir, "dequant_golden.npz")
    vals = mxfp4.dequantize(g["nibbles"], g["scales"], 512)
    assert np.array_equal(vals, g["values"], equal_nan=True)


def test_e2m1_table_known_answers():
    # nibble codes 0..15 at scale byte 127 (2**0): the e2m1 table with sign bit 3
    nib = np.array([[c | (c + 1) << 4 for c in range(0, 16, 2)] * 2], dtype=np.uint8)
    sc = np.full((1, 1), 127, dtype=np.uint8)
    vals = mxfp4.dequantize(nib[:, :16], sc, 32)[0, :16]
    expect = [0, .5, 1, 1.5, 2, 3, 4, 6, -0., -.5, -1, -1.5, -2, -3, -4, -6]
    assert np.array_equal(vals, np.array(expect, np.float32))
    # e8m0 decode 2**(s - 127)
    for s in (0, 1, 126, 127, 128, 254):
        v = mxfp4.dequantize(np.array([[0x02] + [0] * 15], np.uint8), np.array([[s]], np.uint8), 32)[0, 0]
        assert v == np.ldexp(np.float32(1.0), s - 127)


def test_inline_rounding_ties_are_even():
    # amax 4 -> rounded amax 4 -> e = 0, values are used as-is
    x = np.array([[4.0, 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0] + [0.0] * 24], np.float32)
    nib, sc = mxfp4.quantize_inline(x)
    assert sc[0, 0] == 127
    codes = [(b >> s) & 0xF for b in nib[0, :4] for s in (0, 4)]
    #          4.0 0.25->0 0.75->1 1.25->1 1.75->2 2.5->2 3.5->4 5->4
    assert codes == [6, 0, 2, 2, 4, 4, 6, 6]


@pytest.mark.parametrize("case", ["plumbing", "ragged", "tails"])
def test_paged_decode_matches_reference(golden_dir, case):
    g = _load(golden_dir, "decode_golden.npz")
    k = lambda n: g[f"{case}__{n}"]  # noqa: E731
    out = mla.mla_decode(k("q_bits"), k("kv_buffer"), k("kv_scales"), k("kv_indptr"),
                         k("kv_indices"), k("kv_last_page_len"), float(k("sm_scale")))
    ref = k("out")
    assert out.shape == ref.shape
    assert np.abs(out - ref).max() <= 1e-5 * max(1.0, np.abs(ref).max())


def test_split_merge_equals_full_softmax():
    rng = np.random.default_rng(3)
    q = rng.standard_normal((8, 576)).astype(np.float32)
    kv = rng.standard_normal((300, 576)).astype(np.float32)
    bounds = [(0, 0), (0, 97), (97, 200), (200, 300), (300, 300)]
    po, lse = mla.split_partials(q, kv, bounds, 0.07)
    merged = mla.lse_merge(po, lse)
    full = mla.reference_mla_decode(q[None], kv, [0, 300], np.arange(300), 512, 0.07)[0]
    assert np.abs(merged - full).max() < 1e-5


def test_kv_append_reproduces_golden_cache_bytes(golden_dir):
    """Appending the fixture's tokens through the oracle's cache writer must give
    the cache bytes that the reference's Triton quantiser produced."""
    g = _load(golden_dir, "quant_golden.npz")
    x = g["x_bits"][:64]
    rng = np.random.default_rng(0)
    k_pe = rng.integers(0, 1 << 16, size=(64, 64), dtype=np.uint16)
    buf, sc = mla.empty_cache(2)
    slots = rng.permutation(128)[:64]
    mla.kv_append(buf, sc, x, k_pe, slots)
    flat_b = buf.reshape(-1, 384)
    flat_s = sc.reshape(-1, 16)
    assert np.array_equal(flat_b[slots, :256], g["inline_nibbles"][:64])
    assert np.array_equal(flat_s[slots], g["inline_scales"][:64])
    assert np.array_equal(flat_b[slots, 256:].view(np.uint16), k_pe)
