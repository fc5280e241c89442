"""The V up-projection + o_proj oracle against the golden fixture made by
running the reference's own ``forward_heads_first`` / ``forward_standard``
(tests/test_mla_heads_first_e2e.py:39-59) on CPU
(tests/golden/make_vup_golden.py)."""
import os

import numpy as np
import pytest

from oracle import mxfp4 as omx
from oracle import v_up_o_proj as ovu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "vup_golden.npz")
CASES = ["unit_n2_b5_h128", "n4_b4_h64", "n1_b130_h64"]


@pytest.mark.parametrize("name", CASES)
def test_oracle_matches_reference_output(name):
    z = np.load(GOLDEN)
    x_bits, out_bits = ovu.v_up_o_proj(z[f"{name}/o"], z[f"{name}/w_uv"], z[f"{name}/w_o"])
    n, b, _ = z[f"{name}/o"].shape
    assert x_bits.shape == (b, n * 128) and out_bits.shape == z[f"{name}/out_heads_first"].shape
    ref = omx.bf16_bits_to_f32(z[f"{name}/out_heads_first"]).astype(np.float64)
    got = omx.bf16_bits_to_f32(out_bits).astype(np.float64)
    # float32 accumulation orders differ: one bf16 step of x or out, on a few
    # entries (an absolute bound for entries near zero after cancellation)
    np.testing.assert_allclose(got, ref, rtol=2 ** -7, atol=1e-3 * np.abs(ref).max())
    assert (out_bits == z[f"{name}/out_heads_first"]).mean() > 0.99


@pytest.mark.parametrize("name", CASES)
def test_reference_paths_agree(name):
    """The fixture's heads-first and standard outputs are the same bits (the
    reference test's own claim, tests/test_mla_heads_first_e2e.py:62-88)."""
    z = np.load(GOLDEN)
    np.testing.assert_array_equal(z[f"{name}/out_heads_first"], z[f"{name}/out_standard"])
