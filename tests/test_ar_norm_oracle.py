"""CPU checks of the all-reduce + RMSNorm + MXFP4 oracle (oracle/ar_norm.py):
its float32 step order against a float64 restatement of the formula, the new
residual as the bf16 sum, and the quantised output as MXFP4 of the normed rows."""
import numpy as np

from oracle import ar_norm
from oracle import mxfp4 as omx


def _bf16(rng, shape, scale=1.0):
    return omx.f32_to_bf16_bits(rng.standard_normal(shape).astype(np.float32) * np.float32(scale))


def test_oracle_follows_the_formula():
    rng = np.random.default_rng(4)
    rows, hidden = 5, 2080  # 65 groups: the last warp partly idle
    ins = [_bf16(rng, (rows, hidden), 0.5) for _ in range(3)]
    res, w = _bf16(rng, (rows, hidden)), _bf16(rng, (hidden,))
    comb, out, nib, sc = ar_norm.ar_rmsnorm_mxfp4(ins, res, w, 1e-6)
    s64 = sum(omx.bf16_bits_to_f32(x).astype(np.float64) for x in ins) + omx.bf16_bits_to_f32(res)
    c = omx.bf16_bits_to_f32(comb).astype(np.float64)
    np.testing.assert_allclose(c, s64, rtol=2 ** -8, atol=1e-6)
    ref = c / np.sqrt((c * c).mean(-1, keepdims=True) + 1e-6) * omx.bf16_bits_to_f32(w)
    np.testing.assert_allclose(omx.bf16_bits_to_f32(out), ref, rtol=2 ** -7, atol=1e-2)
    n2, s2 = omx.quantize_inline(out)
    np.testing.assert_array_equal(nib, n2)
    np.testing.assert_array_equal(sc, s2)
    assert nib.shape == (rows, hidden // 2) and sc.shape == (rows, hidden // 32)


def test_single_input_is_residual_add_and_norm():
    rng = np.random.default_rng(5)
    x, res, w = _bf16(rng, (2, 7168)), _bf16(rng, (2, 7168)), _bf16(rng, (7168,))
    comb, _, _, _ = ar_norm.ar_rmsnorm_mxfp4([x], res, w, 1e-6)
    want = omx.f32_to_bf16_bits((omx.bf16_bits_to_f32(x) + omx.bf16_bits_to_f32(res)).astype(np.float32))
    np.testing.assert_array_equal(comb, want)


def test_oracle_matches_reference_rmsnorm_lines_golden():
    """rmsnorm_golden.npz holds the output of the reference's own statements
    (tests/test_ar_fusion_correctness.py:128-131, run by
    tests/golden/make_rmsnorm_golden.py on CPU torch): the new residual and
    the normed, weighted rows are bit-exact, for 1 and 4 rows of 7168."""
    import os
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "rmsnorm_golden.npz"))
    for n in ("m1", "m4"):
        comb, out, nib, sc = ar_norm.ar_rmsnorm_mxfp4([g[f"{n}_hidden_states"]], g[f"{n}_residual"],
                                                      g[f"{n}_weight"], float(g["eps"]))
        np.testing.assert_array_equal(comb, g[f"{n}_combined"])
        np.testing.assert_array_equal(out, g[f"{n}_normed_output"])
        n2, s2 = omx.quantize_inline(g[f"{n}_normed_output"])
        np.testing.assert_array_equal(nib, n2)
        np.testing.assert_array_equal(sc, s2)
