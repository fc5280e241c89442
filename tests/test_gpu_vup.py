"""GPU parity of the V up-projection + o_proj (kimi_mla_v_up_o_proj through the
C ABI) against the CPU oracle, the reference's own outputs (golden fixture)
and the reference test's torch formula run on the GPU in fp32.

Tolerances (floating point, fp32 accumulation in another order than the
oracle's): x within one bf16 step (rtol 2^-7) on every entry and bit-equal on
more than 99% of them; out with cosine similarity >= 0.9999 and
|out - oracle| <= 2^-7 |oracle| + 1e-3 max|oracle| on every entry."""
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

import kimi_b200  # noqa: E402
from oracle import mxfp4 as omx  # noqa: E402
from oracle import v_up_o_proj as ovu  # noqa: E402

DEV = "cuda:0"
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "vup_golden.npz")


def _bf16_np(rng, shape, scale=1.0):
    return omx.f32_to_bf16_bits(rng.standard_normal(shape).astype(np.float32) * np.float32(scale))


def _t(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(DEV)


def _bits(t):
    return t.contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def _check_out(got_bits, ref_bits):
    got = omx.bf16_bits_to_f32(got_bits).astype(np.float64)
    ref = omx.bf16_bits_to_f32(ref_bits).astype(np.float64)
    cos = (got * ref).sum() / np.sqrt((got * got).sum() * (ref * ref).sum())
    assert cos >= 0.9999, cos
    np.testing.assert_allclose(got, ref, rtol=2 ** -7, atol=1e-3 * np.abs(ref).max())


def _check_x(got_bits, ref_bits):
    got = omx.bf16_bits_to_f32(got_bits).astype(np.float64)
    ref = omx.bf16_bits_to_f32(ref_bits).astype(np.float64)
    np.testing.assert_allclose(got, ref, rtol=2 ** -7, atol=1e-6 * np.abs(ref).max())
    assert (got_bits == ref_bits).mean() > 0.99


@pytest.mark.parametrize("heads,tokens,hidden,pad_heads,pad_tokens", [
    (8, 128, 7168, 16, 160),  # Kimi-K2 TP8: 8 real heads sliced from 16 padded, one token tile
    (3, 200, 192, 3, 200),    # two token tiles, the second ragged
    (1, 1, 64, 1, 1),         # one token, one head, one output block
    (8, 300, 512, 8, 300),    # three token tiles with the weights resident
])
def test_matches_oracle(heads, tokens, hidden, pad_heads, pad_tokens):
    rng = np.random.default_rng(90 + heads + tokens)
    o_full = _bf16_np(rng, (pad_heads, pad_tokens, 512))
    w_uv, w_o = _bf16_np(rng, (heads, 512, 128), 0.02), _bf16_np(rng, (hidden, heads * 128), 0.02)
    o_np = o_full[:heads, :tokens]
    x_ref, out_ref = ovu.v_up_o_proj(o_np, w_uv, w_o)
    o = _t(o_full)[:heads, :tokens]  # heads-first view: strides (pad_tokens * 512, 512, 1)
    x = torch.empty(tokens, heads * 128, dtype=torch.bfloat16, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = kimi_b200.v_up_proj_and_o_proj(o, _t(w_uv), _t(w_o), x=x, status=status)
    torch.cuda.synchronize()
    assert kimi_b200.device_status(status) == 0  # no wait gave up
    _check_x(_bits(x), x_ref)
    _check_out(_bits(out), out_ref)


@pytest.mark.parametrize("name", ["unit_n2_b5_h128", "n4_b4_h64", "n1_b130_h64"])
def test_matches_reference_outputs(name):
    z = np.load(GOLDEN)
    out = kimi_b200.v_up_proj_and_o_proj(_t(z[f"{name}/o"]), _t(z[f"{name}/w_uv"]), _t(z[f"{name}/w_o"]))
    torch.cuda.synchronize()
    _check_out(_bits(out), z[f"{name}/out_heads_first"])


def test_matches_torch_fp32_formula():
    """The reference test's forward_heads_first (fp32 BMM, bf16 round, bf16
    mm) on the GPU, at the TP8 shape."""
    g = torch.Generator(device=DEV).manual_seed(5)
    o = torch.randn(8, 128, 512, generator=g, device=DEV).to(torch.bfloat16)
    w_uv = (torch.randn(8, 512, 128, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    w_o = (torch.randn(7168, 1024, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    x_ref = torch.bmm(o.float(), w_uv.float()).to(torch.bfloat16).transpose(0, 1).reshape(128, 1024)
    out_ref = (x_ref.float() @ w_o.float().T).to(torch.bfloat16)
    out = kimi_b200.v_up_proj_and_o_proj(o, w_uv, w_o)
    torch.cuda.synchronize()
    _check_out(_bits(out), _bits(out_ref))


def test_strided_out_and_repeat_calls():
    """out as a column slice of a wider buffer (row stride > hidden); the
    columns outside it stay untouched; a second call into the same buffers
    gives the same bits."""
    rng = np.random.default_rng(7)
    o, w_uv, w_o = _bf16_np(rng, (2, 64, 512)), _bf16_np(rng, (2, 512, 128), 0.02), _bf16_np(rng, (128, 256), 0.02)
    _, out_ref = ovu.v_up_o_proj(o, w_uv, w_o)
    full = torch.full((64, 192), 7.0, dtype=torch.bfloat16, device=DEV)
    kimi_b200.v_up_proj_and_o_proj(_t(o), _t(w_uv), _t(w_o), out=full[:, :128])
    first = _bits(full[:, :128])
    kimi_b200.v_up_proj_and_o_proj(_t(o), _t(w_uv), _t(w_o), out=full[:, :128])
    torch.cuda.synchronize()
    _check_out(_bits(full[:, :128]), out_ref)
    np.testing.assert_array_equal(_bits(full[:, :128]), first)
    assert bool((full[:, 128:] == 7.0).all())


def test_empty_and_bad_arguments():
    w_uv = torch.zeros(2, 512, 128, dtype=torch.bfloat16, device=DEV)
    w_o = torch.zeros(128, 256, dtype=torch.bfloat16, device=DEV)
    empty = kimi_b200.v_up_proj_and_o_proj(torch.zeros(2, 0, 512, dtype=torch.bfloat16, device=DEV), w_uv, w_o)
    assert empty.shape == (0, 128)
    o = torch.zeros(2, 4, 512, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(ValueError):  # hidden not a multiple of 64
        kimi_b200.v_up_proj_and_o_proj(o, w_uv, torch.zeros(96, 256, dtype=torch.bfloat16, device=DEV))
    with pytest.raises(ValueError):  # more than 8 heads
        kimi_b200.v_up_proj_and_o_proj(torch.zeros(9, 4, 512, dtype=torch.bfloat16, device=DEV),
                                       torch.zeros(9, 512, 128, dtype=torch.bfloat16, device=DEV),
                                       torch.zeros(128, 9 * 128, dtype=torch.bfloat16, device=DEV))
    with pytest.raises(ValueError):  # w_uv of the wrong head count
        kimi_b200.v_up_proj_and_o_proj(o, w_uv[:1], w_o)
    with pytest.raises(ValueError):  # misaligned o (token stride not a multiple of 8 elements)
        base = torch.zeros(2 * 4 * 516, dtype=torch.bfloat16, device=DEV)
        kimi_b200.v_up_proj_and_o_proj(base.as_strided((2, 4, 512), (4 * 516, 516, 1)), w_uv, w_o)


def test_token_major_o_view():
    """o given as the transposed view of a token-major [T, H, 512] tensor (the
    reference's standard path layout, tests/test_mla_heads_first_e2e.py:39-48):
    head stride 512, token stride H * 512."""
    rng = np.random.default_rng(23)
    H, T, hidden = 8, 100, 256
    o_std = _bf16_np(rng, (T, H, 512))
    w_uv, w_o = _bf16_np(rng, (H, 512, 128), 0.02), _bf16_np(rng, (hidden, H * 128), 0.02)
    x_ref, out_ref = ovu.v_up_o_proj(o_std.transpose(1, 0, 2), w_uv, w_o)
    x = torch.empty(T, H * 128, dtype=torch.bfloat16, device=DEV)
    out = kimi_b200.v_up_proj_and_o_proj(_t(o_std).transpose(0, 1), _t(w_uv), _t(w_o), x=x)
    torch.cuda.synchronize()
    _check_x(_bits(x), x_ref)
    _check_out(_bits(out), out_ref)
