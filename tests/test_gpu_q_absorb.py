"""GPU parity of the fused decode prologue (q absorption by W_UK, RoPE, MXFP4
KV append) through the C ABI, against the CPU oracle.

Bars: the cache bytes (nibbles, e8m0 scales, rotated RoPE part) and the
rotated q_pe in q_out bit-exact (the same float32 operations in the same
order, one rounding to bf16); the absorbed q in bf16 within cosine >= 0.99999
and max-abs <= 1e-2 x max|ref| of the float64-summed product."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

import kimi_b200  # noqa: E402
from oracle import mla as omla  # noqa: E402
from oracle import q_absorb as oqa  # noqa: E402
from tests.cases import bf16_randn, compare  # noqa: E402

DEV = "cuda:0"


def _bf16(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(DEV)


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.cpu().view(torch.int16).numpy().view(np.uint16)


def _case(T, H, pages, seed, max_position=4096):
    rng = np.random.default_rng(seed)
    q = bf16_randn(rng, (T, H, 192))
    w_uk = bf16_randn(rng, (H, 128, 512), scale=1.0 / np.sqrt(128.0))
    kv_c = bf16_randn(rng, (T, 512))
    k_pe = bf16_randn(rng, (T, 64))
    positions = rng.integers(0, max_position, T).astype(np.int64)
    freqs = 1.0 / (10000.0 ** (np.arange(32) / 32.0))
    ang = np.arange(max_position)[:, None] * freqs[None, :]
    cos, sin = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    slots = rng.permutation(pages * omla.PAGE_SIZE)[:T].astype(np.int64)
    return dict(q=q, w_uk=w_uk, kv_c=kv_c, k_pe=k_pe, positions=positions, cos=cos, sin=sin, slots=slots,
                pages=pages)


def _run(c, is_neox, legacy=False):
    q = _bf16(c["q"])
    kvb = torch.zeros(c["pages"], 64, omla.TOKEN_BYTES, dtype=torch.uint8, device=DEV)
    kvs = torch.zeros(c["pages"], 64, omla.SCALE_BYTES, dtype=torch.uint8, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    q_out = kimi_b200.q_absorb_rope_append(
        q[:, :, :128], q[:, :, 128:], _bf16(c["w_uk"]), _bf16(c["kv_c"]), _bf16(c["k_pe"]),
        torch.from_numpy(c["positions"]).to(DEV), torch.from_numpy(c["cos"]).to(DEV),
        torch.from_numpy(c["sin"]).to(DEV), kvb, kvs, torch.from_numpy(c["slots"]).to(DEV), is_neox=is_neox,
        legacy_rule=legacy, status=status)
    torch.cuda.synchronize()
    assert kimi_b200.device_status(status) == 0  # no wait gave up
    return q_out, kvb.cpu().numpy(), kvs.cpu().numpy()


def _oracle(c, is_neox, legacy=False):
    kvb, kvs = omla.empty_cache(c["pages"])
    return oqa.absorb_rope_append(c["q"][:, :, :128], c["q"][:, :, 128:], c["w_uk"], c["kv_c"], c["k_pe"],
                                  c["positions"], c["cos"], c["sin"], kvb, kvs, c["slots"], is_neox, legacy)


def _check(c, is_neox, legacy=False):
    q_out, kvb, kvs = _run(c, is_neox, legacy)
    q_abs, q_rot, kvb_ref, kvs_ref = _oracle(c, is_neox, legacy)
    got = q_out[:, :, :512].float().cpu().numpy()
    cos, err = compare(got, q_abs)
    assert cos >= 0.99999 and err <= 1e-2 * max(1.0, float(np.abs(q_abs).max())), (cos, err)
    np.testing.assert_array_equal(_bits(q_out[:, :, 512:].contiguous()), q_rot)
    np.testing.assert_array_equal(kvb, kvb_ref)
    np.testing.assert_array_equal(kvs, kvs_ref)


@pytest.mark.parametrize("is_neox", [False, True])
def test_tp8_shape_matches_oracle(is_neox):
    # Kimi-K2 TP8: 8 heads per GPU, a decode batch of 128 tokens (one tile)
    _check(_case(128, 8, pages=4, seed=50), is_neox)


def test_ragged_tiles_many_heads_legacy_rule():
    # two tiles (the second partly filled), 16 heads, the legacy quantiser rule
    _check(_case(200, 16, pages=8, seed=51), is_neox=True, legacy=True)


def test_skipped_slots_and_out_of_range_positions():
    c = _case(40, 4, pages=2, seed=52)
    c["slots"][[3, 17]] = -1                    # padding tokens: no cache write
    c["positions"][[5, 30]] = [4096, -2]        # outside the rotary table
    q_out, kvb, kvs = _run(c, False)
    ok = np.ones(40, bool)
    ok[[5, 30]] = False
    keep = ok & (c["slots"] >= 0)
    # cache: only tokens with a valid slot and position are written
    kvb_ref, kvs_ref = omla.empty_cache(2)
    k_rot = oqa.rope_bf16(c["k_pe"][keep], c["positions"][keep], c["cos"], c["sin"], False)
    kvb_ref, kvs_ref = omla.kv_append(kvb_ref, kvs_ref, c["kv_c"][keep], k_rot, c["slots"][keep])
    np.testing.assert_array_equal(kvb, kvb_ref)
    np.testing.assert_array_equal(kvs, kvs_ref)
    # q_out: valid positions rotated, invalid ones zeroed
    q_rot = oqa.rope_bf16(c["q"][ok, :, 128:], c["positions"][ok], c["cos"], c["sin"], False)
    rot = _bits(q_out[:, :, 512:].contiguous())
    np.testing.assert_array_equal(rot[ok], q_rot)
    assert not rot[~ok].any()


def test_rejects_bad_arguments():
    c = _case(8, 2, pages=1, seed=53)
    q = _bf16(c["q"])
    kvb = torch.zeros(1, 64, omla.TOKEN_BYTES, dtype=torch.uint8, device=DEV)
    kvs = torch.zeros(1, 64, omla.SCALE_BYTES, dtype=torch.uint8, device=DEV)
    with pytest.raises(ValueError):
        kimi_b200.q_absorb_rope_append(q[:, :, :128], q[:, :, 128:], _bf16(c["w_uk"])[:1], _bf16(c["kv_c"]),
                                       _bf16(c["k_pe"]), torch.from_numpy(c["positions"]).to(DEV),
                                       torch.from_numpy(c["cos"]).to(DEV), torch.from_numpy(c["sin"]).to(DEV),
                                       kvb, kvs, torch.from_numpy(c["slots"]).to(DEV))
