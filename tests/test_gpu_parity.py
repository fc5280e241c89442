"""GPU parity: the CUDA kernels (through the C ABI) against the CPU oracle and
the golden vectors from the reference.

Bars: cache bytes (nibbles, e8m0 scales, RoPE) bit-exact; decode output in
bf16 within cosine >= 0.9995 and max-abs error <= 2e-2 of the fp32 reference
path; the split-K merge within 1e-5 of the oracle's merge before the bf16
cast."""
import math
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

import kimi_b200  # noqa: E402
from oracle import mla as omla  # noqa: E402
from oracle import mxfp4 as omx  # noqa: E402
from tests.cases import COS_MIN, MAX_ABS, compare, make_case, oracle_out  # noqa: E402

DEV = "cuda:0"


def _bf16(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(DEV)


def _gpu_inputs(case):
    q = _bf16(case["q_bits"])
    kvb = torch.from_numpy(case["kv_buffer"]).to(DEV)
    kvs = torch.from_numpy(case["kv_scales"]).to(DEV)
    ip = torch.from_numpy(case["kv_indptr"]).to(DEV)
    ix = torch.from_numpy(case["kv_indices"]).to(DEV)
    last = torch.from_numpy(case["kv_last_page_len"]).to(DEV)
    return q, kvb, kvs, ip, ix, last


def _decode(case, num_kv_splits=None, heads_first=False):
    q, kvb, kvs, ip, ix, last = _gpu_inputs(case)
    b, h = q.shape[0], q.shape[1]
    if heads_first:
        o_hf = torch.full((h, b, 512), float("nan"), dtype=torch.bfloat16, device=DEV)
        o = o_hf.permute(1, 0, 2)
    else:
        o = torch.full((b, h, 512), float("nan"), dtype=torch.bfloat16, device=DEV)
    kimi_b200.mla_decode_fwd(q, kvb, kvs, o, None, ip, ix, last, sm_scale=case["sm_scale"],
                             num_kv_splits=num_kv_splits)
    torch.cuda.synchronize()
    return o.float().cpu().numpy()


# ---------------------------------------------------------------------------
# quantiser / KV append
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("legacy", [False, True])
def test_quantize_rows_bit_exact_against_golden(golden_dir, legacy):
    g = np.load(os.path.join(golden_dir, "quant_golden.npz"))
    nib, sc = kimi_b200.mxfp4_quantize(_bf16(g["x_bits"]), legacy_rule=legacy)
    torch.cuda.synchronize()
    tag = "legacy" if legacy else "inline"
    assert np.array_equal(sc.cpu().numpy(), g[f"{tag}_scales"])
    assert np.array_equal(nib.cpu().numpy(), g[f"{tag}_nibbles"])


@pytest.mark.parametrize("legacy", [False, True])
def test_kv_append_bit_exact_against_oracle(legacy):
    rng = np.random.default_rng(11)
    n, pages = 300, 7
    kv_c = omx.f32_to_bf16_bits(rng.standard_normal((n, 512), dtype=np.float32) *
                                np.float32(10.0) ** rng.integers(-8, 8, size=(n, 1)).astype(np.float32))
    k_pe = rng.integers(0, 1 << 16, size=(n, 64), dtype=np.uint16)
    slots = rng.permutation(pages * 64)[:n].astype(np.int64)
    slots[::17] = -1  # padded tokens are skipped
    ref_b, ref_s = omla.empty_cache(pages)
    omla.kv_append(ref_b, ref_s, kv_c, k_pe, slots, legacy_rule=legacy)
    kvb, kvs = kimi_b200.alloc_mxfp4_cache(pages, DEV)
    kimi_b200.mxfp4_kv_append(_bf16(kv_c), _bf16(k_pe), kvb, kvs, torch.from_numpy(slots).to(DEV),
                              legacy_rule=legacy)
    torch.cuda.synchronize()
    assert np.array_equal(kvb.cpu().numpy(), ref_b)
    assert np.array_equal(kvs.cpu().numpy(), ref_s)


def test_kv_append_one_token_per_sequence_long_context():
    """The long-context config's append step: one new token for each of 8
    sequences, written into the tail page of each sequence."""
    rng = np.random.default_rng(5)
    pages = 64
    kv_c = omx.f32_to_bf16_bits(rng.standard_normal((8, 512), dtype=np.float32))
    k_pe = omx.f32_to_bf16_bits(rng.standard_normal((8, 64), dtype=np.float32))
    slots = (np.arange(8) * 8 + 7) * 64 + 63  # last row of every 8th page
    ref_b, ref_s = omla.empty_cache(pages)
    omla.kv_append(ref_b, ref_s, kv_c, k_pe, slots)
    kvb, kvs = kimi_b200.alloc_mxfp4_cache(pages, DEV)
    kimi_b200.mxfp4_kv_append(_bf16(kv_c), _bf16(k_pe), kvb, kvs, torch.from_numpy(slots.astype(np.int64)).to(DEV))
    torch.cuda.synchronize()
    assert np.array_equal(kvb.cpu().numpy(), ref_b)
    assert np.array_equal(kvs.cpu().numpy(), ref_s)


# ---------------------------------------------------------------------------
# decode against the golden vectors of the reference
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("case_name", ["plumbing", "ragged", "tails"])
@pytest.mark.parametrize("splits", [None, 1, 4])
def test_decode_against_reference_golden(golden_dir, case_name, splits):
    g = np.load(os.path.join(golden_dir, "decode_golden.npz"))
    case = {k: g[f"{case_name}__{k}"] for k in ("q_bits", "kv_buffer", "kv_scales", "kv_indptr", "kv_indices",
                                                 "kv_last_page_len")}
    case["sm_scale"] = float(g[f"{case_name}__sm_scale"])
    out = _decode(case, num_kv_splits=splits)
    cos, err = compare(out, g[f"{case_name}__out"])
    assert cos >= COS_MIN and err <= MAX_ABS, (cos, err)


# ---------------------------------------------------------------------------
# decode against the oracle on seeded inputs
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("heads", [8, 16, 64, 128])
def test_decode_head_counts(heads):
    case = make_case([512, 200, 1, 129], heads, seed=heads)
    cos, err = compare(_decode(case), oracle_out(case))
    assert cos >= COS_MIN and err <= MAX_ABS, (cos, err)


@pytest.mark.parametrize("ctx", [1, 63, 64, 65, 127, 128, 129, 1000])
def test_decode_tail_lengths(ctx):
    case = make_case([ctx], 16, seed=ctx)
    for splits in (1, 3):
        cos, err = compare(_decode(case, num_kv_splits=splits), oracle_out(case))
        assert cos >= COS_MIN and err <= MAX_ABS, (ctx, splits, cos, err)


def test_decode_empty_sequences_give_zero_rows():
    case = make_case([0, 300, 0, 64], 16, seed=9)
    for splits in (1, 4):
        out = _decode(case, num_kv_splits=splits)
        assert np.all(out[0] == 0) and np.all(out[2] == 0)
        cos, err = compare(out, oracle_out(case))
        assert cos >= COS_MIN and err <= MAX_ABS


@pytest.mark.parametrize("splits", [1, 2, 5, 16, 64])
def test_decode_split_counts(splits):
    case = make_case([2048, 777, 64], 64, seed=100 + splits)
    cos, err = compare(_decode(case, num_kv_splits=splits), oracle_out(case))
    assert cos >= COS_MIN and err <= MAX_ABS, (cos, err)


def test_decode_heads_first_output_layout():
    """o given as the heads-first view (H, B, L).permute(1, 0, 2)
    (patches/atom-optimizations.patch:261-289) is written in place."""
    case = make_case([300, 64, 128], 16, seed=4)
    ref = oracle_out(case)
    for splits in (1, 4):
        out = _decode(case, num_kv_splits=splits, heads_first=True)
        cos, err = compare(out, ref)
        assert cos >= COS_MIN and err <= MAX_ABS


def test_decode_strided_q_rows():
    case = make_case([256, 100], 16, seed=21)
    q, kvb, kvs, ip, ix, last = _gpu_inputs(case)
    big = torch.zeros(2, 24, 576, dtype=torch.bfloat16, device=DEV)
    big[:, 4:20] = q
    o = torch.empty(2, 16, 512, dtype=torch.bfloat16, device=DEV)
    kimi_b200.mla_decode_fwd(big[:, 4:20], kvb, kvs, o, None, ip, ix, last, sm_scale=case["sm_scale"])
    torch.cuda.synchronize()
    cos, err = compare(o.float().cpu().numpy(), oracle_out(case))
    assert cos >= COS_MIN and err <= MAX_ABS


def test_decode_legacy_quantised_cache_and_wide_scales():
    """Cache written by the legacy rule (codes 0 / 0.5 only) and latents whose
    per-token magnitudes span many binades."""
    case = make_case([640, 333], 16, seed=31, legacy_rule=True)
    cos, err = compare(_decode(case), oracle_out(case))
    assert cos >= COS_MIN and err <= MAX_ABS
    case = make_case([640, 333], 16, seed=32, kv_scale=1e-3)
    cos, err = compare(_decode(case), oracle_out(case))
    assert cos >= COS_MIN and err <= MAX_ABS


def test_decode_is_deterministic():
    case = make_case([4096, 1234], 64, seed=77)
    a = _decode(case, num_kv_splits=8)
    b = _decode(case, num_kv_splits=8)
    assert np.array_equal(a, b)


# ---------------------------------------------------------------------------
# split-K merge
# ---------------------------------------------------------------------------
def test_reduce_against_oracle_merge():
    rng = np.random.default_rng(2)
    b, s, h = 3, 5, 16
    po = rng.standard_normal((b, s, h, 512), dtype=np.float32)
    lse = (rng.standard_normal((b, s, h), dtype=np.float32) * 4).astype(np.float32)
    lse[0, 1] = -np.inf
    lse[2, :, 3] = -np.inf  # a head with no tokens at all
    o_hf = torch.empty(h, b, 512, dtype=torch.bfloat16, device=DEV)
    kimi_b200.mla_reduce(torch.from_numpy(po).to(DEV), torch.from_numpy(lse).to(DEV), o_hf.permute(1, 0, 2))
    torch.cuda.synchronize()
    got = o_hf.permute(1, 0, 2).float().cpu().numpy()
    for bi in range(b):
        ref = omla.lse_merge(po[bi], lse[bi])
        assert np.abs(got[bi] - ref).max() <= 2 ** -7 * max(1.0, np.abs(ref).max())
    assert np.all(got[2, 3] == 0)


# ---------------------------------------------------------------------------
# full-size properties (the Kimi-K2 decode shape)
# ---------------------------------------------------------------------------
def test_full_size_kimi_k2_shape_subset_and_split_invariance():
    """64 heads, batch 64, ctx 8192, random page permutation: 16 of the 64
    sequences against the oracle, and the auto split count against 1 and 32
    splits."""
    b, h, ctx = 64, 64, 8192
    gen = torch.Generator(device=DEV).manual_seed(1)
    pages = b * ctx // 64
    kvb, kvs = kimi_b200.alloc_mxfp4_cache(pages, DEV)
    kv_c = torch.randn(pages * 64, 512, generator=gen, device=DEV).to(torch.bfloat16)
    k_pe = torch.randn(pages * 64, 64, generator=gen, device=DEV).to(torch.bfloat16)
    kimi_b200.mxfp4_kv_append(kv_c, k_pe, kvb, kvs, torch.arange(pages * 64, device=DEV))
    perm = torch.randperm(pages, generator=gen, device=DEV).to(torch.int32)
    ip = torch.arange(b + 1, device=DEV, dtype=torch.int32) * (ctx // 64)
    last = torch.full((b,), 64, dtype=torch.int32, device=DEV)
    q = torch.randn(b, h, 576, generator=gen, device=DEV).to(torch.bfloat16)
    sm = 1 / math.sqrt(192)
    outs = {}
    for splits in (None, 1, 32):
        o = torch.empty(b, h, 512, dtype=torch.bfloat16, device=DEV)
        kimi_b200.mla_decode_fwd(q, kvb, kvs, o, None, ip, perm, last, sm_scale=sm, num_kv_splits=splits)
        outs[splits] = o.float().cpu().numpy()
    torch.cuda.synchronize()
    for s in (1, 32):
        cos, err = compare(outs[None], outs[s])
        assert cos >= 0.99999 and err <= 1e-2
    kvb_np, kvs_np = kvb.cpu().numpy(), kvs.cpu().numpy()
    q_bits = q.cpu().view(torch.int16).numpy().view(np.uint16)
    perm_np = perm.cpu().numpy()
    for seq in range(0, 64, 4):  # 16 sequences, a quarter of the batch
        pg = perm_np[seq * 128:(seq + 1) * 128]
        ref = omla.mla_decode(q_bits[seq:seq + 1], kvb_np, kvs_np, np.array([0, 128], np.int32), pg,
                              np.array([64], np.int32), sm)
        cos, err = compare(outs[None][seq:seq + 1], ref)
        assert cos >= COS_MIN and err <= MAX_ABS, (seq, cos, err)
