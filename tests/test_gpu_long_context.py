"""Long-context split-K stress at the DeepSeek-V3 decode shape, on the GPU.

128 heads (two 64-head blocks), 8 sequences of 131071 cached tokens; one new
token per sequence is appended through the MXFP4 KV quantiser (its nibbles,
scales and RoPE must match the oracle's quantisation bit for bit), making
131072 tokens; then the decode runs with 32 splits into a preallocated
workspace.  At this size the oracle checks one whole sequence (its pages are
copied to the host), and the remaining sequences are checked through the
split invariance against the balanced schedule."""
import math

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

import kimi_b200  # noqa: E402
from oracle import mla as omla  # noqa: E402
from tests.cases import COS_MIN, MAX_ABS, compare  # noqa: E402

DEV = "cuda:0"


def test_deepseek_v3_shape_128k_context_32_splits_with_append():
    b, h, ctx = 8, 128, 131072
    gen = torch.Generator(device=DEV).manual_seed(4)
    pages_per = ctx // 64
    pages = b * pages_per
    kvb, kvs = kimi_b200.alloc_mxfp4_cache(pages, DEV)
    perm = torch.randperm(pages, generator=gen, device=DEV).to(torch.int32)
    # flat slot of token t of sequence s: page perm[s * pages_per + t // 64], row t % 64
    tok = torch.arange(ctx - 1, device=DEV, dtype=torch.int64)
    for s in range(b):
        slots = perm[s * pages_per + tok // 64].to(torch.int64) * 64 + tok % 64
        kv_c = torch.randn(ctx - 1, 512, generator=gen, device=DEV).to(torch.bfloat16)
        k_pe = torch.randn(ctx - 1, 64, generator=gen, device=DEV).to(torch.bfloat16)
        kimi_b200.mxfp4_kv_append(kv_c, k_pe, kvb, kvs, slots)
    # the new token of every sequence (position ctx - 1)
    new_c = torch.randn(b, 512, generator=gen, device=DEV).to(torch.bfloat16)
    new_pe = torch.randn(b, 64, generator=gen, device=DEV).to(torch.bfloat16)
    new_slots = (perm[torch.arange(b, device=DEV) * pages_per + (ctx - 1) // 64].to(torch.int64) * 64
                 + (ctx - 1) % 64)
    kimi_b200.mxfp4_kv_append(new_c, new_pe, kvb, kvs, new_slots)
    torch.cuda.synchronize()

    # appended bytes against the oracle quantiser
    want_b, want_s = omla.empty_cache(1)
    omla.kv_append(want_b, want_s, new_c.cpu().view(torch.int16).numpy().view(np.uint16),
                   new_pe.cpu().view(torch.int16).numpy().view(np.uint16), np.arange(b))
    pg = (new_slots // 64).cpu().numpy()
    got_b = kvb.view(-1, 64, 384)[torch.from_numpy(pg).to(DEV), 63].cpu().numpy()
    got_s = kvs.view(-1, 64, 16)[torch.from_numpy(pg).to(DEV), 63].cpu().numpy()
    assert np.array_equal(got_b, want_b.reshape(-1, 384)[:b])
    assert np.array_equal(got_s, want_s.reshape(-1, 16)[:b])

    ip = torch.arange(b + 1, device=DEV, dtype=torch.int32) * pages_per
    last = torch.full((b,), 64, dtype=torch.int32, device=DEV)
    q = torch.randn(b, h, 576, generator=gen, device=DEV).to(torch.bfloat16)
    sm = 1 / math.sqrt(192)
    ws = kimi_b200.alloc_workspace(b, h, 32, torch.device(DEV))
    o32 = torch.empty(b, h, 512, dtype=torch.bfloat16, device=DEV)
    kimi_b200.mla_decode_fwd(q, kvb, kvs, o32, None, ip, perm, last, sm_scale=sm, num_kv_splits=32, workspace=ws)
    o_auto = torch.empty_like(o32)
    kimi_b200.mla_decode_fwd(q, kvb, kvs, o_auto, None, ip, perm, last, sm_scale=sm)
    torch.cuda.synchronize()
    out32 = o32.float().cpu().numpy()
    cos, err = compare(out32, o_auto.float().cpu().numpy())
    # two split layouts round differently: allow one bf16 ulp of the largest output
    ulp = 2.0 ** (math.floor(math.log2(max(float(np.abs(out32).max()), 1e-30))) - 7)
    assert cos >= 0.99999 and err <= max(1e-2, ulp), (cos, err)

    # one whole sequence against the oracle (only its pages leave the GPU)
    seq = 5
    rows = perm[seq * pages_per:(seq + 1) * pages_per].to(torch.int64)
    kvb_seq = kvb.view(-1, 64, 384)[rows].cpu().numpy()
    kvs_seq = kvs.view(-1, 64, 16)[rows].cpu().numpy()
    q_bits = q[seq:seq + 1].cpu().view(torch.int16).numpy().view(np.uint16)
    ref = omla.mla_decode(q_bits, kvb_seq, kvs_seq, np.array([0, pages_per], np.int32),
                          np.arange(pages_per, dtype=np.int32), np.array([64], np.int32), sm)
    cos, err = compare(out32[seq:seq + 1], ref)
    assert cos >= COS_MIN and err <= MAX_ABS, (cos, err)
