"""The decode and the TP8 steps captured into CUDA graphs: a replay with new
inputs written into the captured tensors gives the eager call's bits, and the
decode matches the CPU oracle.  Every entry point is asynchronous, allocates
nothing once its workspace (or scratch) is given, and never synchronises, so
it captures."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

import kimi_b200  # noqa: E402
from tests.cases import COS_MIN, MAX_ABS, compare, make_case, oracle_out  # noqa: E402

DEV = "cuda:0"


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


@pytest.mark.parametrize("num_kv_splits", [None, 4])
def test_decode_replay_matches_eager_and_oracle(num_kv_splits):
    case_a = make_case([700, 64, 1500], 16, seed=31, shuffle=False)
    case_b = make_case([700, 64, 1500], 16, seed=32, shuffle=False)  # same page table, other q and cache
    np.testing.assert_array_equal(case_a["kv_indices"], case_b["kv_indices"])
    q = _dev(case_a["q_bits"].view(np.int16)).view(torch.bfloat16)
    kvb, kvs = _dev(case_a["kv_buffer"]), _dev(case_a["kv_scales"])
    ip, px, la = _dev(case_a["kv_indptr"]), _dev(case_a["kv_indices"]), _dev(case_a["kv_last_page_len"])
    o = torch.empty(3, 16, 512, dtype=torch.bfloat16, device=DEV)
    ws = kimi_b200.alloc_workspace(3, 16, num_kv_splits, DEV)

    def call():
        kimi_b200.mla_decode_fwd(q, kvb, kvs, o, None, ip, px, la, sm_scale=case_a["sm_scale"],
                                 num_kv_splits=num_kv_splits, workspace=ws)

    call()  # eager first: the library's one-time lookups happen outside capture
    torch.cuda.synchronize()
    eager_a = o.clone()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        call()
    # new inputs into the captured tensors, then replay
    q.copy_(_dev(case_b["q_bits"].view(np.int16)).view(torch.bfloat16))
    kvb.copy_(_dev(case_b["kv_buffer"]))
    kvs.copy_(_dev(case_b["kv_scales"]))
    graph.replay()
    torch.cuda.synchronize()
    replay_b = o.clone()
    call()
    torch.cuda.synchronize()
    assert torch.equal(replay_b, o)  # the replay is the eager call, bit for bit
    cos, err = compare(replay_b.float().cpu().numpy(), oracle_out(case_b))
    assert cos >= COS_MIN and err <= MAX_ABS, (cos, err)
    assert not torch.equal(eager_a, replay_b)
    del graph


def test_tp8_steps_replay_matches_eager():
    """q absorption + RoPE + KV append, and V up-projection + o_proj, in one graph."""
    g = torch.Generator(device=DEV).manual_seed(3)
    T, H = 128, 8
    bf = torch.bfloat16
    q = torch.randn(T, H, 192, generator=g, device=DEV).to(bf)
    w_uk = (torch.randn(H, 128, 512, generator=g, device=DEV) / 11.3).to(bf)
    kv_c = torch.randn(T, 512, generator=g, device=DEV).to(bf)
    k_pe = torch.randn(T, 64, generator=g, device=DEV).to(bf)
    pos = torch.randint(0, 4096, (T,), generator=g, device=DEV)
    ang = torch.arange(4096, device=DEV, dtype=torch.float64)[:, None] * (
        1.0 / (10000.0 ** (torch.arange(32, device=DEV, dtype=torch.float64) / 32.0)))[None, :]
    cos, sin = ang.cos().float().contiguous(), ang.sin().float().contiguous()
    kvb, kvs = kimi_b200.alloc_mxfp4_cache(T // 64, DEV)
    slots = torch.arange(T, device=DEV, dtype=torch.int64)
    q_out = torch.empty(T, H, 576, dtype=bf, device=DEV)
    o_hf = torch.randn(H, T, 512, generator=g, device=DEV).to(bf)
    w_uv = (torch.randn(H, 512, 128, generator=g, device=DEV) * 0.02).to(bf)
    w_o = (torch.randn(7168, H * 128, generator=g, device=DEV) * 0.02).to(bf)
    x = torch.empty(T, H * 128, dtype=bf, device=DEV)
    out = torch.empty(T, 7168, dtype=bf, device=DEV)

    def call():
        kimi_b200.q_absorb_rope_append(q[:, :, :128], q[:, :, 128:], w_uk, kv_c, k_pe, pos, cos, sin, kvb, kvs,
                                       slots, q_out=q_out)
        kimi_b200.v_up_proj_and_o_proj(o_hf, w_uv, w_o, out=out, x=x)

    call()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        call()
    q.copy_(torch.randn(T, H, 192, generator=g, device=DEV).to(bf))
    kv_c.copy_(torch.randn(T, 512, generator=g, device=DEV).to(bf))
    o_hf.copy_(torch.randn(H, T, 512, generator=g, device=DEV).to(bf))
    graph.replay()
    torch.cuda.synchronize()
    got = (q_out.clone(), kvb.clone(), kvs.clone(), out.clone())
    call()
    torch.cuda.synchronize()
    for a, b in zip(got, (q_out, kvb, kvs, out)):
        assert torch.equal(a, b)
    del graph
