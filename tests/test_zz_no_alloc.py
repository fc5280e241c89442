"""kimi_mla_decode_static_workspace: the decode for callers that cannot
allocate device memory (a foreign-language binding holding only the pointers
an engine handed it, or an engine that reserved all free HBM up front).

It takes its split-K partials from a 32 MiB array compiled into the library
instead of a caller workspace.  These tests call it through the C ABI, twice
in a row on different inputs, and check each result against the regular
kimi_mla_decode entry point (given a torch-allocated workspace) on the same
inputs, with the tolerance of the other decode tests, and against the CPU
oracle.  The file is named to run last so that a stop-at-first-failure run
has already run every other test."""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

from kimi_b200 import _lib  # noqa: E402
from tests.cases import COS_MIN, MAX_ABS, compare, make_case, oracle_out  # noqa: E402

DEV = "cuda:0"


def _inputs(case):
    def t(a):
        return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    q = t(case["q_bits"].view(np.int16)).view(torch.bfloat16)
    return dict(q=q, kvb=t(case["kv_buffer"]), kvs=t(case["kv_scales"]), ip=t(case["kv_indptr"]),
                ix=t(case["kv_indices"]), last=t(case["kv_last_page_len"]))


def _params(x, o, case, splits):
    b, h = x["q"].shape[0], x["q"].shape[1]
    return _lib.KimiMlaDecodeParams(
        q=x["q"].data_ptr(), q_stride_b=x["q"].stride(0), q_stride_h=x["q"].stride(1),
        kv_buffer=x["kvb"].data_ptr(), kv_scales=x["kvs"].data_ptr(), num_pages=x["kvb"].shape[0],
        kv_indptr=x["ip"].data_ptr(), kv_indices=x["ix"].data_ptr(), kv_last_page_len=x["last"].data_ptr(),
        o=o.data_ptr(), o_stride_b=o.stride(0), o_stride_h=o.stride(1), batch=b, num_heads=h,
        num_kv_splits=splits, sm_scale=case["sm_scale"], logit_cap=0.0)


def _run_regular(lib, case, splits):
    x = _inputs(case)
    b, h = x["q"].shape[0], x["q"].shape[1]
    o = torch.empty(b, h, 512, dtype=torch.bfloat16, device=DEV)
    need = lib.kimi_mla_decode_workspace_size(b, h, splits)
    ws = torch.empty(max(need, 256), dtype=torch.uint8, device=DEV)
    p = _params(x, o, case, splits)
    st = lib.kimi_mla_decode(ctypes.byref(p), ws.data_ptr(), ws.numel(),
                             torch.cuda.current_stream().cuda_stream)
    assert st == 0, _lib.status_text(st)
    torch.cuda.synchronize()
    return o.float().cpu().numpy()


def _run_static(lib, case, splits):
    x = _inputs(case)
    b, h = x["q"].shape[0], x["q"].shape[1]
    o = torch.full((b, h, 512), float("nan"), dtype=torch.bfloat16, device=DEV)
    p = _params(x, o, case, splits)
    st = lib.kimi_mla_decode_static_workspace(ctypes.byref(p), torch.cuda.current_stream().cuda_stream)
    assert st == 0, _lib.status_text(st)
    torch.cuda.synchronize()
    return o.float().cpu().numpy()


def test_static_workspace_decode_matches_regular_entry_point_twice_in_a_row():
    lib = _lib.load()
    case_a = make_case([512, 512], 16, seed=0)                    # batch 2, 16 heads, ctx 512
    case_b = make_case([2048, 700, 1, 1500, 64, 0, 999, 128], 64, seed=1)  # ragged, 64 heads
    splits_a, splits_b = 4, 8
    need_b = lib.kimi_mla_decode_workspace_size(8, 64, splits_b)
    assert 0 < need_b <= 32 << 20
    first = _run_static(lib, case_a, splits_a)
    second = _run_static(lib, case_b, splits_b)
    for got, case, splits in ((first, case_a, splits_a), (second, case_b, splits_b)):
        want = _run_regular(lib, case, splits)
        cos, err = compare(got, want)
        assert cos >= COS_MIN and err <= MAX_ABS, (cos, err)
        cos, err = compare(got, oracle_out(case))
        assert cos >= COS_MIN and err <= MAX_ABS, (cos, err)
    # the array keeps the previous call's contents; a repeat of the first call is unaffected
    again = _run_static(lib, case_a, splits_a)
    assert np.array_equal(again, first)


def test_static_workspace_balanced_schedule_after_a_call_that_filled_the_array():
    """The balanced schedule (num_kv_splits = 0) reads partial rows, log-sum-
    exps and CTA-pair spans from slots that differ from call to call.  A first
    call in split mode fills several MiB of the array with its own partials;
    a balanced call after it, on ragged sequences that straddle pairs, must
    still match the regular entry point: it writes every slot its merge
    reads, whatever the array held."""
    lib = _lib.load()
    fill = make_case([2048] * 16, 64, seed=5)      # 16 x 16 splits x 64 heads of partials
    ragged = make_case([8192, 300, 5000, 64, 12000, 1, 2048, 700], 64, seed=6)
    need_fill = lib.kimi_mla_decode_workspace_size(16, 64, 16)
    need_bal = lib.kimi_mla_decode_workspace_size(8, 64, 0)
    assert need_bal <= need_fill <= 32 << 20
    _run_static(lib, fill, 16)
    got = _run_static(lib, ragged, 0)
    want = _run_regular(lib, ragged, 0)
    cos, err = compare(got, want)
    assert cos >= COS_MIN and err <= MAX_ABS, (cos, err)
    cos, err = compare(got, oracle_out(ragged))
    assert cos >= COS_MIN and err <= MAX_ABS, (cos, err)
    # and twice in a row: the same call again gives the same bits
    assert np.array_equal(_run_static(lib, ragged, 0), got)


def test_static_workspace_rejects_sizes_beyond_its_limit():
    lib = _lib.load()
    # 128 sequences x 64 splits x 128 heads of partials is far beyond 32 MiB
    assert lib.kimi_mla_decode_workspace_size(128, 128, 64) > 32 << 20
    case = make_case([64], 16, seed=3)
    x = _inputs(case)
    o = torch.zeros(1, 16, 512, dtype=torch.bfloat16, device=DEV)
    p = _params(x, o, case, 64)
    p.batch, p.num_heads = 128, 128  # sizes checked on the host; nothing is launched
    st = lib.kimi_mla_decode_static_workspace(ctypes.byref(p), torch.cuda.current_stream().cuda_stream)
    assert st == -7
    assert "32 MiB" in _lib.status_text(st)
    torch.cuda.synchronize()
    assert torch.count_nonzero(o).item() == 0
