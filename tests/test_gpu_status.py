"""Device-side failure reporting of the decode through the C ABI.

Every wait inside the decode kernels is bounded in time; a wait that runs out
ends its CTA's work cleanly and ORs a KIMI_DEVICE_* bit into the caller's
status word, which kimi_device_status (kimi_b200.device_status) reads back.
These tests make waits run out on purpose with a 1 ns bound (the kernels then
give up at the first wait that is not already satisfied: no fault, no hang),
check that the word reports it, and that the next call on the same context
runs normally.  A page id outside the cache is reported the same way; its
tokens read as zeros, which the oracle reproduces with an all-zero page."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

import kimi_b200  # noqa: E402
from kimi_b200 import _lib  # noqa: E402
from tests.cases import COS_MIN, MAX_ABS, compare, make_case, oracle_out  # noqa: E402

DEV = "cuda:0"


def _run(case, splits, status=None, timeout_ns=0, kv=None):
    def t(x):
        return torch.from_numpy(np.ascontiguousarray(x)).to(DEV)
    q = t(case["q_bits"].view(np.int16)).view(torch.bfloat16)
    kvb, kvs = kv if kv is not None else (case["kv_buffer"], case["kv_scales"])
    o = torch.full((q.shape[0], q.shape[1], 512), float("nan"), dtype=torch.bfloat16, device=DEV)
    kimi_b200.mla_decode_fwd(q, t(kvb), t(kvs), o, None, t(case["kv_indptr"]), t(case["kv_indices"]),
                             t(case["kv_last_page_len"]), sm_scale=case["sm_scale"], num_kv_splits=splits,
                             status=status, timeout_ns=timeout_ns)
    torch.cuda.synchronize()
    return o.float().cpu().numpy()


def test_wait_timeout_is_reported_and_the_next_call_runs():
    case = make_case([4096, 700, 2048, 64], 64, seed=21)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    _run(case, 4, status=status, timeout_ns=1)
    bits = kimi_b200.device_status(status, clear=True)
    assert bits != 0 and (bits & _lib.DEVICE_WAIT_BITS) == bits, hex(bits)
    assert "gave up" in _lib.status_text(bits)
    with pytest.raises(RuntimeError):
        status.fill_(bits)
        kimi_b200.check_device_status(status, clear=True)
    assert kimi_b200.device_status(status) == 0  # cleared
    # the context is intact: the same call with the default bound is exact again
    out = _run(case, 4, status=status)
    assert kimi_b200.device_status(status) == 0
    cos, err = compare(out, oracle_out(case))
    assert cos >= COS_MIN and err <= MAX_ABS, (cos, err)


@pytest.mark.parametrize("splits,past_end", [(None, True), (2, True), (None, False)])
def test_out_of_range_page_id_reads_as_zeros_and_is_reported(splits, past_end):
    """A page id past the cache or negative (both map to rows outside the
    cache's tensor map, which the copy engine fills with zeros)."""
    case = make_case([1000, 3000, 200], 64, seed=22)
    pages = case["kv_buffer"].shape[0]
    bad = dict(case)
    bad["kv_indices"] = case["kv_indices"].copy()
    bad["kv_indices"][5] = pages + 7 if past_end else -3  # inside sequence 1
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = _run(bad, splits, status=status)
    bits = kimi_b200.device_status(status)
    assert bits & _lib.DEVICE_BAD_PAGE, hex(bits)
    assert (bits & _lib.DEVICE_WAIT_BITS) == 0, hex(bits)
    # the oracle with that id pointing at an all-zero page
    kvb = np.concatenate([case["kv_buffer"], np.zeros((8,) + case["kv_buffer"].shape[1:], np.uint8)])
    kvs = np.concatenate([case["kv_scales"], np.zeros((8,) + case["kv_scales"].shape[1:], np.uint8)])
    ref_ix = bad["kv_indices"].copy()
    ref_ix[5] = pages  # the first of the appended zero pages
    ref = dict(bad, kv_indices=ref_ix, kv_buffer=kvb, kv_scales=kvs)
    cos, err = compare(out, oracle_out(ref))
    assert cos >= COS_MIN and err <= MAX_ABS, (cos, err)
