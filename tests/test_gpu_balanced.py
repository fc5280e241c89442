"""GPU parity of the balanced schedule (num_kv_splits = None / 0).

With automatic split selection the decode lays the batch's 128-token tiles
end to end and gives every CTA (one per SM per 64-head block) an equal run of
them, so a CTA may finish one sequence, build the next sequence's Q and carry
on, and a sequence may be spread over several CTAs whose partials the
log-sum-exp merge combines.  These cases aim at those paths: runs that cross
many sequence boundaries, sequences spread over many CTAs, empty sequences,
batches far smaller and far larger than the SM count, two head blocks.  Bars
as in the other decode tests: cosine >= 0.9995 and max-abs <= 2e-2 against
the fp32 oracle."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

import kimi_b200  # noqa: E402
from tests.cases import COS_MIN, MAX_ABS, compare, make_case, oracle_out  # noqa: E402
from tests.test_gpu_parity import _decode  # noqa: E402


def _check(case, out):
    cos, err = compare(out, oracle_out(case))
    assert cos >= COS_MIN and err <= MAX_ABS, (cos, err)


def test_ragged_batch_with_empty_sequences():
    rng = np.random.default_rng(7)
    lens = [int(x) for x in rng.integers(1, 1500, 160)]
    for i in (0, 17, 63, 159):
        lens[i] = 0
    case = make_case(lens, 64, seed=7)
    out = _decode(case)
    _check(case, out)
    for i in (0, 17, 63, 159):
        assert np.all(out[i] == 0.0)


def test_one_long_sequence_spread_over_many_ctas():
    case = make_case([8192], 16, seed=8)
    _check(case, _decode(case))


def test_many_short_sequences_per_cta():
    # ~600 tiles for 148 CTAs: every CTA walks several sequences and rebuilds Q
    rng = np.random.default_rng(9)
    lens = [int(x) for x in rng.integers(1, 260, 420)]
    case = make_case(lens, 32, seed=9)
    _check(case, _decode(case))


def test_two_head_blocks():
    case = make_case([3000, 5000, 100, 1, 2049], 128, seed=10)
    _check(case, _decode(case))


def test_balanced_agrees_with_split_mode_and_is_deterministic():
    case = make_case([4000, 2500, 700, 64, 1300, 9000], 64, seed=11)
    auto = _decode(case)
    again = _decode(case)
    split = _decode(case, num_kv_splits=4)
    diff = np.argwhere(~((auto == again) | (np.isnan(auto) & np.isnan(again))))
    assert diff.size == 0, (
        f"{len(diff)} outputs differ between two identical calls; sequences {sorted(set(diff[:, 0].tolist()))}, "
        f"heads {sorted(set(diff[:, 1].tolist()))[:16]}, latents {diff[:, 2].min()}..{diff[:, 2].max()}, "
        f"NaN in the first call {int(np.isnan(auto).sum())}, in the second {int(np.isnan(again).sum())}")
    _check(case, auto)
    _check(case, split)
    assert np.abs(auto - split).max() <= 2 * MAX_ABS


def test_heads_first_output():
    case = make_case([777, 4096, 1, 2000], 64, seed=12)
    _check(case, _decode(case, heads_first=True))


def test_workspace_is_preallocatable_for_graph_capture():
    case = make_case([1200, 300], 64, seed=13)
    ws = kimi_b200.alloc_workspace(2, 64, None, torch.device("cuda:0"))
    assert ws.numel() >= kimi_b200.workspace_bytes(2, 64, None) > 0
    from tests.test_gpu_parity import _gpu_inputs
    q, kvb, kvs, ip, ix, last = _gpu_inputs(case)
    o = torch.empty(2, 64, 512, dtype=torch.bfloat16, device="cuda:0")
    kimi_b200.mla_decode_fwd(q, kvb, kvs, o, None, ip, ix, last, sm_scale=case["sm_scale"], workspace=ws)
    torch.cuda.synchronize()
    _check(case, o.float().cpu().numpy())


@pytest.mark.parametrize("splits", [None, 1, 4])
def test_partial_then_merge_equals_one_call(splits):
    from tests.test_gpu_parity import _gpu_inputs
    case = make_case([2500, 64, 900], 64, seed=14)
    q, kvb, kvs, ip, ix, last = _gpu_inputs(case)
    ws = kimi_b200.alloc_workspace(3, 64, splits, torch.device("cuda:0"))
    o1 = torch.empty(3, 64, 512, dtype=torch.bfloat16, device="cuda:0")
    o2 = torch.full((3, 64, 512), float("nan"), dtype=torch.bfloat16, device="cuda:0")
    args = (q, kvb, kvs)
    kimi_b200.mla_decode_fwd(*args, o1, None, ip, ix, last, sm_scale=case["sm_scale"], num_kv_splits=splits,
                             workspace=ws)
    kimi_b200.mla_decode_partial(*args, o2, None, ip, ix, last, sm_scale=case["sm_scale"], num_kv_splits=splits,
                                 workspace=ws)
    kimi_b200.mla_decode_merge(*args, o2, None, ip, ix, last, sm_scale=case["sm_scale"], num_kv_splits=splits,
                               workspace=ws)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2)


def test_batch_sharded_ranks_on_one_gpu_match_the_oracle():
    # the data-parallel path with its ranks run one after another on this GPU:
    # each decodes its bin-packed share through its own page table, the shares
    # are put back in batch order (as kimi_b200.dp.gather_outputs does on rank 0)
    from kimi_b200 import dp
    from tests.test_gpu_parity import _gpu_inputs
    rng = np.random.default_rng(15)
    lens = [int(x) for x in rng.integers(1, 3000, 24)] + [0]
    case = make_case(lens, 64, seed=15)
    q, kvb, kvs, ip, ix, last = _gpu_inputs(case)
    world = 3
    shards = dp.shard_sequences(lens, world)
    out = torch.full((len(lens), 64, 512), float("nan"), dtype=torch.bfloat16, device="cuda:0")
    for r in range(world):
        lip, lix, llast = dp.local_batch(shards[r], ip, ix, last)
        o_local = torch.empty(len(shards[r]), 64, 512, dtype=torch.bfloat16, device="cuda:0")
        kimi_b200.mla_decode_fwd(q[shards[r]].contiguous(), kvb, kvs, o_local, None, lip, lix, llast,
                                 sm_scale=case["sm_scale"])
        out[torch.tensor(shards[r], dtype=torch.long, device="cuda:0")] = o_local
    torch.cuda.synchronize()
    _check(case, out.float().cpu().numpy())
