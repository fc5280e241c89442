"""Batch sharding across ranks (kimi_b200.dp) on the CPU.

The host logic of the multi-GPU path: longest-first bin packing of sequences
over ranks, the per-rank page tables, and the gather of per-rank outputs to
rank 0 through torch.distributed (gloo, two processes on this host).  The
per-rank "decode" here is the oracle run on the rank's local page table, so
the gathered batch must equal the oracle of the whole batch exactly."""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from kimi_b200 import dp  # noqa: E402
from tests.cases import make_case, oracle_out  # noqa: E402
from oracle import mla as omla  # noqa: E402


def test_shard_sequences_is_a_balanced_partition():
    rng = np.random.default_rng(3)
    for world in (1, 2, 3, 8):
        lens = [int(x) for x in rng.integers(1024, 32768, 256)]
        shards = dp.shard_sequences(lens, world)
        flat = sorted(i for s in shards for i in s)
        assert flat == list(range(len(lens)))
        loads = dp.shard_loads(lens, shards)
        assert max(loads) - sum(lens) / world <= max(lens)
        assert shards == dp.shard_sequences(lens, world)  # deterministic
    # more ranks than sequences: some ranks get nothing
    shards = dp.shard_sequences([5, 3], 4)
    assert sorted(len(s) for s in shards) == [0, 0, 1, 1]


def test_local_batch_renumbers_the_page_table():
    case = make_case([130, 0, 64, 700, 1], 8, seed=4)
    ip, ix, last = (torch.from_numpy(case[k]) for k in ("kv_indptr", "kv_indices", "kv_last_page_len"))
    lip, lix, llast = dp.local_batch([3, 0, 1], ip, ix, last)
    assert lip.tolist() == [0, int(ip[4] - ip[3]), int(ip[4] - ip[3] + ip[1] - ip[0]),
                            int(ip[4] - ip[3] + ip[1] - ip[0])]
    assert lix.tolist() == ix[ip[3]:ip[4]].tolist() + ix[ip[0]:ip[1]].tolist()
    assert llast.tolist() == [int(last[3]), int(last[0]), int(last[1])]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, lens, seed):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        case = make_case(lens, 16, seed=seed)
        shards = dp.shard_sequences(lens, world)
        ip, ix, last = (torch.from_numpy(case[k]) for k in ("kv_indptr", "kv_indices", "kv_last_page_len"))
        lip, lix, llast = dp.local_batch(shards[rank], ip, ix, last)
        q_local = case["q_bits"][shards[rank]]
        out_local = omla.mla_decode(q_local, case["kv_buffer"], case["kv_scales"], lip.numpy(), lix.numpy(),
                                    llast.numpy(), case["sm_scale"]) if shards[rank] else np.zeros((0, 16, 512))
        o_local = torch.from_numpy(np.asarray(out_local, dtype=np.float32))
        full = dp.gather_outputs(o_local, shards, rank, world, batch=len(lens))
        if rank == 0:
            want = oracle_out(case)
            assert full is not None and np.array_equal(full.numpy(), want.astype(np.float32))
        else:
            assert full is None
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_two_rank_gather_equals_single_batch(world):
    import torch.multiprocessing as mp
    rng = np.random.default_rng(11)
    lens = [int(x) for x in rng.integers(1, 600, 7)] + [0]
    mp.spawn(_rank_main, args=(world, _free_port(), lens, 11), nprocs=world, join=True)


def _failing_rank_main(rank, world, port, result_dir, mode):
    """Rank 1 fails before the gather: it raises and exits ("exits"), or
    stays alive without joining ("absent").  Rank 0 must get an error from
    gather_outputs within its timeout, not block."""
    import datetime
    import time
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    done = os.path.join(result_dir, "rank0_done")
    shards = [[0, 2], [1]]
    o_local = torch.ones(len(shards[rank]), 4, 512)
    if rank == 1:
        if mode == "exits":
            os._exit(0)  # a rank that died before the gather (no teardown)
        for _ in range(600):  # alive, never joining, until rank 0 has its answer
            if os.path.exists(done):
                break
            time.sleep(0.05)
        os._exit(0)
    t0 = time.monotonic()
    try:
        dp.gather_outputs(o_local, shards, rank, world, batch=3, timeout=2.0)
        outcome = "returned"
    except RuntimeError as e:
        outcome = "raised" if "not every rank joined" in str(e) else f"other: {e}"
    elapsed = time.monotonic() - t0
    with open(os.path.join(result_dir, "rank0"), "w") as f:
        f.write(f"{outcome} {elapsed:.2f}")
    open(done, "w").close()
    os._exit(0)  # the group is not to be used again after a failed gather


@pytest.mark.parametrize("mode", ["absent", "exits"])
def test_gather_raises_in_bounded_time_when_a_rank_fails(mode, tmp_path):
    import torch.multiprocessing as mp
    ctx = mp.start_processes(_failing_rank_main, args=(2, _free_port(), str(tmp_path), mode), nprocs=2,
                             join=False, start_method="spawn")
    for p in ctx.processes:
        p.join(60)
        assert p.exitcode == 0, p.exitcode
    outcome, elapsed = (tmp_path / "rank0").read_text().split()
    assert outcome == "raised", outcome
    assert float(elapsed) < 30.0
