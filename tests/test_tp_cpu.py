"""The host logic of the tensor-parallel all-reduce step (kimi_b200.tp) on the
CPU: two gloo ranks build a PeerPartials with a stand-in for the CUDA IPC
layer, so the handle exchange, the rank order of the mapped partials, the
argument checks before the first barrier and the collective teardown run
without a GPU.  The kernel itself is covered by tests/test_gpu_ar_norm.py."""
import datetime
import os
import socket

import pytest

torch = pytest.importorskip("torch")

from kimi_b200 import _lib, tp  # noqa: E402

PEER_BASE = 0x7F0000000000  # stand-in base address of rank r's mapping: PEER_BASE * (r + 1)


class FakeIpc:
    """Records what PeerPartials asks of the IPC layer; the handle of rank r is
    b"rank<r>" and its buffer sits 256 * (r + 1) bytes into its allocation."""

    def __init__(self, rank):
        self.rank = rank
        self.current = None
        self.opened, self.closed, self.synced = [], [], 0

    def export(self, ptr):
        return f"rank{self.rank}".encode(), 256 * (self.rank + 1)

    def make_current(self, device):
        self.current = device

    def open(self, raw):
        r = int(raw.decode()[4:])
        assert r != self.rank, "a rank maps only its peers"
        assert self.current is not None, "mappings are opened with the device selected"
        base = PEER_BASE * (r + 1)
        self.opened.append(base)
        return base

    def close(self, base):
        self.closed.append(base)

    def synchronize(self, device):
        self.synced += 1


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, result_dir):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        ipc = FakeIpc(rank)
        peers = tp.PeerPartials(16, 256, torch.device("cpu"), ipc=ipc)
        assert peers.local.shape == (16, 256) and peers.local.dtype == torch.bfloat16
        want = [peers.local.data_ptr() if r == rank else PEER_BASE * (r + 1) + 256 * (r + 1) for r in range(world)]
        assert peers.ptrs == want, (peers.ptrs, want)
        assert sorted(ipc.opened) == sorted(PEER_BASE * (r + 1) for r in range(world) if r != rank)
        # shapes are checked before the first barrier, on every rank alike
        with pytest.raises(ValueError):
            peers.reduce_norm_quant(torch.zeros(17, 256, dtype=torch.bfloat16), torch.zeros(256, dtype=torch.bfloat16))
        with pytest.raises(ValueError):
            peers.reduce_norm_quant(torch.zeros(4, 128, dtype=torch.bfloat16), torch.zeros(128, dtype=torch.bfloat16))
        peers.close()  # collective: synchronise, unmap every peer, barrier
        assert ipc.synced == 1 and sorted(ipc.closed) == sorted(ipc.opened) and peers.ptrs == []
        with pytest.raises(RuntimeError):
            peers.reduce_norm_quant(torch.zeros(4, 256, dtype=torch.bfloat16), torch.zeros(256, dtype=torch.bfloat16))
        # more ranks than the kernel sums is refused before any exchange
        saved = _lib.AR_MAX_INPUTS
        _lib.AR_MAX_INPUTS = world - 1
        try:
            with pytest.raises(ValueError):
                tp.PeerPartials(16, 256, torch.device("cpu"), ipc=FakeIpc(rank))
        finally:
            _lib.AR_MAX_INPUTS = saved
        with open(os.path.join(result_dir, f"rank{rank}"), "w") as f:
            f.write("ok")
    finally:
        dist.destroy_process_group()


def test_two_rank_exchange_and_teardown(tmp_path):
    import torch.multiprocessing as mp
    world = 2
    mp.spawn(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    for r in range(world):
        assert (tmp_path / f"rank{r}").read_text() == "ok"


class FailingExportIpc(FakeIpc):
    """Rank 1's export fails (as cudaIpcGetMemHandle does on an allocation
    from expandable segments)."""

    def export(self, ptr):
        if self.rank == 1:
            raise RuntimeError("cudaIpcGetMemHandle failed: CUDA error 1")
        return super().export(ptr)


class FailingCloseIpc(FakeIpc):
    """Every unmap reports an error after recording the call."""

    def close(self, base):
        super().close(base)
        raise RuntimeError("cudaIpcCloseMemHandle failed: CUDA error 400")


def _failure_rank_main(rank, world, port, result_dir):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    # a short group timeout: a rank left waiting in a collective fails the test quickly
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        # one rank's export fails: every rank joins the gather and raises the same error
        ipc = FailingExportIpc(rank)
        with pytest.raises(RuntimeError, match=r"export failed on rank\(s\) 1: RuntimeError: cudaIpcGetMemHandle"):
            tp.PeerPartials(16, 256, torch.device("cpu"), ipc=ipc)
        assert ipc.opened == []
        # an unmap error is raised, after the closing barrier every rank reaches
        ipc = FailingCloseIpc(rank)
        peers = tp.PeerPartials(16, 256, torch.device("cpu"), ipc=ipc)
        with pytest.raises(RuntimeError, match="cudaIpcCloseMemHandle"):
            peers.close()
        assert sorted(ipc.closed) == sorted(ipc.opened) and peers.ptrs == []
        # the group is still in step: one more collective completes on both ranks
        t = torch.ones(1)
        dist.all_reduce(t)
        assert t.item() == world
        with open(os.path.join(result_dir, f"rank{rank}"), "w") as f:
            f.write("ok")
    finally:
        dist.destroy_process_group()


def test_two_rank_export_and_unmap_failures_raise_on_every_rank(tmp_path):
    import torch.multiprocessing as mp
    world = 2
    mp.spawn(_failure_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    for r in range(world):
        assert (tmp_path / f"rank{r}").read_text() == "ok"
