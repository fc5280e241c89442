"""Batch-sharded (data-parallel) decode over several GPUs, one process per GPU.

Decode sequences are independent, so a batch spreads over ranks by sequence
with no exchange inside the kernel: each rank holds its sequences' cache pages,
page table and workspace and runs the single-GPU decode on them; afterwards the
outputs come together on one rank.  This is the data-parallel attention
arrangement the reference's serving stack runs across an 8-GPU box (every rank
owns whole requests; the TP8 layout with replicated KV is the other one).

* :func:`shard_sequences` assigns sequences to ranks by greedy
  longest-processing-time bin packing on token counts (the longest sequence
  goes to the least-loaded rank), which keeps ragged batches balanced to within
  one sequence.
* :func:`local_batch` cuts a rank's sequences (their page-table rows) out of a
  global page table, for callers that build the whole batch on every rank.
* :func:`gather_outputs` collects the ranks' outputs ``[n_local, heads, 512]``
  into the batch order on rank ``dst`` with one all_gather of padded shards
  (NCCL for CUDA tensors, gloo for CPU tensors).
"""
from __future__ import annotations

import heapq
from typing import Sequence

import torch


def shard_sequences(seq_lens: Sequence[int], world: int) -> list[list[int]]:
    """Sequence indices per rank, each list in ascending order.

    Greedy LPT: sequences in decreasing length (ties by index) each go to the
    rank with the fewest tokens so far (ties to the lower rank), so the most
    loaded rank exceeds the mean by at most one sequence's length."""
    if world < 1:
        raise ValueError("world must be >= 1")
    order = sorted(range(len(seq_lens)), key=lambda i: (-int(seq_lens[i]), i))
    heap = [(0, r) for r in range(world)]
    shards: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        load, r = heapq.heappop(heap)
        shards[r].append(i)
        heapq.heappush(heap, (load + int(seq_lens[i]), r))
    return [sorted(s) for s in shards]


def shard_loads(seq_lens: Sequence[int], shards: Sequence[Sequence[int]]) -> list[int]:
    return [sum(int(seq_lens[i]) for i in s) for s in shards]


def local_batch(indices: Sequence[int], kv_indptr: torch.Tensor, kv_indices: torch.Tensor,
                kv_last_page_len: torch.Tensor | None):
    """Page-table rows of the given sequences, renumbered from 0.

    Returns (kv_indptr, kv_indices, kv_last_page_len) for the local batch; the
    page ids keep pointing into the same cache."""
    ip = kv_indptr.detach().to("cpu", torch.int64)
    idx = torch.as_tensor(list(indices), dtype=torch.int64)
    starts, ends = ip[idx], ip[idx + 1]
    counts = (ends - starts).clamp(min=0)
    new_ip = torch.zeros(len(idx) + 1, dtype=torch.int64)
    new_ip[1:] = torch.cumsum(counts, 0)
    pieces = [kv_indices[int(s):int(s) + int(c)] for s, c in zip(starts, counts)]
    new_ix = torch.cat(pieces) if pieces else kv_indices[:0]
    dev = kv_indptr.device
    last = None if kv_last_page_len is None else kv_last_page_len[idx.to(kv_last_page_len.device)]
    return new_ip.to(device=dev, dtype=torch.int32), new_ix.to(torch.int32).contiguous(), last


def gather_outputs(o_local: torch.Tensor, shards: Sequence[Sequence[int]], rank: int, world: int,
                   batch: int, dst: int = 0, group=None, timeout: float | None = None) -> torch.Tensor | None:
    """Outputs of all ranks in batch order on rank ``dst`` (None elsewhere).

    ``o_local`` is this rank's ``[len(shards[rank]), heads, 512]`` result in
    the order of ``shards[rank]``.  Every rank takes part (one all_gather).

    ``timeout`` (seconds): bound of the wait for the other ranks.  A rank that
    does not join within it (it failed before the gather, or never reached
    it) makes this call raise ``RuntimeError`` on the ranks that did join,
    instead of leaving them blocked until the process group's own timeout;
    the process group is then not to be used again.  ``None`` waits as the
    process group does."""
    import datetime

    import torch.distributed as dist

    if len(shards) != world or o_local.shape[0] != len(shards[rank]):
        raise ValueError("o_local must hold this rank's sequences in shard order")
    tail = tuple(o_local.shape[1:])
    if world == 1:
        out = torch.empty((batch,) + tail, dtype=o_local.dtype, device=o_local.device)
        out[torch.as_tensor(list(shards[0]), dtype=torch.long, device=o_local.device)] = o_local
        return out
    rows = max(len(s) for s in shards)
    padded = torch.zeros((rows,) + tail, dtype=o_local.dtype, device=o_local.device)
    padded[: o_local.shape[0]] = o_local
    parts = [torch.empty_like(padded) for _ in range(world)]
    work = dist.all_gather(parts, padded.contiguous(), group=group, async_op=True)
    try:
        if timeout is None:
            work.wait()
        else:
            work.wait(timeout=datetime.timedelta(seconds=timeout))
    except Exception as e:  # noqa: BLE001 - every backend's timeout or peer-loss error
        raise RuntimeError(f"gather_outputs: not every rank joined the gather on rank {rank} "
                           f"({type(e).__name__}: {e})") from e
    if rank != dst:
        return None
    out = torch.empty((batch,) + tail, dtype=o_local.dtype, device=o_local.device)
    for r, idx in enumerate(shards):
        if idx:
            out[torch.as_tensor(list(idx), dtype=torch.long, device=o_local.device)] = parts[r][: len(idx)]
    return out
