"""Benchmark of the MXFP4 absorbed-MLA decode path on B200.

Workload (per GPU, weak scaling across GPUs): Kimi-K2 decode shape -- 64
heads, batch 64, every sequence 8192 tokens of paged MXFP4 latent (512) +
bf16 RoPE (64), page size 64, seeded random-permutation page table,
heads-first output, num_kv_splits automatic, sm_scale 1/sqrt(192).  Inputs
are synthetic (seeded normal q and latents; the cache is written by this
library's KV-append quantiser).  A step is one decode call over the whole
batch (one layer).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload kimi_k2|ragged|long|tp8_block|tp8_prologue|tp8_ar_norm|tp8_vup_oproj]

``--workload ragged`` runs the batch-sharded sweep instead: one batch of 256
sequences with lengths drawn uniformly from 1K-32K tokens (seeded), spread
over the N ranks by longest-first bin packing (kimi_b200.dp), each rank
holding only its sequences' pages; the whole batch is fixed as N grows
(strong scaling) and the gather of the outputs to rank 0 is timed separately.

``--workload long`` runs the long-context decode of the DeepSeek-V3 shape:
128 heads, batch 8, 131072 tokens every sequence, 32 splits into
preallocated partials, one token appended per sequence per step; it reports
the HBM fraction and the tensor-pipe fraction of the MMA work.

``--workload tp8_block`` times the whole TP8 decode attention block per GPU
(config 5): q absorption + RoPE + KV append, the decode (8 heads, 128
sequences of 4096 tokens), W_UV + o_proj, all-reduce + RMSNorm + MXFP4, as
one captured chain, in microseconds per layer, with each call's share.

``--workload tp8_prologue`` times the decode step before attention instead:
q absorption by W_UK + RoPE + MXFP4 KV append (kimi_b200.q_absorb_rope_append)
at the Kimi-K2 TP8 shape per GPU (8 heads, 128 tokens), in microseconds per
call, next to the same step as separate torch / library calls.
``--workload tp8_ar_norm`` times the layer-input step after the TP8
all-reduce (kimi_b200.tp: 8 partials + residual + RMSNorm + MXFP4): on one GPU
with 8 local buffers standing in for the ranks, under torchrun with every
rank's real buffer read over NVLink.
``--workload tp8_vup_oproj`` times the decode step after attention: the V
up-projection of the heads-first output by W_UV, then o_proj
(kimi_b200.v_up_proj_and_o_proj) at the Kimi-K2 TP8 shape per GPU (8 heads,
128 tokens, hidden 7168), next to the reference's torch.bmm + torch.mm path.

Prints one JSON line on rank 0.  ``value`` is the aggregate achieved HBM
bandwidth over all ranks computed from the algorithmic bytes (latent nibbles
+ e8m0 scales + RoPE of every token, plus q), divided by the max-over-ranks
device time of the K timed steps; ``ms_per_step`` is the per-layer time.
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "MLA decode µs/layer & achieved HBM TB/s (Kimi-K2, b64 ctx8K) at 1/2/4/8 B200"
HEADS, BATCH, CTX, PAGE = 64, 64, 8192, 64
SM_SCALE = 1.0 / math.sqrt(192.0)
# stage-1 kernel the library launches
STAGE1_KERNEL = "mla_decode_fp4_kernel"
# kernels of one stage-1 call: the fp4 kernel's Q operand prep kernel runs first
# (the decode kernel starts as its programmatic dependent and overlaps it)
STAGE1_LAUNCHES = ([STAGE1_KERNEL] if STAGE1_KERNEL != "mla_decode_fp4_kernel"
                   else ["q_prep_fp4_kernel", STAGE1_KERNEL])
TOKEN_BYTES_ALGO = 256 + 16 + 128  # nibbles + e8m0 scales + bf16 RoPE per token
FALLBACK_HBM_GBS = 6650.0
WORKLOAD = (f"Kimi-K2 MXFP4 MLA decode: {HEADS} heads, batch {BATCH} per GPU, ctx {CTX} every sequence, "
            f"page {PAGE}, seeded random-permutation page table, heads-first o, num_kv_splits auto")


def algorithmic_bytes(batch=BATCH, heads=HEADS, ctx=CTX) -> int:
    return batch * ctx * TOKEN_BYTES_ALGO + batch * heads * 576 * 2


def _peak_hbm():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def _traffic_summary():
    """ncu DRAM bytes per launch of the dominant kernel, from the committed
    profile summary (profiles/decode_traffic.json), or None."""
    path = os.path.join(ROOT, "profiles", "decode_traffic.json")
    try:
        with open(path) as f:
            return json.load(f)
    except Exception:
        return None


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while running."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
        0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
        0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
    }

    def __init__(self, device_index: int, period: float = 0.02):
        self.idx, self.period = device_index, period
        self.samples, self.reasons = [], set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nvml = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(self.idx)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nvml = None
            return self
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()
        return self

    def _run(self):
        n = self._nvml
        while not self._stop.is_set():
            try:
                self.samples.append(n.nvmlDeviceGetClockInfo(self._h, n.NVML_CLOCK_SM))
                mask = n.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                for bit, name in self.REASONS.items():
                    if mask & bit and bit != 0x1:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self.period)

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread:
            self._thread.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"], "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
RAGGED_BATCH, RAGGED_MIN, RAGGED_MAX, RAGGED_SEED = 256, 1024, 32768, 3
RAGGED_WORKLOAD = (f"batch-sharded MXFP4 MLA decode: {HEADS} heads, one batch of {RAGGED_BATCH} sequences, ctx "
                   f"uniform {RAGGED_MIN}-{RAGGED_MAX} (seed {RAGGED_SEED}), page {PAGE}, shuffled pages, "
                   f"longest-first bin packing over the ranks, num_kv_splits auto")


def ragged_lengths():
    import numpy as np
    rng = np.random.default_rng(RAGGED_SEED)
    return [int(x) for x in rng.integers(RAGGED_MIN, RAGGED_MAX + 1, RAGGED_BATCH)]


def build_ragged_workload(torch, kimi, dev, rank: int, world: int):
    """This rank's share of the ragged batch: its sequences' pages only."""
    from kimi_b200 import dp
    lens = ragged_lengths()
    shards = dp.shard_sequences(lens, world)
    mine = shards[rank]
    gen = torch.Generator(device=dev).manual_seed(RAGGED_SEED * 1000 + rank)
    local_lens = [lens[i] for i in mine]
    pages_per = [(n + PAGE - 1) // PAGE for n in local_lens]
    pages = max(sum(pages_per), 1)
    kvb, kvs = kimi.alloc_mxfp4_cache(pages, dev, zero=False)
    chunk = 1 << 16
    for start in range(0, pages * PAGE, chunk):
        n = min(chunk, pages * PAGE - start)
        kv_c = torch.randn(n, 512, generator=gen, device=dev).to(torch.bfloat16)
        k_pe = torch.randn(n, 64, generator=gen, device=dev).to(torch.bfloat16)
        kimi.mxfp4_kv_append(kv_c, k_pe, kvb, kvs, torch.arange(start, start + n, device=dev))
    perm = torch.randperm(pages, generator=gen, device=dev).to(torch.int32)
    indptr = torch.zeros(len(mine) + 1, dtype=torch.int32)
    indptr[1:] = torch.cumsum(torch.tensor(pages_per, dtype=torch.int32), 0) if mine else indptr[1:]
    last = torch.tensor([n - (p - 1) * PAGE for n, p in zip(local_lens, pages_per)], dtype=torch.int32)
    qgen = torch.Generator(device=dev).manual_seed(RAGGED_SEED)
    q_all = torch.randn(RAGGED_BATCH, HEADS, 576, generator=qgen, device=dev).to(torch.bfloat16)
    idx = torch.tensor(mine, dtype=torch.long, device=dev)
    q = q_all[idx].contiguous()
    o = torch.empty(len(mine), HEADS, 512, dtype=torch.bfloat16, device=dev)
    ws = kimi.alloc_workspace(max(len(mine), 1), HEADS, None, dev)
    tokens_local = sum(local_lens)
    return dict(kvb=kvb, kvs=kvs, perm=perm, indptr=indptr.to(dev), last=last.to(dev), q=q, o=o, ws=ws,
                shards=shards, lens=lens, batch=len(mine),
                bytes_local=tokens_local * TOKEN_BYTES_ALGO + len(mine) * HEADS * 576 * 2,
                bytes_total=sum(lens) * TOKEN_BYTES_ALGO + RAGGED_BATCH * HEADS * 576 * 2)


def build_workload(torch, kimi, dev, seed: int):
    gen = torch.Generator(device=dev).manual_seed(seed)
    pages = BATCH * CTX // PAGE
    kvb, kvs = kimi.alloc_mxfp4_cache(pages, dev, zero=False)
    chunk = 1 << 16
    for start in range(0, pages * PAGE, chunk):
        n = min(chunk, pages * PAGE - start)
        kv_c = torch.randn(n, 512, generator=gen, device=dev).to(torch.bfloat16)
        k_pe = torch.randn(n, 64, generator=gen, device=dev).to(torch.bfloat16)
        kimi.mxfp4_kv_append(kv_c, k_pe, kvb, kvs, torch.arange(start, start + n, device=dev))
    perm = torch.randperm(pages, generator=gen, device=dev).to(torch.int32)
    indptr = (torch.arange(BATCH + 1, device=dev, dtype=torch.int32) * (CTX // PAGE)).contiguous()
    last = torch.full((BATCH,), PAGE, dtype=torch.int32, device=dev)
    q = torch.randn(BATCH, HEADS, 576, generator=gen, device=dev).to(torch.bfloat16)
    o_hf = torch.empty(HEADS, BATCH, 512, dtype=torch.bfloat16, device=dev)
    ws = kimi.alloc_workspace(BATCH, HEADS, None, dev)
    return dict(kvb=kvb, kvs=kvs, perm=perm, indptr=indptr, last=last, q=q, o_hf=o_hf, o=o_hf.permute(1, 0, 2),
                ws=ws, batch=BATCH)


E2E_GROUP = 64  # pipelined end-to-end steps per captured graph
E2E_MIN_REPLAYS = 8  # the end-to-end figure always times at least this many graph replays


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    import kimi_b200 as kimi

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    ragged = args.workload == "ragged"
    if ragged:
        # one cache of ~1.7 GB / N per rank (far larger than the 126 MB L2)
        wl = [build_ragged_workload(torch, kimi, dev, rank, world)]
    else:
        # Two independent caches (2 x 210 MB > 126 MB L2), alternated step by step.
        wl = [build_workload(torch, kimi, dev, seed=1000 * rank + s) for s in (1, 2)]
    splits = kimi.num_kv_splits_for(wl[0]["batch"], HEADS, None)
    stream = torch.cuda.current_stream(dev)

    def step(i):
        w = wl[i % len(wl)]
        kimi.mla_decode_fwd(w["q"], w["kvb"], w["kvs"], w["o"], None, w["indptr"], w["perm"], w["last"],
                            sm_scale=SM_SCALE, workspace=w["ws"])

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()

    with ClockSampler(dev.index) as clocks:
        # ---- device-timed steps (inputs resident in HBM) ----
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(args.steps):
            step(i)
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        ms_total = max_over_ranks(e0.elapsed_time(e1))

        # ---- average launch durations: events around K back-to-back stage-1
        # calls (the caches alternate, so every launch reads from HBM), then
        # around K back-to-back merges of the last partials ----
        def calls(i):
            w = wl[i % len(wl)]
            return (w["q"], w["kvb"], w["kvs"], w["o"], None, w["indptr"], w["perm"], w["last"]), w["ws"]

        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        ev[0].record(stream)
        for i in range(args.steps):
            call, ws = calls(i)
            kimi.mla_decode_partial(*call, sm_scale=SM_SCALE, workspace=ws)
        ev[1].record(stream)
        for i in range(args.steps):
            call, ws = calls(args.steps - 1)
            kimi.mla_decode_merge(*call, sm_scale=SM_SCALE, workspace=ws)
        ev[2].record(stream)
        torch.cuda.synchronize()
        stage1_ms = [ev[0].elapsed_time(ev[1]) / args.steps]
        merge_ms = [ev[1].elapsed_time(ev[2]) / args.steps]

        # ---- end to end through the public API with host buffers ----
        q_host = [torch.empty_like(w["q"], device="cpu").pin_memory() for w in wl]
        for qh, w in zip(q_host, wl):
            qh.copy_(w["q"].cpu())
        meta_host = [(w["indptr"].cpu().pin_memory(), w["perm"].cpu().pin_memory(), w["last"].cpu().pin_memory())
                     for w in wl]
        o_host = [torch.empty(w["batch"], HEADS, 512, dtype=torch.bfloat16).pin_memory() for w in wl]
        dev_meta = [(torch.empty_like(w["indptr"]), torch.empty_like(w["perm"]), torch.empty_like(w["last"]))
                    for w in wl]
        h2d = q_host[0].numel() * 2 + sum(t.numel() * 4 for t in meta_host[0])
        d2h = o_host[0].numel() * 2
        # A serving loop's overlap: step i + 1's inputs go up on one copy
        # stream and step i - 1's output comes back on another while step i
        # decodes.  The two workloads' device buffers are the double buffers;
        # events order every reuse (inputs are overwritten only after the
        # decode two steps back has read them, outputs only after their copy
        # to the host).  Every step still copies its own inputs in and its own
        # output out inside the timed region.
        # The pipelined steps are captured into a CUDA graph of E2E_GROUP steps
        # and replayed, as a serving loop replays its captured decode step:
        # the host's per-step enqueue (about ten calls) would otherwise set
        # the pace.  Replays run back to back, so the pipeline drains once
        # per group.
        s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        nbuf = len(wl)
        group = E2E_GROUP
        h2d_done = [torch.cuda.Event() for _ in range(group)]
        dec_done = [torch.cuda.Event() for _ in range(group)]
        d2h_done = [torch.cuda.Event() for _ in range(group)]

        def enqueue_group(cs):
            s_in.wait_stream(cs)
            s_out.wait_stream(cs)
            for i in range(group):
                k = i % nbuf
                w, (ip_h, px_h, la_h), (ip_d, px_d, la_d) = wl[k], meta_host[k], dev_meta[k]
                with torch.cuda.stream(s_in):
                    if i >= nbuf:
                        s_in.wait_event(dec_done[i - nbuf])
                    w["q"].copy_(q_host[k], non_blocking=True)
                    ip_d.copy_(ip_h, non_blocking=True)
                    px_d.copy_(px_h, non_blocking=True)
                    la_d.copy_(la_h, non_blocking=True)
                    h2d_done[i].record(s_in)
                cs.wait_event(h2d_done[i])
                if i >= nbuf:
                    cs.wait_event(d2h_done[i - nbuf])
                with torch.cuda.stream(cs):
                    kimi.mla_decode_fwd(w["q"], w["kvb"], w["kvs"], w["o"], None, ip_d, px_d, la_d,
                                        sm_scale=SM_SCALE, workspace=w["ws"])
                dec_done[i].record(cs)
                with torch.cuda.stream(s_out):
                    s_out.wait_event(dec_done[i])
                    o_host[k].copy_(w["o"], non_blocking=True)
                    d2h_done[i].record(s_out)
            cs.wait_stream(s_in)
            cs.wait_stream(s_out)

        enqueue_group(stream)  # eager once: the same work, outside the graph
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            enqueue_group(torch.cuda.current_stream())
        torch.cuda.synchronize()
        reps = max(E2E_MIN_REPLAYS, args.steps // group)
        graph.replay()
        torch.cuda.synchronize()
        barrier()
        e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e2.record(stream)
        for _ in range(reps):
            graph.replay()
        e3.record(stream)
        torch.cuda.synchronize()
        barrier()
        e2e_steps = reps * group
        e2e_ms = max_over_ranks(e2.elapsed_time(e3)) * args.steps / e2e_steps  # per step, scaled to K steps
        del graph
        # the host copies hold the last steps' outputs
        for k in range(nbuf):
            if not torch.equal(o_host[k], wl[k]["o"].cpu()):
                raise RuntimeError("end-to-end output on the host differs from the device result")

    # the gather of the outputs to rank 0 (ragged workload), timed on its own
    gather_ms = None
    if ragged:
        from kimi_b200 import dp
        w = wl[0]
        for _ in range(3):
            dp.gather_outputs(w["o"], w["shards"], rank, world, batch=RAGGED_BATCH)
        torch.cuda.synchronize()
        barrier()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 20
        g0.record(stream)
        for _ in range(reps):
            dp.gather_outputs(w["o"], w["shards"], rank, world, batch=RAGGED_BATCH)
        g1.record(stream)
        torch.cuda.synchronize()
        gather_ms = max_over_ranks(g0.elapsed_time(g1) / reps)
    nbytes = wl[0]["bytes_local"] if ragged else algorithmic_bytes()
    nbytes_job = wl[0]["bytes_total"] if ragged else world * nbytes
    ms_step = ms_total / args.steps
    stage1_avg = sum(stage1_ms) / len(stage1_ms)
    red_ms = sum(merge_ms) / len(merge_ms)
    value_tbs = nbytes_job / (ms_step * 1e-3) / 1e12
    e2e_tbs = nbytes_job / (e2e_ms / args.steps * 1e-3) / 1e12
    peak, peak_kind = _peak_hbm()
    achieved_gbs = nbytes / (stage1_avg * 1e-3) / 1e9
    traffic = None if ragged else _traffic_summary()  # the committed capture is of the kimi_k2 workload
    clk = clocks.summary()
    if rank != 0:
        return None
    cpu = cpu_baseline_sample(args.cpu_baseline_seconds) if (world == 1 and args.cpu_baseline_seconds > 0
                                                                 and not ragged) else None
    line = {
        "metric": METRIC, "value": round(value_tbs, 4), "unit": "TB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 5), "us_per_layer": round(ms_step * 1e3, 2),
        "higher_is_better": True, "scaling": "strong" if ragged else "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded normal q and latents, cache written by the library's MXFP4 KV-append)",
        "config": ({"workload": RAGGED_WORKLOAD, "heads": HEADS, "batch_total": RAGGED_BATCH,
                    "batch_this_rank": wl[0]["batch"], "tokens_total": sum(wl[0]["lens"]), "page_size": PAGE,
                    "num_kv_splits": f"auto (balanced schedule over {splits} CTAs)", "sm_scale": "1/sqrt(192)",
                    "algorithmic_bytes_per_job_step": nbytes_job,
                    "l2": "inputs larger than L2: one ~1.7 GB / N cache per rank",
                    "parallelism": f"dp{world} (sequences bin-packed over ranks; outputs gathered to rank 0 "
                                   "outside the timed steps)",
                    "gather_ms": None if gather_ms is None else round(gather_ms, 5)}
                   if ragged else
                   {"workload": WORKLOAD, "heads": HEADS, "batch_per_gpu": BATCH, "ctx": CTX, "page_size": PAGE,
                    "num_kv_splits": f"auto (balanced schedule over {splits} CTAs)", "sm_scale": "1/sqrt(192)",
                    "algorithmic_bytes_per_gpu_step": nbytes,
                    "l2": "inputs larger than L2: two independent 210 MB caches alternated between steps",
                    "parallelism": f"dp{world} (batch-sharded, no collective in the step)"}),
        "e2e": {"value": round(e2e_tbs, 4), "unit": "TB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": round(e2e_ms / args.steps, 5), "steps_timed": e2e_steps,
                "path": "kimi_b200.mla_decode_fwd with q + page table copied from pinned host memory and o "
                        "copied back every step, the copies on two copy streams overlapping the neighbouring "
                        "steps' decode (double-buffered, event-ordered), groups of %d steps captured in a "
                        "CUDA graph and replayed" % E2E_GROUP},
        "gpu_launches": args.steps * (len(STAGE1_LAUNCHES) + 1),
        "kernels": {"stage1_ms": round(stage1_avg, 5), "merge_ms": round(red_ms, 5),
                    "launches_per_step": STAGE1_LAUNCHES + ["mla_reduce_kernel"]},
        "roofline": {"bound": "hbm", "achieved": round(achieved_gbs, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved_gbs / peak, 4), "peak_kind": f"{peak_kind} (MEASURED_PEAKS hbm_gbs)"
                     if peak_kind == "measured" else "fallback",
                     "kernel": "mla_decode stage 1 (split-K partial attention"
                               + (", with its Q operand prep kernel)" if len(STAGE1_LAUNCHES) > 1 else ")"),
                     "traffic": None if traffic is None else traffic.get("dram_bytes_per_launch"),
                     "traffic_source": None if traffic is None else traffic.get("source")},
        "clocks": clk,
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    return line


# ---------------------------------------------------------------------------
# CPU baseline / reference arm: the oracle port of the reference torch path
# ---------------------------------------------------------------------------
def _cpu_sample_case(tokens: int, seed: int = 7):
    import numpy as np

    from oracle import mla as omla
    from oracle import mxfp4 as omx
    rng = np.random.default_rng(seed)
    pages = tokens // PAGE
    kv_c = omx.f32_to_bf16_bits(rng.standard_normal((pages * PAGE, 512), dtype=np.float32))
    k_pe = omx.f32_to_bf16_bits(rng.standard_normal((pages * PAGE, 64), dtype=np.float32))
    kvb, kvs = omla.empty_cache(pages)
    omla.kv_append(kvb, kvs, kv_c, k_pe, np.arange(pages * PAGE))
    q = omx.f32_to_bf16_bits(rng.standard_normal((1, HEADS, 576), dtype=np.float32))
    return dict(q=q, kvb=kvb, kvs=kvs, indptr=np.array([0, pages], np.int32),
                indices=rng.permutation(pages).astype(np.int32), last=np.array([PAGE], np.int32))


def _cpu_decode(case):
    from oracle import mla as omla
    return omla.mla_decode(case["q"], case["kvb"], case["kvs"], case["indptr"], case["indices"], case["last"],
                           SM_SCALE)


# The oracle runs one whole sequence per task in worker processes (started
# with spawn, one per host core, each with one BLAS thread), so a step uses
# every core the box has.
_WORKER_CASE = None


def _cpu_worker_init(tokens: int):
    global _WORKER_CASE
    _WORKER_CASE = _cpu_sample_case(tokens)


def _cpu_worker_run(_):
    t0 = time.perf_counter()
    _cpu_decode(_WORKER_CASE)
    return time.perf_counter() - t0


def _cpu_pool(workers: int):
    import concurrent.futures
    import multiprocessing as mp
    env = {k: "1" for k in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS")}
    saved = {k: os.environ.get(k) for k in env}
    os.environ.update(env)  # inherited by the spawned workers
    try:
        pool = concurrent.futures.ProcessPoolExecutor(max_workers=workers, mp_context=mp.get_context("spawn"),
                                                      initializer=_cpu_worker_init, initargs=(CTX,))
        list(pool.map(_cpu_worker_run, range(workers)))  # start every worker and warm it up
    finally:
        for k, v in saved.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
    return pool


def _cpu_steps(pool, workers: int, steps: int):
    """Time `steps` steps of `workers` whole sequences each (one per worker)."""
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        list(pool.map(_cpu_worker_run, range(workers)))
        times.append(time.perf_counter() - t0)
    return times


def cpu_baseline_sample(target_s: float = 10.0):
    """Time the oracle port of the reference's torch path on all host cores:
    steps of one whole 8192-token, 64-head sequence per core, for about
    ``target_s`` seconds."""
    workers = os.cpu_count() or 1
    pool = _cpu_pool(workers)
    try:
        times = []
        while sum(times) < target_s:
            times += _cpu_steps(pool, workers, 1)
    finally:
        pool.shutdown()
    dt, n = sum(times), len(times) * workers
    nbytes = n * algorithmic_bytes(batch=1)
    return {"value": round(nbytes / dt / 1e12, 6), "unit": "TB/s", "cores": workers, "kind": "port",
            "sample": f"{n} sequences of {CTX} tokens x {HEADS} heads, {workers} worker processes (one per core, "
                      f"one BLAS thread each) running the numpy oracle of the reference torch path (e2m1/e8m0 "
                      f"dequant + fp32 attention), {dt:.1f} s",
            "us_per_layer_equiv": round(dt / n * BATCH * 1e6, 1)}


def run_reference(args, rank):
    """The reference arm: the reference's CPU path for this decode (its torch
    dequantise-then-fp32 attention, here the numpy oracle that restates it:
    the reference is scripts with no installable package, and nothing of it
    compiles) on the box's host cores.  One step = one whole 8192-token,
    64-head sequence per core, so ms_per_step is measured, not extrapolated;
    the time the host would need for the full 64-sequence batch is reported
    apart as ms_per_batch_equiv."""
    if rank != 0:
        return None
    workers = os.cpu_count() or 1
    pool = _cpu_pool(workers)
    try:
        _cpu_steps(pool, workers, max(args.warmup, 1))
        times = _cpu_steps(pool, workers, args.steps)
    finally:
        pool.shutdown()
    dt = sum(times)
    nbytes_step = workers * algorithmic_bytes(batch=1)
    val = nbytes_step * args.steps / dt / 1e12
    ms_step = dt / args.steps * 1e3
    return {
        "impl": "reference", "metric": METRIC, "value": round(val, 6), "unit": "TB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 3),
        "ms_per_batch_equiv": round(ms_step * BATCH / workers, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded normal q and latents)",
        "config": {"workload": WORKLOAD, "heads": HEADS, "batch_per_gpu": BATCH, "ctx": CTX, "page_size": PAGE,
                   "step_sample": f"{workers} whole sequences ({CTX} tokens x {HEADS} heads), one per host core",
                   "parallelism": f"{workers} worker processes"},
        "cpu_baseline": {"value": round(val, 6), "unit": "TB/s", "cores": workers, "kind": "port",
                         "sample": f"{args.steps} steps x {workers} sequences of {CTX} tokens x {HEADS} heads "
                                   "through the numpy oracle of the reference torch path"},
        "e2e": {"value": round(val, 6), "unit": "TB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# ---------------------------------------------------------------------------
# the decode prologue (q absorb + RoPE + MXFP4 KV append), Kimi-K2 TP8 shape
# ---------------------------------------------------------------------------
PRO_TOKENS, PRO_HEADS, PRO_MAXPOS, PRO_SETS = 128, 8, 8192, 64


def prologue_bytes(T=PRO_TOKENS, H=PRO_HEADS) -> int:
    """Algorithmic bytes of one call: q (nope + pe), W_UK, kv_c + k_pe,
    positions / slots, the cos / sin rows, q_out and the cache rows written."""
    return (T * H * 192 * 2 + H * 128 * 512 * 2 + T * 576 * 2 + T * 16 + T * 2 * 32 * 4
            + T * H * 576 * 2 + T * 400)


def run_prologue(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    import kimi_b200 as kimi

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    T, H = PRO_TOKENS, PRO_HEADS
    g = torch.Generator(device=dev).manual_seed(5 + 1000 * rank)
    bf = torch.bfloat16
    freqs = 1.0 / (10000.0 ** (torch.arange(32, device=dev, dtype=torch.float64) / 32.0))
    ang = torch.arange(PRO_MAXPOS, device=dev, dtype=torch.float64)[:, None] * freqs[None, :]
    cos, sin = ang.cos().float().contiguous(), ang.sin().float().contiguous()
    kvb, kvs = kimi.alloc_mxfp4_cache(PRO_SETS * T // 64, dev)
    # PRO_SETS independent call inputs (~180 MB in all, more than the 126 MB L2), used in turn
    sets = []
    for i in range(PRO_SETS):
        sets.append(dict(
            q=torch.randn(T, H, 192, generator=g, device=dev).to(bf),
            w=(torch.randn(H, 128, 512, generator=g, device=dev) / math.sqrt(128.0)).to(bf),
            kv_c=torch.randn(T, 512, generator=g, device=dev).to(bf),
            k_pe=torch.randn(T, 64, generator=g, device=dev).to(bf),
            pos=torch.randint(0, PRO_MAXPOS, (T,), generator=g, device=dev),
            slots=torch.arange(i * T, (i + 1) * T, device=dev, dtype=torch.int64),
            out=torch.empty(T, H, 576, dtype=bf, device=dev)))

    def fused(i):
        s_ = sets[i % PRO_SETS]
        kimi.q_absorb_rope_append(s_["q"][:, :, :128], s_["q"][:, :, 128:], s_["w"], s_["kv_c"], s_["k_pe"],
                                  s_["pos"], cos, sin, kvb, kvs, s_["slots"], q_out=s_["out"])

    def rope_torch(x, pos):  # (x[2i], x[2i+1]) pairs, float32
        c, sn = cos[pos], sin[pos]
        while c.dim() < x.dim():
            c, sn = c.unsqueeze(-2), sn.unsqueeze(-2)
        xf = x.float()
        a, b = xf[..., 0::2], xf[..., 1::2]
        return torch.stack((a * c - b * sn, b * c + a * sn), dim=-1).flatten(-2).to(bf)

    def unfused(i):  # the same step as separate library / torch calls
        s_ = sets[i % PRO_SETS]
        out = s_["out"]
        out[:, :, :512] = torch.bmm(s_["q"][:, :, :128].transpose(0, 1), s_["w"]).transpose(0, 1)
        out[:, :, 512:] = rope_torch(s_["q"][:, :, 128:], s_["pos"])
        kimi.mxfp4_kv_append(s_["kv_c"], rope_torch(s_["k_pe"], s_["pos"]), kvb, kvs, s_["slots"])

    stream = torch.cuda.current_stream(dev)

    def timed(fn):
        # Both paths are captured into a CUDA graph of PRO_SETS calls and the
        # graph is replayed: the host's per-call Python and launch overhead
        # (tens of microseconds) would otherwise set the pace, not the GPU.
        for i in range(args.warmup):
            fn(i)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(PRO_SETS):
                fn(i)
        reps = max(1, args.steps // PRO_SETS)
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier(device_ids=[local_rank])
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / (reps * PRO_SETS)
        del graph
        if world > 1:
            t = torch.tensor([ms], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    with ClockSampler(dev.index) as clocks:
        ms = timed(fused)
    ms_unfused = timed(unfused)
    if rank != 0:
        return None
    peak, peak_kind = _peak_hbm()
    nbytes = prologue_bytes()
    achieved = nbytes / (ms * 1e-3) / 1e9
    return {
        "metric": "decode prologue latency (q absorb by W_UK + RoPE + MXFP4 KV append), Kimi-K2 TP8 per GPU",
        "value": round(ms * 1e3, 3), "unit": "us", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 6), "higher_is_better": False, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (seeded normal q, W_UK ~ N(0, 1/128), latents; random positions)",
        "config": {"workload": f"Kimi-K2 TP8 decode prologue: {H} heads per GPU, {T} tokens, W_UK [{H}, 128, 512], "
                               f"RoPE table {PRO_MAXPOS} positions (GPT-J pairing), cache page 64",
                   "l2": f"inputs larger than L2: {PRO_SETS} independent input sets used in turn",
                   "parallelism": f"{world} replica(s), one per GPU, no collective"},
        "gpu_launches": max(1, args.steps // PRO_SETS) * PRO_SETS,
        "timing": "CUDA graph of 64 calls replayed; device time per call",
        "unfused_us": round(ms_unfused * 1e3, 3),
        "unfused_path": "torch.bmm + torch RoPE + kimi_b200.mxfp4_kv_append (same results, several launches)",
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": None,
                     "note": f"{nbytes} algorithmic bytes per call; launch- and latency-bound at this size"},
        "clocks": clocks.summary(),
    }


# ---------------------------------------------------------------------------
# the layer-input step after the TP8 all-reduce: sum of 8 partials + residual +
# RMSNorm + MXFP4, Kimi-K2 hidden 7168, 128 tokens
# ---------------------------------------------------------------------------
AR_ROWS, AR_HIDDEN, AR_RANKS, AR_SETS = 128, 7168, 8, 8


def run_ar_norm(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    import kimi_b200 as kimi
    from kimi_b200 import tp

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(9 + rank)
    bf = torch.bfloat16
    rows, hidden = AR_ROWS, AR_HIDDEN
    weight = torch.randn(hidden, generator=g, device=dev).to(bf)
    if world > 1:
        # the ranks' real partial buffers, read over NVLink
        peers = tp.PeerPartials(rows, hidden, dev)
        peers.local.copy_(torch.randn(rows, hidden, generator=g, device=dev).to(bf))
        torch.cuda.synchronize()
        dist.barrier(device_ids=[local_rank])  # every rank's partial is written before any rank reads it
        sets = [dict(inputs=peers.ptrs, res=torch.randn(rows, hidden, generator=g, device=dev).to(bf))
                for _ in range(AR_SETS)]
        ranks = world
    else:
        # one GPU: the 8 ranks' partials as 8 local buffers per input set (the same
        # bytes per call, from HBM instead of over NVLink)
        sets = [dict(inputs=[torch.randn(rows, hidden, generator=g, device=dev).to(bf) for _ in range(AR_RANKS)],
                     res=torch.randn(rows, hidden, generator=g, device=dev).to(bf)) for _ in range(AR_SETS)]
        ranks = AR_RANKS
    outs = [dict(r=torch.empty(rows, hidden, dtype=bf, device=dev),
                 n=torch.empty(rows, hidden // 2, dtype=torch.uint8, device=dev),
                 s=torch.empty(rows, hidden // 32, dtype=torch.uint8, device=dev)) for _ in range(AR_SETS)]

    def fused(i):
        st, o = sets[i % AR_SETS], outs[i % AR_SETS]
        tp.ar_rmsnorm_mxfp4(st["inputs"], st["res"], weight, 1e-6, residual_out=o["r"], nibbles=o["n"], scales=o["s"])

    def unfused(i):  # the same arithmetic as separate torch / library calls (the all-reduce as a sum on one GPU)
        st = sets[i % AR_SETS]
        acc = st["inputs"][0].float()
        for x in st["inputs"][1:]:
            acc = acc + x.float()
        comb = (acc + st["res"].float()).to(bf)
        normed = (comb.float() * torch.rsqrt(comb.float().pow(2).mean(-1, keepdim=True) + 1e-6)).to(bf) * weight
        kimi.mxfp4_quantize(normed)

    stream = torch.cuda.current_stream(dev)

    def timed(fn, graphed):
        for i in range(args.warmup):
            fn(i)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier(device_ids=[local_rank])
        if graphed:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for i in range(AR_SETS):
                    fn(i)
            run = graph.replay
            per = AR_SETS
        else:
            run, per = (lambda: fn(0)), 1
        reps = max(1, args.steps // per)
        run()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            run()
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / (reps * per)
        if world > 1:
            t = torch.tensor([ms], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    # with peers the kernel runs between the callers' barriers; only the kernel is timed here
    with ClockSampler(dev.index) as clocks:
        ms = timed(fused, graphed=True)
    ms_unfused = timed(unfused, graphed=True) if world == 1 else None
    if world > 1:
        peers.close()
    if rank != 0:
        return None
    peak, peak_kind = _peak_hbm()
    nbytes = rows * hidden * 2 * (ranks + 2) + rows * hidden // 2 + rows * hidden // 32 + hidden * 2
    # with peers the bound is the bytes that cross NVLink into this GPU (the
    # other ranks' partials) at the measured 770 GB/s peer-copy rate per direction
    link_bytes = rows * hidden * 2 * (ranks - 1)
    achieved = (nbytes if world == 1 else link_bytes) / (ms * 1e-3) / 1e9
    line = {
        "metric": "TP8 layer-input step (all-reduce of 8 partials + residual + RMSNorm + MXFP4), Kimi-K2 hidden 7168",
        "value": round(ms * 1e3, 3), "unit": "us", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 6), "higher_is_better": False, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (seeded normal partials, residual and weight)",
        "config": {"workload": f"{rows} tokens x hidden {hidden}, {ranks} partials summed, eps 1e-6, "
                               "MXFP4 inline rule, unshuffled scales",
                   "partials": "peer buffers over NVLink" if world > 1 else
                               f"{AR_RANKS} local buffers standing in for the {AR_RANKS} ranks",
                   "l2": f"{AR_SETS} input sets used in turn",
                   "timing": "CUDA graph of the kernel calls replayed; device time per call"},
        "gpu_launches": max(1, args.steps // AR_SETS) * AR_SETS,
        "roofline": {"bound": "hbm" if world == 1 else "nvlink", "achieved": round(achieved, 1),
                     "peak": peak if world == 1 else 770.0,
                     "unit": "GB/s", "frac": None, "traffic": None,
                     "note": f"{nbytes} algorithmic bytes per call" if world == 1 else
                             f"{link_bytes} bytes over NVLink into this GPU per call ({nbytes} in all); "
                             "peak = measured peer copy per direction"},
        "clocks": clocks.summary(),
    }
    line["roofline"]["frac"] = round(achieved / line["roofline"]["peak"], 4)
    if ms_unfused is not None:
        line["unfused_us"] = round(ms_unfused * 1e3, 3)
        line["unfused_path"] = "torch sum + add + RMSNorm + kimi_b200.mxfp4_quantize (same arithmetic)"
    return line


# ---------------------------------------------------------------------------
# the decode step after attention at the Kimi-K2 TP8 shape per GPU: W_UV BMM of
# the heads-first output, then o_proj [1024 -> 7168]
# ---------------------------------------------------------------------------
VU_TOKENS, VU_HEADS, VU_HIDDEN, VU_SETS = 128, 8, 7168, 8


def run_vup(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    import kimi_b200 as kimi

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    T, H, D = VU_TOKENS, VU_HEADS, VU_HIDDEN
    g = torch.Generator(device=dev).manual_seed(17 + 1000 * rank)
    bf = torch.bfloat16
    # VU_SETS independent layers' inputs and weights (~148 MB, more than the 126 MB L2), used in turn
    sets = [dict(o=torch.randn(16, T, 512, generator=g, device=dev).to(bf)[:H],  # heads-first, 16 padded heads
                 w_uv=(torch.randn(H, 512, 128, generator=g, device=dev) * 0.02).to(bf),
                 w_o=(torch.randn(D, H * 128, generator=g, device=dev) * 0.02).to(bf),
                 x=torch.empty(T, H * 128, dtype=bf, device=dev),
                 out=torch.empty(T, D, dtype=bf, device=dev)) for _ in range(VU_SETS)]

    def fused(i):
        s_ = sets[i % VU_SETS]
        kimi.v_up_proj_and_o_proj(s_["o"], s_["w_uv"], s_["w_o"], out=s_["out"], x=s_["x"])

    def unfused(i):  # the reference's path: fp32 BMM, bf16 round, transpose, bf16 mm (cuBLAS)
        s_ = sets[i % VU_SETS]
        x = torch.bmm(s_["o"].float(), s_["w_uv"].float()).to(bf).transpose(0, 1).reshape(T, H * 128)
        torch.mm(x, s_["w_o"].T, out=s_["out"])

    stream = torch.cuda.current_stream(dev)

    def timed(fn):
        for i in range(args.warmup):
            fn(i)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(VU_SETS):
                fn(i)
        reps = max(1, args.steps // VU_SETS)
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier(device_ids=[local_rank])
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / (reps * VU_SETS)
        del graph
        if world > 1:
            t = torch.tensor([ms], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    with ClockSampler(dev.index) as clocks:
        ms = timed(fused)
    ms_unfused = timed(unfused)
    if rank != 0:
        return None
    peak, peak_kind = _peak_hbm()
    # o + W_UV + W_o read, out written (the x scratch round trip stays in L2)
    nbytes = (H * T * 512 + H * 512 * 128 + D * H * 128 + T * D) * 2
    achieved = nbytes / (ms * 1e-3) / 1e9
    flops = 2 * T * (H * 512 * 128 + H * 128 * D)
    return {
        "metric": "decode epilogue latency (V up-projection by W_UV + o_proj), Kimi-K2 TP8 per GPU",
        "value": round(ms * 1e3, 3), "unit": "us", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 6), "higher_is_better": False, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (seeded normal heads-first o, W_UV and W_o ~ N(0, 0.02))",
        "config": {"workload": f"Kimi-K2 TP8 decode epilogue: {H} heads per GPU sliced from 16 padded, {T} tokens, "
                               f"W_UV [{H}, 512, 128], o_proj [{H * 128} -> {D}]",
                   "l2": f"inputs larger than L2: {VU_SETS} independent layers' inputs and weights used in turn",
                   "parallelism": f"{world} replica(s), one per GPU, no collective"},
        "gpu_launches": max(1, args.steps // VU_SETS) * VU_SETS * 2,
        "timing": f"CUDA graph of {VU_SETS} calls (two launches each) replayed; device time per call",
        "unfused_us": round(ms_unfused * 1e3, 3),
        "unfused_path": "torch.bmm (fp32) + bf16 round + transpose + torch.mm (the reference's path)",
        "tflops": round(flops / (ms * 1e-3) / 1e12, 1),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": None,
                     "note": f"{nbytes} algorithmic bytes per call ({flops} FLOPs: far below the tensor roofline)"},
        "clocks": clocks.summary(),
    }


BLK_TOKENS, BLK_HEADS, BLK_CTX, BLK_HIDDEN, BLK_STEPS_PER_GRAPH = 128, 8, 4096, 7168, 8
BLK_WORKLOAD = (f"Kimi-K2 TP8 decode attention block per GPU: {BLK_TOKENS} decode tokens (one per sequence, "
                f"ctx {BLK_CTX}), {BLK_HEADS} heads, hidden {BLK_HIDDEN}: q absorption by W_UK + RoPE + KV "
                f"append, MXFP4 MLA decode (num_kv_splits auto), W_UV + o_proj [1024 -> 7168], all-reduce of "
                f"the ranks' partials + residual + RMSNorm (eps 1e-6) + MXFP4; weights N(0, 0.02)")


def run_block(args, rank, world, local_rank):
    """The TP8 attention block per GPU as one chain of the library's four
    calls, captured in a CUDA graph and replayed (the per-call host overhead
    would otherwise set the pace).  On one GPU, 8 local buffers stand in for
    the ranks' partials (the one-shot kernel reads them all); under torchrun
    each rank's real partial is exchanged over NVLink with the two-shot call
    (its barriers are on the device, so the whole chain captures)."""
    import torch
    import torch.distributed as dist

    import kimi_b200 as kimi
    from kimi_b200 import tp

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    T, H, C, D = BLK_TOKENS, BLK_HEADS, BLK_CTX, BLK_HIDDEN
    bf = torch.bfloat16
    g = torch.Generator(device=dev).manual_seed(23 + 1000 * rank)
    freqs = 1.0 / (10000.0 ** (torch.arange(32, device=dev, dtype=torch.float64) / 32.0))
    ang = torch.arange(C, device=dev, dtype=torch.float64)[:, None] * freqs[None, :]
    cos, sin = ang.cos().float().contiguous(), ang.sin().float().contiguous()
    pages = T * C // PAGE
    kvb, kvs = kimi.alloc_mxfp4_cache(pages, dev, zero=False)
    for start in range(0, pages * PAGE, 1 << 16):
        n = min(1 << 16, pages * PAGE - start)
        kimi.mxfp4_kv_append(torch.randn(n, 512, generator=g, device=dev).to(bf),
                             torch.randn(n, 64, generator=g, device=dev).to(bf), kvb, kvs,
                             torch.arange(start, start + n, device=dev))
    perm = torch.randperm(pages, generator=g, device=dev).to(torch.int32)
    indptr = (torch.arange(T + 1, device=dev, dtype=torch.int32) * (C // PAGE)).contiguous()
    last = torch.full((T,), PAGE, dtype=torch.int32, device=dev)
    slots = (perm[indptr[1:].long() - 1].long() * PAGE + (PAGE - 1)).contiguous()  # each sequence's newest token
    positions = torch.full((T,), C - 1, dtype=torch.int64, device=dev)
    q = torch.randn(T, H, 192, generator=g, device=dev).to(bf)
    w_uk = (torch.randn(H, 128, 512, generator=g, device=dev) * 0.02).to(bf)
    w_uv = (torch.randn(H, 512, 128, generator=g, device=dev) * 0.02).to(bf)
    w_o = (torch.randn(D, H * 128, generator=g, device=dev) * 0.02).to(bf)
    kv_c = torch.randn(T, 512, generator=g, device=dev).to(bf)
    k_pe = torch.randn(T, 64, generator=g, device=dev).to(bf)
    residual = torch.randn(T, D, generator=g, device=dev).to(bf)
    norm_w = torch.randn(D, generator=g, device=dev).to(bf)
    q_out = torch.empty(T, H, 576, dtype=bf, device=dev)
    o_hf = torch.empty(H, T, 512, dtype=bf, device=dev)
    x = torch.empty(T, H * 128, dtype=bf, device=dev)
    ws = kimi.alloc_workspace(T, H, None, dev)
    if world > 1:
        peers = tp.PeerPartials(T, D, dev)
        partial = peers.local
    else:
        partial = torch.empty(T, D, dtype=bf, device=dev)
        others = [torch.randn(T, D, generator=g, device=dev).to(bf) for _ in range(7)]
        res_out = torch.empty_like(residual)
        nib = torch.empty(T, D // 2, dtype=torch.uint8, device=dev)
        sc = torch.empty(T, D // 32, dtype=torch.uint8, device=dev)

    def prologue():
        kimi.q_absorb_rope_append(q[:, :, :128], q[:, :, 128:], w_uk, kv_c, k_pe, positions, cos, sin, kvb, kvs,
                                  slots, q_out=q_out)

    def decode():
        kimi.mla_decode_fwd(q_out, kvb, kvs, o_hf.permute(1, 0, 2), None, indptr, perm, last, sm_scale=SM_SCALE,
                            workspace=ws)

    def epilogue():
        kimi.v_up_proj_and_o_proj(o_hf, w_uv, w_o, out=partial, x=x)

    def allreduce():
        if world > 1:
            peers.reduce_norm_quant_two_shot(residual, norm_w, 1e-6)
        else:
            tp.ar_rmsnorm_mxfp4([partial] + others, residual, norm_w, 1e-6, residual_out=res_out, nibbles=nib,
                                scales=sc)

    def block():
        prologue()
        decode()
        epilogue()
        allreduce()

    stream = torch.cuda.current_stream(dev)

    def graph_us(fn, reps):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(BLK_STEPS_PER_GRAPH):
                fn()
        graph.replay()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier(device_ids=[local_rank])
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (reps * BLK_STEPS_PER_GRAPH)
        del graph
        if world > 1:
            t = torch.tensor([us], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            us = float(t.item())
        return us

    reps = max(1, args.steps // BLK_STEPS_PER_GRAPH)
    with ClockSampler(dev.index) as clocks:
        us_block = graph_us(block, reps)
        parts = {name: round(graph_us(fn, reps), 2) for name, fn in
                 (("prologue", prologue), ("decode", decode), ("v_up_o_proj", epilogue), ("allreduce_norm_quant", allreduce))}
    status = 0
    if world > 1:
        status = kimi.device_status(peers.status)
        peers.close()
    if rank != 0:
        return None
    return {
        "metric": "TP8 decode attention block µs/layer per GPU (Kimi-K2, 128 tokens, ctx 4096, hidden 7168)",
        "value": round(us_block, 2), "unit": "us", "n_gpus": world, "steps": reps * BLK_STEPS_PER_GRAPH,
        "warmup": args.warmup, "ms_per_step": round(us_block / 1e3, 5), "higher_is_better": False,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded normal activations, N(0, 0.02) weights, cache written by the library's MXFP4 "
                "KV-append)",
        "config": {"workload": BLK_WORKLOAD, "tokens": T, "heads_per_gpu": H, "ctx": C, "hidden": D,
                   "allreduce": ("two-shot over NVLink, device barriers" if world > 1 else
                                 "one-shot over 8 local buffers standing in for the ranks' partials"),
                   "parallelism": f"tp{world}" if world > 1 else "tp8 block on one GPU (8 stand-in partials)",
                   "graph": f"{BLK_STEPS_PER_GRAPH} blocks per captured graph, {reps} replays"},
        "parts_us": parts, "gpu_launches": reps * BLK_STEPS_PER_GRAPH * 8,
        "peer_status": status, "clocks": clocks.summary(),
    }


LONG_HEADS, LONG_BATCH, LONG_CTX, LONG_SPLITS = 128, 8, 131072, 32
LONG_WORKLOAD = (f"DeepSeek-V3-shape MXFP4 MLA decode, long context: {LONG_HEADS} heads, batch {LONG_BATCH}, "
                 f"ctx {LONG_CTX} every sequence, page {PAGE}, seeded random-permutation page table, "
                 f"num_kv_splits {LONG_SPLITS} (preallocated partials), one token appended per sequence per step")
# tensor-core work per token and head: Q K^T as three block-scaled e2m1 terms
# over the 512 latents (kind::mxf4), q_pe . k_pe in bf16 (64), P V as two
# e4m3 terms against e5m2 V'' (kind::f8f6f4)
LONG_FLOPS_MXF4, LONG_FLOPS_BF16, LONG_FLOPS_F8 = 2 * 3 * 512, 2 * 64, 2 * 2 * 512


def run_long(args, rank, world, local_rank):
    """The long-context decode (one GPU; other ranks run their own copy): a
    step is the append of one token to every sequence plus one decode call
    over the batch.  Reports the HBM fraction and the tensor-pipe fraction:
    the MMA work of a step at the measured dense bf16 rate for the bf16 RoPE
    MMAs, twice it for the fp8 kind and four times it for the fp4 kind (the
    B200's dense ratios), divided by the measured stage-1 time."""
    import torch

    import kimi_b200 as kimi

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    gen = torch.Generator(device=dev).manual_seed(17 + rank)
    pages = LONG_BATCH * LONG_CTX // PAGE
    kvb, kvs = kimi.alloc_mxfp4_cache(pages, dev, zero=False)
    chunk = 1 << 16
    for start in range(0, pages * PAGE, chunk):
        n = min(chunk, pages * PAGE - start)
        kv_c = torch.randn(n, 512, generator=gen, device=dev).to(torch.bfloat16)
        k_pe = torch.randn(n, 64, generator=gen, device=dev).to(torch.bfloat16)
        kimi.mxfp4_kv_append(kv_c, k_pe, kvb, kvs, torch.arange(start, start + n, device=dev))
    perm = torch.randperm(pages, generator=gen, device=dev).to(torch.int32)
    indptr = (torch.arange(LONG_BATCH + 1, device=dev, dtype=torch.int32) * (LONG_CTX // PAGE)).contiguous()
    last = torch.full((LONG_BATCH,), PAGE, dtype=torch.int32, device=dev)
    q = torch.randn(LONG_BATCH, LONG_HEADS, 576, generator=gen, device=dev).to(torch.bfloat16)
    o = torch.empty(LONG_BATCH, LONG_HEADS, 512, dtype=torch.bfloat16, device=dev)
    ws = kimi.alloc_workspace(LONG_BATCH, LONG_HEADS, LONG_SPLITS, dev)
    # the appended token: the last slot of each sequence's last page
    last_pages = perm[indptr[1:].long() - 1].long()
    slots = last_pages * PAGE + (PAGE - 1)
    new_c = torch.randn(LONG_BATCH, 512, generator=gen, device=dev).to(torch.bfloat16)
    new_pe = torch.randn(LONG_BATCH, 64, generator=gen, device=dev).to(torch.bfloat16)
    stream = torch.cuda.current_stream(dev)
    call = (q, kvb, kvs, o, None, indptr, perm, last)

    def step():
        kimi.mxfp4_kv_append(new_c, new_pe, kvb, kvs, slots)
        kimi.mla_decode_fwd(*call, sm_scale=SM_SCALE, num_kv_splits=LONG_SPLITS, workspace=ws)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    steps = args.steps
    with ClockSampler(dev.index) as clocks:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
        ms_step = e0.elapsed_time(e1) / steps
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2 * steps)]
        for i in range(steps):
            ev[2 * i].record(stream)
            kimi.mla_decode_partial(*call, sm_scale=SM_SCALE, num_kv_splits=LONG_SPLITS, workspace=ws)
            ev[2 * i + 1].record(stream)
        torch.cuda.synchronize()
        stage1_ms = statistics.median(ev[2 * i].elapsed_time(ev[2 * i + 1]) for i in range(steps))
        # end to end: q up from pinned host memory and o back every step
        q_host = q.cpu().pin_memory()
        o_host = torch.empty(o.shape, dtype=o.dtype).pin_memory()
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(steps):
            q.copy_(q_host, non_blocking=True)
            step()
            o_host.copy_(o, non_blocking=True)
        e1.record(stream)
        torch.cuda.synchronize()
        e2e_ms = e0.elapsed_time(e1) / steps
    tokens = LONG_BATCH * LONG_CTX
    nbytes = algorithmic_bytes(batch=LONG_BATCH, heads=LONG_HEADS, ctx=LONG_CTX)
    peak, peak_kind = _peak_hbm()
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            bf16_tf, tf_kind = float(json.load(f)["bf16_tflops"]), "measured bf16 (burst)"
    except Exception:
        bf16_tf, tf_kind = 1590.0, "fallback bf16"
    per_tok = tokens * LONG_HEADS
    ideal_ms = (per_tok * LONG_FLOPS_MXF4 / (4 * bf16_tf) + per_tok * LONG_FLOPS_BF16 / bf16_tf +
                per_tok * LONG_FLOPS_F8 / (2 * bf16_tf)) / 1e9
    achieved_gbs = nbytes / (stage1_ms * 1e6)
    if rank != 0:
        return None
    return {
        "metric": "MLA decode µs/layer, achieved HBM TB/s and tensor-pipe fraction (DeepSeek-V3 shape, "
                  "8 x 131072, 32 splits)",
        "value": round(nbytes / (ms_step * 1e9), 4), "unit": "TB/s", "n_gpus": 1, "steps": steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 5), "us_per_layer": round(ms_step * 1e3, 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded normal q and latents, cache written by the library's MXFP4 KV-append)",
        "config": {"workload": LONG_WORKLOAD, "heads": LONG_HEADS, "batch": LONG_BATCH, "ctx": LONG_CTX,
                   "num_kv_splits": LONG_SPLITS, "algorithmic_bytes_per_step": nbytes,
                   "l2": "inputs larger than L2: one 420 MB cache", "parallelism": "dp1"},
        "e2e": {"value": round(nbytes / (e2e_ms * 1e9), 4), "unit": "TB/s", "ms_per_step": round(e2e_ms, 5),
                "h2d_bytes_per_step": q.numel() * 2, "d2h_bytes_per_step": o.numel() * 2,
                "path": "q copied up from pinned host memory, append + kimi_b200.mla_decode_fwd, o copied back, "
                        "in stream order every step"},
        "gpu_launches": steps * (1 + len(STAGE1_LAUNCHES) + 1),
        "kernels": {"stage1_ms_median": round(stage1_ms, 5)},
        "roofline": {"bound": "hbm", "achieved": round(achieved_gbs, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved_gbs / peak, 4), "peak_kind": f"{peak_kind} (MEASURED_PEAKS hbm_gbs)",
                     "traffic": None},
        "tensor": {"flops_per_step": per_tok * (LONG_FLOPS_MXF4 + LONG_FLOPS_BF16 + LONG_FLOPS_F8),
                   "ideal_ms": round(ideal_ms, 5), "frac": round(ideal_ms / stage1_ms, 4),
                   "peak": f"{tf_kind} {bf16_tf} TFLOP/s for the bf16 MMAs, x2 for kind::f8f6f4, "
                           f"x4 for kind::mxf4 (the dense fp8/fp4 ratios)"},
        "clocks": clocks.summary(),
    }


def run_launches(args, rank, world, local_rank):
    """Profiler case: build the workload's inputs and make `--launches` stage-1
    calls (Q prep + decode, no merge), untimed, then print one line.  The
    captures under `profiles/` run this form (`kimi_k2`: the default Kimi-K2
    batch; `long`: the 128-head, 8 x 131072 cache with 32 splits)."""
    import torch

    import kimi_b200 as kimi

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    if args.workload == "long":
        gen = torch.Generator(device=dev).manual_seed(17 + rank)
        b, h, c, splits = LONG_BATCH, LONG_HEADS, LONG_CTX, LONG_SPLITS
        pages = b * c // PAGE
        kvb, kvs = kimi.alloc_mxfp4_cache(pages, dev, zero=False)
        for start in range(0, pages * PAGE, 1 << 16):
            n = min(1 << 16, pages * PAGE - start)
            kimi.mxfp4_kv_append(torch.randn(n, 512, generator=gen, device=dev).to(torch.bfloat16),
                                 torch.randn(n, 64, generator=gen, device=dev).to(torch.bfloat16), kvb, kvs,
                                 torch.arange(start, start + n, device=dev))
        perm = torch.randperm(pages, generator=gen, device=dev).to(torch.int32)
        indptr = (torch.arange(b + 1, device=dev, dtype=torch.int32) * (c // PAGE)).contiguous()
        last = torch.full((b,), PAGE, dtype=torch.int32, device=dev)
        q = torch.randn(b, h, 576, generator=gen, device=dev).to(torch.bfloat16)
        o = torch.empty(b, h, 512, dtype=torch.bfloat16, device=dev)
        ws = kimi.alloc_workspace(b, h, splits, dev)
    elif args.workload == "kimi_k2":
        wl = build_workload(torch, kimi, dev, seed=1)
        q, kvb, kvs, o, indptr, perm, last, ws = (wl[k] for k in ("q", "kvb", "kvs", "o", "indptr", "perm", "last", "ws"))
        splits = None
    else:
        raise SystemExit("--launches takes --workload kimi_k2 or long")
    for _ in range(args.launches):
        kimi.mla_decode_partial(q, kvb, kvs, o, None, indptr, perm, last, sm_scale=SM_SCALE, num_kv_splits=splits,
                                workspace=ws)
    torch.cuda.synchronize()
    print(f"{args.launches} stage-1 launches of {args.workload}: done", flush=True)
    return None


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["kimi_k2", "ragged", "long", "tp8_block", "tp8_prologue", "tp8_ar_norm",
                                                "tp8_vup_oproj"],
                    default="kimi_k2")
    ap.add_argument("--cpu-baseline-seconds", type=float, default=10.0,
                    help="host seconds spent timing the CPU oracle for cpu_baseline (0: omit it)")
    ap.add_argument("--launches", type=int, default=0,
                    help="profiler case: make this many untimed stage-1 calls of the workload and exit")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        line = run_reference(args, rank)
        if line is not None:
            print(json.dumps(line), flush=True)
        return

    import torch
    import torch.distributed as dist
    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        runner = {"tp8_prologue": run_prologue, "tp8_ar_norm": run_ar_norm, "tp8_vup_oproj": run_vup,
                  "long": run_long, "tp8_block": run_block}.get(args.workload, run_ours)
        if args.launches > 0:
            runner = run_launches
        line = runner(args, rank, world, local_rank)
        if line is not None:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
