"""GPU parity of the fused all-reduce + residual + RMSNorm + MXFP4 kernel
(kimi_ar_rmsnorm_mxfp4 through the C ABI) against the CPU oracle: the new
residual, the MXFP4 nibbles and the e8m0 scales bit-exact (the kernel and the
oracle take the same float32 steps in the same order).  The ranks' partials
are separate buffers on this GPU; runs of 2 and 8 processes over as many
GPUs, reading the peers' buffers through CUDA IPC mappings, check both the
one-shot and the two-shot form where that many GPUs are visible."""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

from kimi_b200 import tp  # noqa: E402
import kimi_b200  # noqa: E402
from oracle import ar_norm  # noqa: E402
from oracle import mxfp4 as omx  # noqa: E402

DEV = "cuda:0"


def _bf16_np(rng, shape, scale=1.0):
    return omx.f32_to_bf16_bits(rng.standard_normal(shape).astype(np.float32) * np.float32(scale))


def _t(bits, dev=DEV):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(dev)


def _bits(t):
    return t.cpu().view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("n,rows,hidden,legacy", [(1, 1, 7168, False), (2, 128, 7168, False),
                                                  (8, 64, 7168, False), (4, 3, 2080, True),
                                                  (3, 5, 8192, False), (2, 2, 32, True)])
def test_matches_oracle(n, rows, hidden, legacy):
    rng = np.random.default_rng(60 + n + rows)
    ins = [_bf16_np(rng, (rows, hidden), 0.5) for _ in range(n)]
    res, w = _bf16_np(rng, (rows, hidden)), _bf16_np(rng, (hidden,))
    comb, _, nib, sc = ar_norm.ar_rmsnorm_mxfp4(ins, res, w, 1e-6, legacy)
    r_out, g_nib, g_sc = tp.ar_rmsnorm_mxfp4([_t(x) for x in ins], _t(res), _t(w), 1e-6, legacy_rule=legacy)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(_bits(r_out), comb)
    np.testing.assert_array_equal(g_nib.cpu().numpy(), nib)
    np.testing.assert_array_equal(g_sc.cpu().numpy(), sc)


def test_matches_reference_rmsnorm_lines_golden():
    """The kernel on the inputs of rmsnorm_golden.npz (one rank: the
    all-reduce is the identity) against the reference's own statements
    (tests/test_ar_fusion_correctness.py:128-131): the new residual bit-exact,
    the nibbles and scales those of MXFP4 of the reference's normed rows."""
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "rmsnorm_golden.npz"))
    for n in ("m1", "m4"):
        r_out, g_nib, g_sc = tp.ar_rmsnorm_mxfp4([_t(g[f"{n}_hidden_states"])], _t(g[f"{n}_residual"]),
                                                 _t(g[f"{n}_weight"]), float(g["eps"]))
        torch.cuda.synchronize()
        nib, sc = omx.quantize_inline(g[f"{n}_normed_output"])
        np.testing.assert_array_equal(_bits(r_out), g[f"{n}_combined"])
        np.testing.assert_array_equal(g_nib.cpu().numpy(), nib)
        np.testing.assert_array_equal(g_sc.cpu().numpy(), sc)


def test_residual_updated_in_place():
    rng = np.random.default_rng(70)
    ins = [_bf16_np(rng, (16, 7168)) for _ in range(2)]
    res, w = _bf16_np(rng, (16, 7168)), _bf16_np(rng, (7168,))
    comb, _, nib, _ = ar_norm.ar_rmsnorm_mxfp4(ins, res, w, 1e-5)
    residual = _t(res)
    r_out, g_nib, _ = tp.ar_rmsnorm_mxfp4([_t(x) for x in ins], residual, _t(w), 1e-5, residual_out=residual)
    torch.cuda.synchronize()
    assert r_out.data_ptr() == residual.data_ptr()
    np.testing.assert_array_equal(_bits(residual), comb)
    np.testing.assert_array_equal(g_nib.cpu().numpy(), nib)


# ---------------------------------------------------------------------------
# two-shot form (kimi_ar_rmsnorm_mxfp4_two_shot)
# ---------------------------------------------------------------------------
def _two_shot_params(world, rank, parts, outs, flags, counter, res, w, rows, hidden, status=None,
                     timeout_ns=0):
    from kimi_b200 import _lib
    p = _lib.KimiArTwoShotParams()
    for r in range(world):
        p.inputs[r] = parts[r].data_ptr()
        p.residual_out[r], p.nibbles[r], p.scales[r] = (t.data_ptr() for t in outs[r])
        p.flags[r] = flags[r].data_ptr()
    p.counter = counter.data_ptr()
    p.residual, p.weight = res.data_ptr(), w.data_ptr()
    p.eps, p.rows, p.hidden, p.legacy_rule = 1e-6, rows, hidden, 0
    p.world, p.rank = world, rank
    p.status = status.data_ptr() if status is not None else None
    p.timeout_ns = timeout_ns
    return p


def _outs(rows, hidden, dev=DEV):
    return (torch.zeros(rows, hidden, dtype=torch.bfloat16, device=dev),
            torch.zeros(rows, hidden // 2, dtype=torch.uint8, device=dev),
            torch.zeros(rows, hidden // 32, dtype=torch.uint8, device=dev))


def test_two_shot_one_rank_matches_oracle_over_several_epochs():
    """One rank: both barriers meet at once; three calls (epochs 1..3, kept
    on the device) on new inputs, each bit-exact against the oracle; the CTA
    counter is left at zero and the call counter at 3.  Then a captured call
    replayed twice takes epochs 4 and 5."""
    import ctypes
    from kimi_b200 import _lib
    lib = _lib.load()
    rows, hidden = 37, 7168
    flags = [torch.zeros(16, dtype=torch.int32, device=DEV)]
    counter = torch.zeros(2, dtype=torch.int32, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    outs = [_outs(rows, hidden)]
    for epoch in (1, 2, 3):
        rng = np.random.default_rng(90 + epoch)
        x, res, w = _bf16_np(rng, (rows, hidden)), _bf16_np(rng, (rows, hidden)), _bf16_np(rng, (hidden,))
        part, rt, wt = _t(x), _t(res), _t(w)
        p = _two_shot_params(1, 0, [part], outs, flags, counter, rt, wt, rows, hidden, status)
        st = lib.kimi_ar_rmsnorm_mxfp4_two_shot(ctypes.byref(p), torch.cuda.current_stream().cuda_stream)
        assert st == 0, _lib.status_text(st)
        torch.cuda.synchronize()
        comb, _, nib, sc = ar_norm.ar_rmsnorm_mxfp4([x], res, w, 1e-6)
        np.testing.assert_array_equal(_bits(outs[0][0]), comb)
        np.testing.assert_array_equal(outs[0][1].cpu().numpy(), nib)
        np.testing.assert_array_equal(outs[0][2].cpu().numpy(), sc)
    assert counter.cpu().tolist() == [0, 3] and status.item() == 0
    assert flags[0].cpu().tolist()[:1] == [3] and flags[0].cpu().tolist()[8:9] == [3]
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        lib.kimi_ar_rmsnorm_mxfp4_two_shot(ctypes.byref(p), torch.cuda.current_stream().cuda_stream)
    for _ in range(2):
        g.replay()
    torch.cuda.synchronize()
    np.testing.assert_array_equal(_bits(outs[0][0]), comb)
    assert counter.cpu().tolist() == [0, 5] and flags[0].cpu().tolist()[8:9] == [5] and status.item() == 0


def test_two_shot_missing_rank_runs_out_and_reports():
    """Rank 0 of two, with rank 1 never called (its flag words are local
    memory nothing writes): the entry wait runs out (0.2 ms), no row is
    computed, the exit wait runs out too, the status word carries
    DEVICE_PEER_WAIT and the stream stays usable."""
    import ctypes
    from kimi_b200 import _lib
    lib = _lib.load()
    rows, hidden = 16, 256
    parts = [torch.zeros(rows, hidden, dtype=torch.bfloat16, device=DEV) for _ in range(2)]
    outs = [_outs(rows, hidden) for _ in range(2)]
    flags = [torch.zeros(16, dtype=torch.int32, device=DEV) for _ in range(2)]
    counter = torch.zeros(2, dtype=torch.int32, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    res = torch.ones(rows, hidden, dtype=torch.bfloat16, device=DEV)
    w = torch.ones(hidden, dtype=torch.bfloat16, device=DEV)
    p = _two_shot_params(2, 0, parts, outs, flags, counter, res, w, rows, hidden, status, timeout_ns=200_000)
    st = lib.kimi_ar_rmsnorm_mxfp4_two_shot(ctypes.byref(p), torch.cuda.current_stream().cuda_stream)
    assert st == 0
    bits = kimi_b200.device_status(status)
    assert bits == _lib.DEVICE_PEER_WAIT, hex(bits)
    assert torch.count_nonzero(outs[0][0]).item() == 0  # nothing was computed
    assert counter.cpu().tolist() == [0, 1]
    torch.ones(4, device=DEV).sum().item()  # the context still works


def _ranks_worker(rank, world, port, result_dir):
    """Both forms on `world` GPUs, [128, 7168]: bit-exact against the oracle
    for three different inputs (two-shot calls 1..3), then each form timed
    with CUDA events over 50 calls replayed from a CUDA graph (the two-shot
    call with its device barriers; the one-shot kernel without the host
    barriers it needs) -- written to the result file."""
    import datetime
    import json
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    result = {"ok": True}
    try:
        rows, hidden = 128, 7168
        peers = tp.PeerPartials(rows, hidden, dev)
        for it in range(3):
            rng = np.random.default_rng(200 + it)
            ins = [_bf16_np(rng, (rows, hidden), 0.5) for _ in range(world)]
            res, w = _bf16_np(rng, (rows, hidden)), _bf16_np(rng, (hidden,))
            comb, _, nib_ref, sc_ref = ar_norm.ar_rmsnorm_mxfp4(ins, res, w, 1e-6)
            peers.local.copy_(_t(ins[rank], dev))
            rt, wt = _t(res, dev), _t(w, dev)
            r1, n1, s1 = peers.reduce_norm_quant(rt, wt, 1e-6)
            torch.cuda.synchronize()
            one_ok = (np.array_equal(_bits(r1), comb) and np.array_equal(n1.cpu().numpy(), nib_ref)
                      and np.array_equal(s1.cpu().numpy(), sc_ref))
            r2, n2, s2 = peers.reduce_norm_quant_two_shot(rt, wt, 1e-6)
            torch.cuda.synchronize()
            two_ok = (np.array_equal(_bits(r2), comb) and np.array_equal(n2.cpu().numpy(), nib_ref)
                      and np.array_equal(s2.cpu().numpy(), sc_ref))
            result["ok"] = result["ok"] and one_ok and two_ok
            result.setdefault("one_shot_ok", []).append(one_ok)
            result.setdefault("two_shot_ok", []).append(two_ok)
        result["status"] = kimi_b200.device_status(peers.status)
        result["ok"] = result["ok"] and result["status"] == 0
        # timing: 50 calls captured in a CUDA graph (the two-shot call, whose
        # barriers are on the device, and the one-shot kernel alone) and
        # replayed once on every rank together, so the host's launch rate
        # does not enter (the two-shot call numbers itself on the device)
        for name, fn in (("two_shot_us", lambda: peers.reduce_norm_quant_two_shot(rt, wt, 1e-6)),
                         ("one_shot_kernel_us", lambda: tp.ar_rmsnorm_mxfp4(peers.ptrs, rt, wt, 1e-6))):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for _ in range(50):
                    fn()
            torch.cuda.synchronize()
            dist.barrier()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            g.replay()
            e.record()
            torch.cuda.synchronize()
            result[name] = s.elapsed_time(e) * 1e3 / 50
            del g
        result["status_after_timing"] = kimi_b200.device_status(peers.status)
        with open(os.path.join(result_dir, f"rank{rank}.json"), "w") as f:
            json.dump(result, f)
        peers.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 8])
def test_ranks_over_nvlink_one_and_two_shot(world, tmp_path):
    import json
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.start_processes(_ranks_worker, args=(world, port, str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    results = [json.loads((tmp_path / f"rank{r}.json").read_text()) for r in range(world)]
    out = os.environ.get("KIMI_AR_TIMING_OUT")
    if out:  # a summary of the timings (max over ranks), for the profiles
        with open(out, "a") as f:
            f.write(json.dumps({"world": world, "two_shot_us": max(r["two_shot_us"] for r in results),
                                "one_shot_kernel_us": max(r["one_shot_kernel_us"] for r in results)}) + "\n")
    for r, res in enumerate(results):
        assert res["ok"], (r, res)
        assert res["status_after_timing"] == 0, (r, res)
