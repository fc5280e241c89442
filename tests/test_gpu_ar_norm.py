"""GPU parity of the fused all-reduce + residual + RMSNorm + MXFP4 kernel
(kimi_ar_rmsnorm_mxfp4 through the C ABI) against the CPU oracle: the new
residual, the MXFP4 nibbles and the e8m0 scales bit-exact (the kernel and the
oracle take the same float32 steps in the same order).  The ranks' partials
are separate buffers on this GPU; a two-process run over two GPUs, reading
the peer's buffer through a CUDA IPC mapping, runs where two GPUs are
visible."""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

from kimi_b200 import tp  # noqa: E402
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


def _two_rank_worker(rank, world, port, result_dir):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    import datetime
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        rng = np.random.default_rng(80)
        rows, hidden = 128, 7168
        ins = [_bf16_np(rng, (rows, hidden), 0.5) for _ in range(world)]
        res, w = _bf16_np(rng, (rows, hidden)), _bf16_np(rng, (hidden,))
        peers = tp.PeerPartials(rows, hidden, dev)
        peers.local.copy_(_t(ins[rank], dev))
        r_out, nib, sc = peers.reduce_norm_quant(_t(res, dev), _t(w, dev), 1e-6)
        torch.cuda.synchronize()
        comb, _, nib_ref, sc_ref = ar_norm.ar_rmsnorm_mxfp4(ins, res, w, 1e-6)
        ok = (np.array_equal(_bits(r_out), comb) and np.array_equal(nib.cpu().numpy(), nib_ref)
              and np.array_equal(sc.cpu().numpy(), sc_ref))
        with open(os.path.join(result_dir, f"rank{rank}"), "w") as f:
            f.write("ok" if ok else "mismatch")
        peers.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_ranks_over_nvlink(tmp_path):
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.start_processes(_two_rank_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    for r in range(2):
        assert (tmp_path / f"rank{r}").read_text() == "ok"
