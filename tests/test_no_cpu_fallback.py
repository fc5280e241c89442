"""The product path has no CPU fallback: every public entry point refuses CPU
tensors with an error, and a missing C-ABI library is an error too (the CPU
oracle is test infrastructure only)."""
import pytest

torch = pytest.importorskip("torch")

import kimi_b200  # noqa: E402
from kimi_b200 import _lib, tp  # noqa: E402

bf = torch.bfloat16


def _z(*shape, dtype=bf):
    return torch.zeros(*shape, dtype=dtype)


ENTRY_POINTS = {
    "mla_decode_fwd": lambda: kimi_b200.mla_decode_fwd(
        _z(2, 16, 576), _z(2, 64, 384, dtype=torch.uint8), _z(2, 64, 16, dtype=torch.uint8), _z(2, 16, 512), None,
        torch.tensor([0, 1, 2], dtype=torch.int32), torch.tensor([0, 1], dtype=torch.int32), None),
    "mxfp4_kv_append": lambda: kimi_b200.mxfp4_kv_append(
        _z(4, 512), _z(4, 64), _z(1, 64, 384, dtype=torch.uint8), _z(1, 64, 16, dtype=torch.uint8),
        torch.arange(4)),
    "mxfp4_quantize": lambda: kimi_b200.mxfp4_quantize(_z(4, 64)),
    "q_absorb_rope_append": lambda: kimi_b200.q_absorb_rope_append(
        _z(4, 2, 128), _z(4, 2, 64), _z(2, 128, 512), _z(4, 512), _z(4, 64), torch.zeros(4, dtype=torch.int64),
        _z(8, 32, dtype=torch.float32), _z(8, 32, dtype=torch.float32), _z(1, 64, 384, dtype=torch.uint8),
        _z(1, 64, 16, dtype=torch.uint8), torch.arange(4)),
    "v_up_proj_and_o_proj": lambda: kimi_b200.v_up_proj_and_o_proj(_z(2, 4, 512), _z(2, 512, 128), _z(64, 256)),
    "ar_rmsnorm_mxfp4": lambda: tp.ar_rmsnorm_mxfp4([_z(4, 256), _z(4, 256)], _z(4, 256), _z(256)),
}


@pytest.mark.parametrize("name", sorted(ENTRY_POINTS))
def test_cpu_tensors_are_refused(name):
    with pytest.raises(ValueError, match="CUDA"):
        ENTRY_POINTS[name]()


def test_missing_library_is_an_error(monkeypatch):
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", "/nonexistent/libkimi_mla.so")
    with pytest.raises(RuntimeError, match="no CPU or Python fallback"):
        _lib.load()
