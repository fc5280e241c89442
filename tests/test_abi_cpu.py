"""The C-ABI library without a GPU: it loads, exports every symbol the header
declares, and rejects bad arguments on the host before any launch."""
import ctypes
import os
import re

import pytest

from kimi_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "kimi_mla.h")


def _declared_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"KIMI_API\s+[\w\s\*]*?\b(kimi_\w+)\s*\(", text)))


def test_header_declarations_match_binding_list():
    assert _declared_functions() == sorted(_lib.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(_lib.LIB_PATH)
    for name in _declared_functions():
        assert hasattr(lib, name), name


def test_status_strings_and_version():
    lib = _lib.load()
    assert lib.kimi_abi_version() == _lib.ABI_VERSION == 201
    assert _lib.status_text(0) == "ok"
    assert "workspace" in _lib.status_text(-5)
    assert _lib.status_text(-12345) == "unknown status"


def test_device_status_texts():
    # positive codes below KIMI_ERR_CUDA_BASE are device status words
    # (KIMI_DEVICE_* bits) read back by kimi_device_status
    assert "gave up" in _lib.status_text(0x010)
    assert "gave up" in _lib.status_text(0x001 | 0x080)
    bad = _lib.status_text(_lib.DEVICE_BAD_PAGE)
    assert "outside the cache" in bad and "gave up" not in bad
    both = _lib.status_text(_lib.DEVICE_BAD_PAGE | 0x040)
    assert "gave up" in both and "outside the cache" in both
    assert "peer rank" in _lib.status_text(_lib.DEVICE_PEER_WAIT)
    assert "gave up" in _lib.status_text(_lib.DEVICE_QABSORB_WAIT)
    assert "gave up" in _lib.status_text(_lib.DEVICE_VUP_WAIT)
    # every combination of device bits stays below the CUDA error range
    assert "gave up" in _lib.status_text(0x3FF) and "peer rank" in _lib.status_text(0x7FF)
    assert 0x7FF < _lib.KIMI_ERR_CUDA_BASE
    # CUDA errors keep their own range
    assert "gave up" not in _lib.status_text(_lib.KIMI_ERR_CUDA_BASE + 2)


def test_device_status_argument_checks():
    lib = _lib.load()
    assert lib.kimi_device_status(None, 0, None) == -1  # KIMI_ERR_NULL_POINTER
    assert lib.kimi_device_status(3, 0, None) == -4  # KIMI_ERR_MISALIGNED


# Q operand images of the decode kernel per (sequence, head block of NH heads):
# three e2m1 terms (2 x 3 NH x 128 B), q_pe (NH x 128 B) and the terms' e8m0
# scales (3 NH rows x 16 blocks).  NH = 64, or 16 when the call has at most 16
# heads.
def q_image_bytes(nh):
    return 2 * 3 * nh * 128 + nh * 128 + 3 * nh * 16


def heads_per_block(h):
    return 16 if h <= 16 else 64


Q_IMAGE_BYTES = q_image_bytes(64)
assert Q_IMAGE_BYTES == 60416 and q_image_bytes(16) == 15104


def test_workspace_size_arithmetic():
    lib = _lib.load()
    # explicit splits: partial O (B*S*H*512 bf16) + LSE (B*S*H f32) + the fp4
    # kernel's Q operand images (B * head blocks * 60416 B), each rounded to 256 B
    b, h, s = 64, 64, 4
    rows = b * s * h
    r256 = lambda n: ((n + 255) // 256) * 256
    expect = r256(rows * 512 * 2) + r256(rows * 4) + r256(b * 1 * Q_IMAGE_BYTES)
    assert lib.kimi_mla_decode_workspace_size(b, h, s) == expect
    assert lib.kimi_mla_decode_workspace_size(b, h, 1) == 0  # single split writes o directly
    assert lib.kimi_mla_decode_workspace_size(b, 0, 4) == 0  # invalid
    # 8 heads (a TP8 shard): one 16-head block per sequence
    rows8 = b * s * 8
    assert lib.kimi_mla_decode_workspace_size(b, 8, s) == (r256(rows8 * 512 * 2) + r256(rows8 * 4)
                                                         + r256(b * 1 * q_image_bytes(16)))
    assert lib.kimi_mla_decode_num_splits(b, h, 7) == 7
    assert lib.kimi_mla_decode_num_splits(b, h, 999) == 64


def test_balanced_workspace_size_arithmetic():
    # num_kv_splits = 0: balanced schedule over G CTAs per head block; the
    # workspace holds B + G partial slots plus one int2 CTA span per sequence
    lib = _lib.load()
    for b, h in ((64, 64), (2, 16), (8, 128), (128, 8)):
        g = lib.kimi_mla_decode_num_splits(b, h, 0)
        assert g >= 1
        slots = b + g
        r256 = lambda n: ((n + 255) // 256) * 256
        nh = heads_per_block(h)
        expect = (r256(slots * h * 512 * 2) + r256(slots * h * 4) + r256(b * 8)
                  + r256(b * -(-h // nh) * q_image_bytes(nh)))
        assert lib.kimi_mla_decode_workspace_size(b, h, 0) == expect
    assert lib.kimi_mla_decode_num_splits(8, 128, 0) * 2 <= lib.kimi_mla_decode_num_splits(8, 64, 0) + 1


def test_decode_rejects_bad_arguments_on_host():
    lib = _lib.load()
    assert lib.kimi_mla_decode(None, None, 0, None) == -1
    p = _lib.KimiMlaDecodeParams(batch=2, num_heads=0, num_kv_splits=1, sm_scale=0.1)
    assert lib.kimi_mla_decode(ctypes.byref(p), None, 0, None) == -2
    p = _lib.KimiMlaDecodeParams(batch=2, num_heads=16, num_kv_splits=1, sm_scale=0.1, logit_cap=30.0)
    assert lib.kimi_mla_decode(ctypes.byref(p), None, 0, None) == -6
    p = _lib.KimiMlaDecodeParams(batch=2, num_heads=16, num_kv_splits=1, sm_scale=0.1)
    assert lib.kimi_mla_decode(ctypes.byref(p), None, 0, None) == -1  # null tensors
    # misaligned q pointer (the library never dereferences host-side checks' inputs)
    p = _lib.KimiMlaDecodeParams(q=0x1002, q_stride_b=16 * 576, q_stride_h=576, kv_buffer=0x1000,
                                 kv_scales=0x2000, num_pages=1, kv_indptr=0x3000, kv_indices=0x4000,
                                 o=0x5000, o_stride_b=16 * 512, o_stride_h=512, batch=2, num_heads=16,
                                 num_kv_splits=1, sm_scale=0.1)
    assert lib.kimi_mla_decode(ctypes.byref(p), None, 0, None) == -4
    p.q = 0x1000
    p.q_stride_h = 577
    assert lib.kimi_mla_decode(ctypes.byref(p), None, 0, None) == -3
    p.q_stride_h = 576
    p.status = 0x6002  # the optional device status word must be 4-byte aligned
    assert lib.kimi_mla_decode(ctypes.byref(p), None, 0, None) == -4
    p.status = None
    p.num_kv_splits = 4
    assert lib.kimi_mla_decode(ctypes.byref(p), None, 0, None) == -5  # no workspace for 4 splits
    # batch 0 is a no-op
    p0 = _lib.KimiMlaDecodeParams(batch=0, num_heads=16, num_kv_splits=1, sm_scale=0.1)
    assert lib.kimi_mla_decode(ctypes.byref(p0), None, 0, None) == 0


def test_append_and_quantize_reject_bad_arguments_on_host():
    lib = _lib.load()
    assert lib.kimi_mxfp4_kv_append(None, None) == -1
    p = _lib.KimiKvAppendParams(num_tokens=4, num_pages=1, legacy_rule=2)
    assert lib.kimi_mxfp4_kv_append(ctypes.byref(p), None) == -6
    p = _lib.KimiKvAppendParams(kv_c=0x1000, kv_c_stride=500, k_pe=0x2000, k_pe_stride=64, slot_mapping=0x3000,
                                kv_buffer=0x4000, kv_scales=0x5000, num_pages=1, num_tokens=4)
    assert lib.kimi_mxfp4_kv_append(ctypes.byref(p), None) == -3
    assert lib.kimi_mxfp4_quantize(None, 4, 48, 48, None, None, 0, None) == -2   # cols % 32
    assert lib.kimi_mxfp4_quantize(None, 4, 64, 64, None, None, 0, None) == -1
    assert lib.kimi_mxfp4_quantize(0x1000, 0, 64, 64, 0x2000, 0x3000, 0, None) == 0  # empty


def test_python_wrappers_reject_cpu_tensors():
    import torch

    import kimi_b200

    q = torch.zeros(1, 16, 576, dtype=torch.bfloat16)
    kvb, kvs = torch.zeros(1, 64, 384, dtype=torch.uint8), torch.zeros(1, 64, 16, dtype=torch.uint8)
    o = torch.zeros(1, 16, 512, dtype=torch.bfloat16)
    ip = torch.tensor([0, 1], dtype=torch.int32)
    with pytest.raises(ValueError):
        kimi_b200.mla_decode_fwd(q, kvb, kvs, o, None, ip, ip[:1], None)


def test_tp8_entry_points_reject_bad_arguments_on_host():
    """The prologue, V up-projection + o_proj and all-reduce + RMSNorm + MXFP4
    entry points check their arguments before any launch."""
    lib = _lib.load()
    # decode prologue
    assert lib.kimi_mla_q_absorb_rope_append(None, None) == -1
    p = _lib.KimiQAbsorbParams(num_tokens=4, num_heads=0, max_position=8)
    assert lib.kimi_mla_q_absorb_rope_append(ctypes.byref(p), None) == -2      # no heads
    p = _lib.KimiQAbsorbParams(num_tokens=4, num_heads=8, max_position=8, is_neox=2)
    assert lib.kimi_mla_q_absorb_rope_append(ctypes.byref(p), None) == -6      # is_neox not 0/1
    p = _lib.KimiQAbsorbParams(num_tokens=0, num_heads=8, max_position=8)
    assert lib.kimi_mla_q_absorb_rope_append(ctypes.byref(p), None) == 0       # nothing to do
    p = _lib.KimiQAbsorbParams(num_tokens=4, num_heads=8, max_position=8)
    assert lib.kimi_mla_q_absorb_rope_append(ctypes.byref(p), None) == -1      # null tensors
    # V up-projection + o_proj
    assert lib.kimi_mla_v_up_o_proj(None, None) == -1
    for heads, hidden in ((9, 128), (0, 128), (8, 96), (8, 0)):
        p = _lib.KimiVUpOProjParams(num_tokens=4, num_heads=heads, hidden=hidden)
        assert lib.kimi_mla_v_up_o_proj(ctypes.byref(p), None) == -2, (heads, hidden)
    p = _lib.KimiVUpOProjParams(num_tokens=0, num_heads=8, hidden=128)
    assert lib.kimi_mla_v_up_o_proj(ctypes.byref(p), None) == 0
    p = _lib.KimiVUpOProjParams(num_tokens=4, num_heads=8, hidden=128)
    assert lib.kimi_mla_v_up_o_proj(ctypes.byref(p), None) == -1
    ptrs = dict(o=0x10000, w_uv=0x20000, w_o=0x30000, x=0x40000, out=0x50000)
    p = _lib.KimiVUpOProjParams(num_tokens=4, num_heads=8, hidden=128, o_stride_h=2048, o_stride_t=516,
                                out_stride=128, **ptrs)
    assert lib.kimi_mla_v_up_o_proj(ctypes.byref(p), None) == -3               # token stride % 8
    p = _lib.KimiVUpOProjParams(num_tokens=4, num_heads=8, hidden=128, o_stride_h=2048, o_stride_t=512,
                                out_stride=64, **ptrs)
    assert lib.kimi_mla_v_up_o_proj(ctypes.byref(p), None) == -3               # out rows overlap
    p = _lib.KimiVUpOProjParams(num_tokens=4, num_heads=8, hidden=128, o_stride_h=2048, o_stride_t=512,
                                out_stride=128, **dict(ptrs, out=0x50008))
    assert lib.kimi_mla_v_up_o_proj(ctypes.byref(p), None) == -4               # misaligned out
    # all-reduce + residual + RMSNorm + MXFP4
    assert lib.kimi_ar_rmsnorm_mxfp4(None, None) == -1
    for rows, hidden, n in ((4, 48, 2), (4, 8224, 2), (4, 256, 0), (4, 256, _lib.AR_MAX_INPUTS + 1)):
        p = _lib.KimiArRmsNormParams(rows=rows, hidden=hidden, num_inputs=n, eps=1e-6)
        assert lib.kimi_ar_rmsnorm_mxfp4(ctypes.byref(p), None) == -2, (rows, hidden, n)
    p = _lib.KimiArRmsNormParams(rows=4, hidden=256, num_inputs=2, eps=float("nan"))
    assert lib.kimi_ar_rmsnorm_mxfp4(ctypes.byref(p), None) == -2
    p = _lib.KimiArRmsNormParams(rows=0, hidden=256, num_inputs=2, eps=1e-6)
    assert lib.kimi_ar_rmsnorm_mxfp4(ctypes.byref(p), None) == 0
    p = _lib.KimiArRmsNormParams(rows=4, hidden=256, num_inputs=2, eps=1e-6, residual=0x1000, residual_out=0x2000,
                                 weight=0x3000, nibbles=0x4000, scales=0x5000)
    p.inputs[0], p.inputs[1] = 0x6000, 0x7008
    assert lib.kimi_ar_rmsnorm_mxfp4(ctypes.byref(p), None) == -4              # misaligned partial


def test_ctypes_structs_match_the_header_layout(tmp_path):
    """Every params struct of _lib has the C header's field offsets and size:
    a small C program built against include/kimi_mla.h prints them."""
    import os
    import shutil
    import subprocess
    if shutil.which("gcc") is None:
        pytest.skip("no C compiler")
    structs = [name for name in dir(_lib) if name.startswith("Kimi") and name.endswith("Params")]
    assert structs
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "kimi_mla.h"', "int main(void) {"]
    for name in structs:
        lines.append(f'  printf("{name} size %zu\\n", sizeof({name}));')
        for field, _ in getattr(_lib, name)._fields_:
            lines.append(f'  printf("{name} {field} %zu\\n", offsetof({name}, {field}));')
    lines += ["  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    inc = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include")
    subprocess.run(["gcc", "-I", inc, str(src), "-o", str(exe)], check=True)
    got = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split("\n")
    c_layout = {tuple(line.split()[:2]): int(line.split()[2]) for line in got if line}
    for name in structs:
        st = getattr(_lib, name)
        assert c_layout[(name, "size")] == ctypes.sizeof(st), name
        for field, _ in st._fields_:
            assert c_layout[(name, field)] == getattr(st, field).offset, (name, field)
