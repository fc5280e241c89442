"""Generate ``vup_golden.npz`` from the reference's own V up-projection + o_proj.

Run once, in a container where the reference checkout is mounted (the path
is the first argument, default /root/reference):

    python tests/golden/make_vup_golden.py [/path/to/kimi]

It imports, unmodified, tests/test_mla_heads_first_e2e.py and calls
``MockMLAVUpProj.forward_heads_first`` (:50-59: ``bmm(o.float(),
W_V.float()).to(bf16)``, the transpose to [B, N * 128], ``mm(x,
o_proj_weight.T)`` in bf16) and ``forward_standard`` (:39-48) on CPU
tensors.  The module's constructor allocates its weights on a GPU, so the
module object is built without it and given CPU weights of the same shapes.

Each case stores (bf16 as uint16 bit patterns): o [N, B, 512] heads-first,
w_uv [N, 512, 128], w_o [hidden, N * 128], the heads-first output and the
standard path's output [B, hidden].
"""
from __future__ import annotations

import importlib.util
import os
import sys

import numpy as np
import torch
import torch.nn as nn

CASES = [
    # (name, N heads, B tokens, hidden, weight scale, seed)
    ("unit_n2_b5_h128", 2, 5, 128, 1.0, 11),   # the reference test's randn weights, ragged batch
    ("n4_b4_h64", 4, 4, 64, 0.02, 12),         # N(0, 0.02) weights, as the TP8 block's
    ("n1_b130_h64", 1, 130, 64, 0.02, 13),     # more than one 128-token tile
]


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def main(ref_root: str) -> None:
    path = os.path.join(ref_root, "tests", "test_mla_heads_first_e2e.py")
    spec = importlib.util.spec_from_file_location("ref_heads_first_e2e", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    out = {}
    for name, n, b, hidden, scale, seed in CASES:
        g = torch.Generator().manual_seed(seed)
        model = mod.MockMLAVUpProj.__new__(mod.MockMLAVUpProj)
        nn.Module.__init__(model)
        model.num_heads, model.kv_lora_rank, model.v_head_dim = n, 512, 128
        model.hidden_size, model.dtype = hidden, torch.bfloat16
        model.W_V = nn.Parameter((torch.randn(n, 512, 128, generator=g) * scale).to(torch.bfloat16),
                                 requires_grad=False)
        model.o_proj_weight = nn.Parameter((torch.randn(hidden, n * 128, generator=g) * scale).to(torch.bfloat16),
                                           requires_grad=False)
        o = torch.randn(n, b, 512, generator=g).to(torch.bfloat16)
        with torch.no_grad():
            hf = model.forward_heads_first(o.contiguous())
            std = model.forward_standard(o.permute(1, 0, 2).contiguous())
        out[f"{name}/o"] = _bits(o)
        out[f"{name}/w_uv"] = _bits(model.W_V.data)
        out[f"{name}/w_o"] = _bits(model.o_proj_weight.data)
        out[f"{name}/out_heads_first"] = _bits(hf)
        out[f"{name}/out_standard"] = _bits(std)
    dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "vup_golden.npz")
    np.savez_compressed(dst, **out)
    print(f"wrote {dst}: {len(CASES)} cases")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
