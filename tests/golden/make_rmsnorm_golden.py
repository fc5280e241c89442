"""Generate ``rmsnorm_golden.npz`` from the reference's own residual-add +
RMSNorm lines.

Run once, in a container where the reference checkout is mounted (the path
is the first argument, default /root/reference):

    python tests/golden/make_rmsnorm_golden.py [/path/to/kimi]

The statements are read from tests/test_ar_fusion_correctness.py:128-131
(``test_ar_fusion_forward_path_shapes``):

    combined = (hidden_states.float() + residual.float()).to(torch.bfloat16)
    variance = combined.float().pow(2).mean(-1, keepdim=True)
    normed = (combined.float() * torch.rsqrt(variance + eps)).to(torch.bfloat16)
    normed_output = normed * weight.unsqueeze(0)

and executed unmodified on CPU tensors (the test itself builds its tensors on
a GPU and then calls aiter, so the function is not called; its all-reduce is
the identity there, as it is for one rank here).  The inputs are seeded
torch.randn bf16 tensors of the test's shape (hidden 7168, eps 1e-6), for 1
row (the test's M) and 4 rows.

Each case stores bf16 bit patterns (uint16): hidden_states, residual and
weight, and the reference's ``combined`` (the new residual) and
``normed_output``.
"""
from __future__ import annotations

import os
import sys
import textwrap

import numpy as np
import torch

HIDDEN, EPS = 7168, 1e-6
CASES = [("m1", 1, 123), ("m4", 4, 124)]  # (name, rows, seed)
FIRST = "combined = (hidden_states.float() + residual.float()).to(torch.bfloat16)"
LAST = "normed_output = normed * weight.unsqueeze(0)"


def reference_lines(root: str) -> str:
    path = os.path.join(root, "tests", "test_ar_fusion_correctness.py")
    with open(path) as f:
        lines = f.read().splitlines()
    start = next(i for i, l in enumerate(lines) if l.strip() == FIRST)
    end = next(i for i in range(start, len(lines)) if lines[i].strip() == LAST)
    assert end - start == 3, "the four statements are no longer contiguous"
    return textwrap.dedent("\n".join(lines[start:end + 1]))


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def main(root: str) -> None:
    code = reference_lines(root)
    out = {}
    for name, rows, seed in CASES:
        torch.manual_seed(seed)
        ns = dict(torch=torch, eps=EPS,
                  hidden_states=torch.randn(rows, HIDDEN, dtype=torch.bfloat16),
                  residual=torch.randn(rows, HIDDEN, dtype=torch.bfloat16),
                  weight=torch.randn(HIDDEN, dtype=torch.bfloat16))
        exec(code, ns)  # the reference's statements, as written
        for key in ("hidden_states", "residual", "weight", "combined", "normed_output"):
            out[f"{name}_{key}"] = _bits(ns[key])
    dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "rmsnorm_golden.npz")
    np.savez_compressed(dst, eps=np.float32(EPS), **out)
    print("wrote", dst, sorted(out))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
