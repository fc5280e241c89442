"""Generate the golden fixtures in this folder from the reference's own code.

Run once, in a container where the reference checkout is mounted (the path
is the first argument, default /root/reference):

    python tests/golden/make_golden.py [/path/to/kimi]

It imports, unmodified:

* archive/mla-mxfp4-dead-end/mla_decode_mxfp4_v5.py -- ``_quantize_mxfp4_torch``
  (legacy torch quantiser, :421-438), ``_dequant_mxfp4_torch`` (:381-400) and
  the Triton device quantiser ``_mxfp4_quant_inline`` (:18-75).  The Triton
  function runs under Triton's CPU interpreter (``TRITON_INTERPRET=1``).  Two
  interpreter gaps are closed first so that it computes what the Triton
  compiler would: the ``tensor.floor()`` member form is bound to
  ``triton.language.math.floor``, and a Python ``not`` applied to a tensor is
  rewritten to the tensor's element-wise ``__not__`` (the compiler's
  ``visit_UnaryOp`` does this; the interpreter would otherwise take the
  truth value of the whole tensor).  The reference source is not touched.
* tests/test_triton_mla_decode.py -- ``reference_mla_decode`` (:12-62), the
  fp32 paged MLA decode, composed with ``_dequant_mxfp4_torch`` for the
  512-dim MXFP4 latent + 64-dim bf16 RoPE cache layout.

Outputs (numpy ``.npz``, bf16 stored as uint16 bit patterns):

* ``quant_golden.npz``   -- quantiser inputs and both rules' nibbles/scales.
* ``dequant_golden.npz`` -- random nibbles/scales and their float32 dequant.
* ``decode_golden.npz``  -- paged decode cases: q, page table, cache bytes
  (quantised by the reference's Triton rule) and the fp32 reference output.

No file under this folder is read from the reference at test time; the
tests only read the committed ``.npz`` files.
"""
from __future__ import annotations

import ast
import math
import os
import sys

os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
v5 = None  # the reference module, bound by _load_reference (the jit kernel resolves it as a global)


def _load_reference(root: str):
    sys.path.insert(0, os.path.join(root, "archive", "mla-mxfp4-dead-end"))
    sys.path.insert(0, os.path.join(root, "tests"))
    import triton
    import triton.language as tl
    import triton.language.math as tmath
    from triton.runtime import interpreter

    tl.tensor.floor = lambda self: tmath.floor(self, _semantic=interpreter.interpreter_semantic)

    def _tensor_logical_not(x):
        if isinstance(x, tl.tensor):
            return x.__not__(_semantic=interpreter.interpreter_semantic)
        return not x

    def _visit_unary(self, node):
        node = self.generic_visit(node)
        if isinstance(node.op, ast.Not):
            call = ast.Call(func=ast.Name(id="_tensor_logical_not", ctx=ast.Load()),
                            args=[node.operand], keywords=[])
            return ast.copy_location(call, node)
        return node

    orig_visit_assign = interpreter.ASTTransformer.visit_Assign

    def _visit_assign(self, node):
        node.value = self.visit(node.value)  # the stock visit_Assign does not descend into values
        return orig_visit_assign(self, node)

    interpreter._tensor_logical_not = _tensor_logical_not  # copied into jit globals on rewrite
    interpreter.ASTTransformer.visit_UnaryOp = _visit_unary
    interpreter.ASTTransformer.visit_Assign = _visit_assign
    global v5
    import mla_decode_mxfp4_v5 as v5
    import test_triton_mla_decode as tmd

    @triton.jit
    def _quant_rows(X, OUT_Q, OUT_S, BLOCK_M: tl.constexpr, BLOCK_K: tl.constexpr):
        pid = tl.program_id(0)
        offs_m = pid * BLOCK_M + tl.arange(0, BLOCK_M)
        offs_k = tl.arange(0, BLOCK_K)
        x = tl.load(X + offs_m[:, None] * BLOCK_K + offs_k[None, :])
        q, s = v5._mxfp4_quant_inline(x, BLOCK_K, BLOCK_M)
        tl.store(OUT_Q + offs_m[:, None] * (BLOCK_K // 2) + tl.arange(0, BLOCK_K // 2)[None, :], q)
        tl.store(OUT_S + offs_m[:, None] * (BLOCK_K // 32) + tl.arange(0, BLOCK_K // 32)[None, :], s)

    def quant_inline(x_bf16: torch.Tensor):
        n, k = x_bf16.shape
        block_m = 16
        pad = (-n) % block_m
        xp = torch.cat([x_bf16, torch.zeros(pad, k, dtype=x_bf16.dtype)]) if pad else x_bf16
        oq = torch.empty(xp.shape[0], k // 2, dtype=torch.uint8)
        osc = torch.empty(xp.shape[0], k // 32, dtype=torch.uint8)
        _quant_rows[(xp.shape[0] // block_m,)](xp.contiguous(), oq, osc, BLOCK_M=block_m, BLOCK_K=k)
        return oq[:n], osc[:n]

    return v5, tmd, quant_inline


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def _edge_rows(d: int) -> torch.Tensor:
    """Hand-made 32-element groups: zeros, exact rounding ties for both rules,
    amax values that round up at mantissa 0b11, negative zeros, tiny and huge
    magnitudes (all finite bf16)."""
    groups = []
    groups.append([0.0] * 32)
    groups.append([-0.0] * 32)
    ties = [0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 4.0]
    groups.append((ties + [-t for t in ties]) * 2)
    groups.append([t * 0.125 for t in ties] * 4)
    groups.append([7.0, 3.5, 1.75, 0.875, 6.0, 5.5, 7.5, 0.1] * 4)
    groups.append([1e-30, -2e-30, 3e-38, 1e-38] * 8)
    groups.append([1e30, -3e35, 2e38, 1.0] * 8)
    groups.append([6.0, 12.0, 24.0, 3.0, -6.0, -12.0, 0.5, 0.0] * 4)
    groups.append([1.0 + i / 64.0 for i in range(32)])
    groups.append([-(1.75 + i / 128.0) for i in range(32)])
    groups.append([0.0] * 31 + [1e-12])
    groups.append([0.0] * 31 + [9.0e-13])
    flat = [v for g in groups for v in g]
    per_row = d
    while len(flat) % per_row:
        flat.append(0.0)
    return torch.tensor(flat, dtype=torch.float32).reshape(-1, per_row).to(torch.bfloat16)


def make_quant(quant_inline, v5) -> dict:
    d = 512
    g = torch.Generator().manual_seed(0)
    gauss = torch.randn(128, d, generator=g).to(torch.bfloat16)
    scales = torch.tensor([10.0 ** k for k in range(-30, 34)], dtype=torch.float32)
    scaled = (torch.randn(64, d, generator=g) * scales[:, None]).to(torch.bfloat16)
    x = torch.cat([gauss, scaled, _edge_rows(d)])
    q_in, s_in = quant_inline(x)
    q_lg, s_lg = v5._quantize_mxfp4_torch(x)
    return {
        "x_bits": _bits(x),
        "inline_nibbles": q_in.numpy(), "inline_scales": s_in.numpy(),
        "legacy_nibbles": q_lg.numpy(), "legacy_scales": s_lg.numpy(),
    }


def make_dequant(v5) -> dict:
    g = torch.Generator().manual_seed(1)
    n, d = 96, 512
    nib = torch.randint(0, 256, (n, d // 2), generator=g, dtype=torch.int64).to(torch.uint8)
    sc = torch.randint(100, 150, (n, d // 32), generator=g, dtype=torch.int64).to(torch.uint8)
    sc[0, :] = torch.tensor([0, 1, 2, 126, 127, 128, 200, 253, 254, 3, 4, 5, 120, 121, 122, 123],
                            dtype=torch.uint8)
    out = v5._dequant_mxfp4_torch(nib, sc, d)
    return {"nibbles": nib.numpy(), "scales": sc.numpy(), "values": out.numpy()}


def _decode_case(v5, tmd, quant_inline, seed, seq_lens, heads, sm_scale, shuffle_pages):
    page = 64
    g = torch.Generator().manual_seed(seed)
    n_pages_per = [max(1, math.ceil(l / page)) if l > 0 else 0 for l in seq_lens]
    num_pages = sum(n_pages_per) + 1  # one spare page never referenced
    perm = torch.randperm(num_pages, generator=g) if shuffle_pages else torch.arange(num_pages)
    kv_indptr = [0]
    kv_indices = []
    last = []
    cursor = 0
    for l, npg in zip(seq_lens, n_pages_per):
        kv_indices += perm[cursor:cursor + npg].tolist()
        cursor += npg
        kv_indptr.append(len(kv_indices))
        last.append(l - (npg - 1) * page if npg else 0)
    b = len(seq_lens)
    q = torch.randn(b, heads, 576, generator=g).to(torch.bfloat16)
    kv_c = torch.randn(num_pages * page, 512, generator=g).to(torch.bfloat16)
    k_pe = torch.randn(num_pages * page, 64, generator=g).to(torch.bfloat16)
    nib, sc = quant_inline(kv_c)
    rope_bytes = k_pe.contiguous().view(torch.uint8).reshape(-1, 128)
    kv_buffer = torch.cat([nib, rope_bytes], dim=1).reshape(num_pages, page, 384)
    kv_scales = sc.reshape(num_pages, page, 16)
    # reference path: dequant latent (v5) + bf16 rope -> fp32 [T, 576]; token-level page table
    latent = v5._dequant_mxfp4_torch(nib, sc, 512)
    kv_cache = torch.cat([latent, k_pe.float()], dim=1)
    tok_indptr = [0]
    tok_idx = []
    for bi in range(b):
        pages = kv_indices[kv_indptr[bi]:kv_indptr[bi + 1]]
        rows = [p * page + r for p in pages for r in range(page)][:seq_lens[bi]]
        tok_idx += rows
        tok_indptr.append(len(tok_idx))
    out = tmd.reference_mla_decode(q, kv_cache, torch.tensor(tok_indptr, dtype=torch.int32),
                                   torch.tensor(tok_idx, dtype=torch.int64), 512, sm_scale)
    return {
        "q_bits": _bits(q),
        "kv_buffer": kv_buffer.numpy(), "kv_scales": kv_scales.numpy(),
        "kv_indptr": np.array(kv_indptr, np.int32), "kv_indices": np.array(kv_indices, np.int32),
        "kv_last_page_len": np.array(last, np.int32), "sm_scale": np.float64(sm_scale),
        "out": out.numpy(),
    }


def make_decode(v5, tmd, quant_inline) -> dict:
    cases = {
        # CPU plumbing shape: batch 2, 16 heads, ctx 512, contiguous pages, sm_scale 1/sqrt(192)
        "plumbing": dict(seed=0, seq_lens=[512, 512], heads=16, sm_scale=1 / math.sqrt(192),
                         shuffle_pages=False),
        # ragged lengths of tests/test_triton_mla_decode.py:184 with shuffled pages, 8 heads
        "ragged": dict(seed=123, seq_lens=[32, 128, 1, 64], heads=8, sm_scale=1 / math.sqrt(576),
                       shuffle_pages=True),
        # an empty sequence, a one-token tail page, a page-and-two, 64 heads
        "tails": dict(seed=7, seq_lens=[0, 65, 130], heads=64, sm_scale=1 / math.sqrt(192),
                      shuffle_pages=True),
    }
    out = {}
    for name, kw in cases.items():
        for k, v in _decode_case(v5, tmd, quant_inline, **kw).items():
            out[f"{name}__{k}"] = v
    out["cases"] = np.array(list(cases.keys()))
    return out


def main():
    root = sys.argv[1] if len(sys.argv) > 1 else "/root/reference"
    v5, tmd, quant_inline = _load_reference(root)
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    np.savez_compressed(os.path.join(HERE, "quant_golden.npz"), **make_quant(quant_inline, v5))
    np.savez_compressed(os.path.join(HERE, "dequant_golden.npz"), **make_dequant(v5))
    np.savez_compressed(os.path.join(HERE, "decode_golden.npz"), **make_decode(v5, tmd, quant_inline))
    print("wrote", sorted(f for f in os.listdir(HERE) if f.endswith(".npz")))


if __name__ == "__main__":
    main()
