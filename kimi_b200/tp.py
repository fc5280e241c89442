"""Tensor-parallel layer-input step: all-reduce of the ranks' partial hidden
states + residual + RMSNorm + MXFP4 quantisation in one kernel.

The reference fuses the one-shot all-reduce with the residual add and
RMSNorm in a custom all-reduce kernel that reads every rank's buffer over
the GPU links (patches/aiter-1stage-nloop-ar-rmsnorm.patch:12-253), then
quantises the normed rows to MXFP4 (patches/aiter-mxfp4-quant-only.patch:29-125).
Here one kernel (``kimi_ar_rmsnorm_mxfp4`` of include/kimi_mla.h) does all
of it, reading the ranks' partials straight from their buffers.

* :func:`ar_rmsnorm_mxfp4` runs the kernel on a list of partial buffers the
  current GPU can read (its own, and peers' mapped over NVLink).
* :class:`PeerPartials` maps every rank's partial buffer into every rank
  (CUDA IPC handles exchanged through ``torch.distributed``) and orders the
  kernel between two stream-ordered barriers: the partials are complete
  before any rank reads them, and no rank overwrites its partial until every
  rank has read it.  The kernel itself waits for nothing.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .mla import _require_cuda, _stream_handle


def ar_rmsnorm_mxfp4(inputs, residual: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6,
                     residual_out: torch.Tensor | None = None, nibbles: torch.Tensor | None = None,
                     scales: torch.Tensor | None = None, legacy_rule: bool = False):
    """``residual_out = bf16(sum(inputs) + residual)`` (float32 sum in list
    order), ``out = bf16(bf16(residual_out * rsqrt(mean(residual_out^2) + eps))
    * weight)``, and ``out`` quantised to MXFP4: returns ``(residual_out,
    nibbles uint8 [rows, hidden/2], scales uint8 [rows, hidden/32])``.

    ``inputs``: 1..8 bf16 [rows, hidden] contiguous tensors (rank order) the
    residual's GPU can read; ``residual`` bf16 [rows, hidden] contiguous,
    ``weight`` bf16 [hidden].  ``residual_out`` may be ``residual`` itself.
    """
    dev = _require_cuda(residual, weight)
    inputs = list(inputs)
    if not 1 <= len(inputs) <= _lib.AR_MAX_INPUTS:
        raise ValueError(f"1..{_lib.AR_MAX_INPUTS} inputs")
    rows, hidden = residual.shape
    for t in inputs + [residual]:
        if t.dtype != torch.bfloat16 or t.shape != (rows, hidden) or not t.is_contiguous() or t.device.type != "cuda":
            raise ValueError("inputs and residual must be contiguous bf16 CUDA tensors of one shape [rows, hidden]")
    if weight.dtype != torch.bfloat16 or weight.shape != (hidden,) or not weight.is_contiguous():
        raise ValueError("weight must be a contiguous bf16 [hidden] tensor")
    if residual_out is None:
        residual_out = torch.empty_like(residual)
    if nibbles is None:
        nibbles = torch.empty(rows, hidden // 2, dtype=torch.uint8, device=dev)
    if scales is None:
        scales = torch.empty(rows, hidden // 32, dtype=torch.uint8, device=dev)
    p = _lib.KimiArRmsNormParams()
    for i, t in enumerate(inputs):
        p.inputs[i] = t.data_ptr()
    p.num_inputs = len(inputs)
    p.residual, p.residual_out, p.weight = residual.data_ptr(), residual_out.data_ptr(), weight.data_ptr()
    p.eps = float(eps)
    p.nibbles, p.scales = nibbles.data_ptr(), scales.data_ptr()
    p.rows, p.hidden, p.legacy_rule = rows, hidden, int(bool(legacy_rule))
    with torch.cuda.device(dev):
        status = _lib.load().kimi_ar_rmsnorm_mxfp4(ctypes.byref(p), _stream_handle(dev))
    _lib.check(status, "kimi_ar_rmsnorm_mxfp4")
    return residual_out, nibbles, scales


class PeerPartials:
    """One partial buffer bf16 [rows, hidden] per rank, mapped into every rank.

    Collective constructor (every rank of ``group`` calls it with the same
    shape): each rank allocates its buffer, and the buffers' CUDA IPC handles
    are exchanged with ``all_gather_object``.  ``local`` is this rank's buffer
    (the o_proj output is written there); :meth:`reduce_norm_quant` runs the
    fused kernel over all ranks' buffers between two barriers.
    """

    def __init__(self, rows: int, hidden: int, device: torch.device, group=None):
        import torch.distributed as dist
        from torch.multiprocessing.reductions import reduce_tensor

        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > _lib.AR_MAX_INPUTS:
            raise ValueError(f"at most {_lib.AR_MAX_INPUTS} ranks")
        self.local = torch.zeros(rows, hidden, dtype=torch.bfloat16, device=device)
        handles = [None] * self.world
        dist.all_gather_object(handles, reduce_tensor(self.local), group=group)
        self.buffers = []
        for r, (fn, args) in enumerate(handles):
            self.buffers.append(self.local if r == self.rank else fn(*args))
        self.device = device

    def _barrier(self):
        import torch.distributed as dist
        # stream-ordered: an all-reduce of one element on the current stream
        t = torch.zeros(1, device=self.device)
        dist.all_reduce(t, group=self.group)

    def reduce_norm_quant(self, residual: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6,
                          residual_out: torch.Tensor | None = None, legacy_rule: bool = False):
        """All-reduce of the ranks' ``local`` buffers + residual + RMSNorm +
        MXFP4 (every rank computes the full result for its own use)."""
        self._barrier()  # every rank's partial is written
        out = ar_rmsnorm_mxfp4(self.buffers, residual, weight, eps, residual_out=residual_out,
                               legacy_rule=legacy_rule)
        self._barrier()  # every rank has read every partial
        return out
