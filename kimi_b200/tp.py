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
  (CUDA IPC handles exchanged through ``torch.distributed``, each opened with
  the reading GPU current, so that GPU's kernels may read it) and orders the
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

    ``inputs``: 1..8 partials in rank order, each a bf16 [rows, hidden]
    contiguous CUDA tensor or the integer device address of one (a peer's
    buffer mapped into this process, as :class:`PeerPartials` gives), readable
    from the residual's GPU; ``residual`` bf16 [rows, hidden] contiguous,
    ``weight`` bf16 [hidden].  ``residual_out`` may be ``residual`` itself.
    """
    dev = _require_cuda(residual, weight)
    if residual.dim() != 2 or residual.dtype != torch.bfloat16 or not residual.is_contiguous():
        raise ValueError("residual must be a contiguous bf16 [rows, hidden] tensor")
    rows, hidden = residual.shape
    input_ptrs = []
    for t in inputs:
        if isinstance(t, int):
            input_ptrs.append(t)
            continue
        if t.dtype != torch.bfloat16 or t.shape != (rows, hidden) or not t.is_contiguous() or t.device.type != "cuda":
            raise ValueError("inputs must be contiguous bf16 CUDA tensors of the residual's shape [rows, hidden]")
        input_ptrs.append(t.data_ptr())
    if not 1 <= len(input_ptrs) <= _lib.AR_MAX_INPUTS:
        raise ValueError(f"1..{_lib.AR_MAX_INPUTS} inputs")
    if weight.dtype != torch.bfloat16 or weight.shape != (hidden,) or not weight.is_contiguous():
        raise ValueError("weight must be a contiguous bf16 [hidden] tensor")
    if residual_out is None:
        residual_out = torch.empty_like(residual)
    if nibbles is None:
        nibbles = torch.empty(rows, hidden // 2, dtype=torch.uint8, device=dev)
    if scales is None:
        scales = torch.empty(rows, hidden // 32, dtype=torch.uint8, device=dev)
    p = _lib.KimiArRmsNormParams()
    for i, ptr in enumerate(input_ptrs):
        p.inputs[i] = int(ptr)
    p.num_inputs = len(input_ptrs)
    p.residual, p.residual_out, p.weight = residual.data_ptr(), residual_out.data_ptr(), weight.data_ptr()
    p.eps = float(eps)
    p.nibbles, p.scales = nibbles.data_ptr(), scales.data_ptr()
    p.rows, p.hidden, p.legacy_rule = rows, hidden, int(bool(legacy_rule))
    with torch.cuda.device(dev):
        status = _lib.load().kimi_ar_rmsnorm_mxfp4(ctypes.byref(p), _stream_handle(dev))
    _lib.check(status, "kimi_ar_rmsnorm_mxfp4")
    return residual_out, nibbles, scales


def _check_cuda(err, what):
    if int(err) != 0:
        raise RuntimeError(f"{what} failed: CUDA error {int(err)}")


class CudaIpc:
    """The CUDA IPC calls :class:`PeerPartials` makes (cuda-python bindings).

    ``export(ptr)`` names the allocation a device pointer lies in:
    ``(handle bytes, offset of ptr in it)``.  ``open(handle)`` maps a peer's
    allocation into the CURRENT device's context and returns its base address;
    ``close(base)`` unmaps it.  ``make_current(device)`` selects the device
    whose context the mappings go into.
    """

    def export(self, ptr: int):
        from cuda.bindings import driver, runtime
        err, base, _ = driver.cuMemGetAddressRange(driver.CUdeviceptr(ptr))
        _check_cuda(err, "cuMemGetAddressRange")
        err, handle = runtime.cudaIpcGetMemHandle(int(base))
        _check_cuda(err, "cudaIpcGetMemHandle")
        return bytes(handle.reserved), ptr - int(base)

    def make_current(self, device: torch.device):
        from cuda.bindings import runtime
        err, = runtime.cudaSetDevice(device.index)
        _check_cuda(err, "cudaSetDevice")

    def open(self, raw: bytes) -> int:
        from cuda.bindings import runtime
        h = runtime.cudaIpcMemHandle_t()
        h.reserved = raw
        err, base = runtime.cudaIpcOpenMemHandle(h, runtime.cudaIpcMemLazyEnablePeerAccess)
        _check_cuda(err, "cudaIpcOpenMemHandle")
        return int(base)

    def close(self, base: int):
        from cuda.bindings import runtime
        err, = runtime.cudaIpcCloseMemHandle(base)
        _check_cuda(err, "cudaIpcCloseMemHandle")

    def synchronize(self, device: torch.device):
        torch.cuda.synchronize(device)


class PeerPartials:
    """One partial buffer bf16 [rows, hidden] per rank, mapped into every rank.

    Collective constructor (every rank of ``group`` calls it with the same
    shape): each rank allocates its buffer, and the buffers' CUDA IPC handles
    are exchanged with ``all_gather_object``.  ``local`` is this rank's buffer
    (the o_proj output is written there); ``ptrs`` are every rank's buffer as
    device addresses this rank's GPU reads (rank order);
    :meth:`reduce_norm_quant` runs the fused kernel over them between two
    barriers; :meth:`close` (collective) unmaps the peers' buffers.  ``ipc``
    is the IPC layer (:class:`CudaIpc` unless another is given).
    """

    def __init__(self, rows: int, hidden: int, device: torch.device, group=None, ipc=None):
        import torch.distributed as dist

        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > _lib.AR_MAX_INPUTS:
            raise ValueError(f"at most {_lib.AR_MAX_INPUTS} ranks")
        self.ipc = ipc if ipc is not None else CudaIpc()
        self.device = torch.device(device)
        self.rows, self.hidden = rows, hidden
        self.local = torch.zeros(rows, hidden, dtype=torch.bfloat16, device=self.device)
        ptr = self.local.data_ptr()
        # Every rank joins the gather even when its export failed (an
        # allocation from PYTORCH_CUDA_ALLOC_CONF=expandable_segments has no
        # IPC handle, for one): each sends (ok, payload) and all of them raise
        # together, instead of the peers waiting out the group's timeout.
        try:
            mine = (True, self.ipc.export(ptr))
        except Exception as e:  # noqa: BLE001 - reported to every rank below
            mine = (False, f"{type(e).__name__}: {e}")
        shared = [None] * self.world
        dist.all_gather_object(shared, mine, group=group)
        failed = [(r, msg) for r, (ok, msg) in enumerate(shared) if not ok]
        if failed:
            raise RuntimeError("PeerPartials: IPC export failed on rank(s) " +
                               "; ".join(f"{r}: {msg}" for r, msg in failed))
        # open every peer's allocation with this rank's GPU current: the mapping
        # (and the peer access it enables) belongs to this GPU's context
        self.ipc.make_current(self.device)
        self._opened, self.ptrs = [], []
        try:
            for r, (_, (raw, offset)) in enumerate(shared):
                if r == self.rank:
                    self.ptrs.append(ptr)
                    continue
                base = self.ipc.open(raw)
                self._opened.append(base)
                self.ptrs.append(base + offset)
        except Exception:
            self._unmap()
            raise

    def _unmap(self):
        """Close every mapping this rank opened; the first failure is raised
        once all of them have been tried."""
        first = None
        for b in self._opened:
            try:
                self.ipc.close(b)
            except Exception as e:  # noqa: BLE001 - re-raised below
                first = first or e
        self._opened, self.ptrs = [], []
        if first is not None:
            raise first

    def close(self):
        """Unmap the peers' buffers (collective: call on every rank once no
        kernel reads them any more).  Every rank reaches the closing barrier
        even when an unmap failed; the failure is raised after it."""
        self.ipc.synchronize(self.device)
        err = None
        try:
            self._unmap()
        except Exception as e:  # noqa: BLE001 - re-raised after the barrier
            err = e
        self._barrier()
        if err is not None:
            raise err

    def _barrier(self):
        import torch.distributed as dist
        # stream-ordered: an all-reduce of one element on the current stream
        t = torch.zeros(1, device=self.device)
        dist.all_reduce(t, group=self.group)

    def reduce_norm_quant(self, residual: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6,
                          residual_out: torch.Tensor | None = None, legacy_rule: bool = False):
        """All-reduce of the ranks' ``local`` buffers + residual + RMSNorm +
        MXFP4 (every rank computes the full result for its own use) over the
        first ``residual.shape[0]`` rows of every rank's buffer."""
        if residual.dim() != 2 or residual.shape[0] > self.rows or residual.shape[1] != self.hidden:
            raise ValueError(f"residual must be [<= {self.rows}, {self.hidden}]")
        if not self.ptrs:
            raise RuntimeError("PeerPartials is closed")
        self._barrier()  # every rank's partial is written
        out = ar_rmsnorm_mxfp4(self.ptrs, residual, weight, eps, residual_out=residual_out, legacy_rule=legacy_rule)
        self._barrier()  # every rank has read every partial
        return out
