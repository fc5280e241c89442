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
* :class:`PeerPartials` maps every rank's exchange buffer (its partial, the
  two-shot outputs and flag words) into every rank (CUDA IPC handles
  exchanged through ``torch.distributed``, each opened with the reading GPU
  current, so that GPU's kernels may read it).  Two forms:

  - :meth:`PeerPartials.reduce_norm_quant` (one-shot): every rank reads every
    partial whole; the kernel waits for nothing, so it runs between two
    stream-ordered barriers (the partials are complete before any rank reads
    them, and no rank overwrites its partial until every rank has read it);
  - :meth:`PeerPartials.reduce_norm_quant_two_shot`: rank r reduces, norms
    and quantises 1 / N of the rows from all partials and stores them into
    every rank's outputs (``kimi_ar_rmsnorm_mxfp4_two_shot``), with the two
    barriers done on the device over flag words in peer memory.
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


def _exchange_layout(rows: int, hidden: int) -> dict:
    """Byte offsets of the regions of a rank's exchange buffer."""
    a16 = lambda n: (n + 15) // 16 * 16
    off, pos = {}, 0
    for name, nbytes in (("partial", rows * hidden * 2), ("residual_out", rows * hidden * 2),
                         ("nibbles", rows * hidden // 2), ("scales", rows * hidden // 32),
                         ("flags", 2 * _lib.AR_MAX_INPUTS * 4)):
        off[name] = pos
        pos += a16(nbytes)
    off["total"] = pos
    return off


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
    """One exchange buffer per rank, mapped into every rank.

    Collective constructor (every rank of ``group`` calls it with the same
    shape): each rank allocates its buffer -- its partial bf16 [rows, hidden],
    the two-shot outputs (``residual_out``, ``nibbles``, ``scales``) and its
    flag words -- and the buffers' CUDA IPC handles are exchanged with
    ``all_gather_object``.  ``local`` is this rank's partial (the o_proj
    output is written there); ``ptrs`` are every rank's partial and ``bases``
    every rank's buffer, as device addresses this rank's GPU reads (rank
    order).  :meth:`reduce_norm_quant` runs the one-shot kernel between two
    host-ordered barriers, :meth:`reduce_norm_quant_two_shot` the two-shot
    kernel with its device barriers; :meth:`close` (collective) unmaps the
    peers' buffers.  ``ipc`` is the IPC layer (:class:`CudaIpc` unless
    another is given).
    """

    def __init__(self, rows: int, hidden: int, device: torch.device, group=None, ipc=None):
        import torch.distributed as dist

        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > _lib.AR_MAX_INPUTS:
            raise ValueError(f"at most {_lib.AR_MAX_INPUTS} ranks")
        if hidden % 32:
            raise ValueError("hidden must be a multiple of 32")
        self.ipc = ipc if ipc is not None else CudaIpc()
        self.device = torch.device(device)
        self.rows, self.hidden = rows, hidden
        # one allocation (one IPC handle): the partial, then the two-shot
        # outputs and this rank's flag words, each region 16-byte aligned
        self._off = _exchange_layout(rows, hidden)
        self.buffer = torch.zeros(self._off["total"], dtype=torch.uint8, device=self.device)
        self.local = self._region("partial", torch.bfloat16, (rows, hidden))
        self.residual_out = self._region("residual_out", torch.bfloat16, (rows, hidden))
        self.nibbles = self._region("nibbles", torch.uint8, (rows, hidden // 2))
        self.scales = self._region("scales", torch.uint8, (rows, hidden // 32))
        # this rank's two-shot counter words (CTA count, call number) and its
        # device status word (not shared)
        self._words = torch.zeros(4, dtype=torch.int32, device=self.device)
        self.status = self._words[2:3]
        ptr = self.buffer.data_ptr()
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
        self._opened, self.ptrs, self.bases = [], [], []
        try:
            for r, (_, (raw, offset)) in enumerate(shared):
                if r == self.rank:
                    self.bases.append(ptr)
                else:
                    base = self.ipc.open(raw)
                    self._opened.append(base)
                    self.bases.append(base + offset)
                self.ptrs.append(self.bases[-1] + self._off["partial"])
        except Exception:
            self._unmap()
            raise

    def _region(self, name: str, dtype: torch.dtype, shape) -> torch.Tensor:
        n = 1
        for d in shape:
            n *= d
        start = self._off[name]
        return self.buffer[start:start + n * torch.empty(0, dtype=dtype).element_size()].view(dtype).view(*shape)

    def _unmap(self):
        """Close every mapping this rank opened; the first failure is raised
        once all of them have been tried."""
        first = None
        for b in self._opened:
            try:
                self.ipc.close(b)
            except Exception as e:  # noqa: BLE001 - re-raised below
                first = first or e
        self._opened, self.ptrs, self.bases = [], [], []
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

    def reduce_norm_quant_two_shot(self, residual: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6,
                                   legacy_rule: bool = False, timeout_ns: int = 0):
        """The same result as :meth:`reduce_norm_quant` for the first
        ``residual.shape[0]`` rows, as a two-shot exchange: this rank reduces
        1 / N of the rows from every partial and stores them into every rank's
        outputs, the ranks meeting at two device barriers (no host barrier).
        Collective: every rank calls it, in the same order, with the same
        shapes (the call numbers that pair the ranks' barriers live on the
        device, so the call may be captured in a CUDA graph and replayed).
        Returns views of this rank's outputs ``(residual_out [rows,
        hidden], nibbles [rows, hidden/2], scales [rows, hidden/32])``, valid
        until the next call.  A barrier wait that runs out (``timeout_ns``, 0 =
        2 s) sets ``_lib.DEVICE_PEER_WAIT`` in ``self.status`` (read it with
        :func:`kimi_b200.device_status`); the exchange is then to be set up
        anew."""
        rows = residual.shape[0] if residual.dim() == 2 else -1
        if rows < 0 or rows > self.rows or residual.shape[1] != self.hidden:
            raise ValueError(f"residual must be [<= {self.rows}, {self.hidden}]")
        if residual.dtype != torch.bfloat16 or not residual.is_contiguous():
            raise ValueError("residual must be a contiguous bf16 tensor")
        if weight.dtype != torch.bfloat16 or weight.shape != (self.hidden,) or not weight.is_contiguous():
            raise ValueError("weight must be a contiguous bf16 [hidden] tensor")
        if not self.bases:
            raise RuntimeError("PeerPartials is closed")
        p = _lib.KimiArTwoShotParams()
        for r, base in enumerate(self.bases):
            p.inputs[r] = base + self._off["partial"]
            p.residual_out[r] = base + self._off["residual_out"]
            p.nibbles[r] = base + self._off["nibbles"]
            p.scales[r] = base + self._off["scales"]
            p.flags[r] = base + self._off["flags"]
        p.counter = self._words.data_ptr()
        p.residual, p.weight = residual.data_ptr(), weight.data_ptr()
        p.eps = float(eps)
        p.rows, p.hidden, p.legacy_rule = rows, self.hidden, int(bool(legacy_rule))
        p.world, p.rank = self.world, self.rank
        p.status = self.status.data_ptr()
        p.timeout_ns = int(timeout_ns)
        with torch.cuda.device(self.device):
            st = _lib.load().kimi_ar_rmsnorm_mxfp4_two_shot(ctypes.byref(p), _stream_handle(self.device))
        _lib.check(st, "kimi_ar_rmsnorm_mxfp4_two_shot")
        return self.residual_out[:rows], self.nibbles[:rows], self.scales[:rows]
