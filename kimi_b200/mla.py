"""Host-side operator API of the MXFP4 MLA decode path.

Mirrors the reference's operator interface (paths inside ianye23301/kimi):

* :func:`mla_decode_fwd` -- aiter ``mla_decode_fwd(q, kv_buffer, o, qo_indptr,
  kv_indptr, kv_indices, kv_last_page_len, max_seqlen_q, page_size, nhead_kv,
  sm_scale, logit_cap, num_kv_splits, ...)`` as called at
  scripts/submission.py:115-133 and patches/atom-optimizations.patch:741-748,
  with the MXFP4 cache's scale tensor ``kv_scales`` next to ``kv_buffer``.
  Writes ``o`` in place on the current stream (``o`` may be the heads-first
  view ``o_hf.permute(1, 0, 2)``, patches/atom-optimizations.patch:261-289).
* :func:`mxfp4_kv_append` -- the cache writer
  ``fused_qk_rope_concat_and_cache_mla(..., slot_mapping, ...)``
  (patches/atom-optimizations.patch:615-634) with the MXFP4 quantiser.
* :func:`mxfp4_quantize` -- aiter ``dynamic_mxfp4_quant``
  (archive/mla-mxfp4-dead-end/mla_decode_mxfp4.py:139-156).
* :func:`mla_reduce` -- the split-K merge ``_mla_reduce``
  (archive/mla-mxfp4-dead-end/mla_decode_mxfp4_v5.py:264-306).

Errors are Python exceptions (``ValueError`` for bad arguments, as the
reference's asserts, ``RuntimeError`` for CUDA failures).  Every call runs the
CUDA kernels of ``libkimi_mla.so``; there is no other path.
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _lib

KV_LORA_RANK = 512
ROPE_DIM = 64
QK_DIM = KV_LORA_RANK + ROPE_DIM
PAGE_SIZE = 64
TOKEN_BYTES = 384
SCALE_BYTES = 16


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(*tensors: torch.Tensor) -> torch.device:
    dev = tensors[0].device
    if dev.type != "cuda":
        raise ValueError("kimi_b200 kernels run on CUDA tensors only")
    for t in tensors:
        if t is not None and t.device != dev:
            raise ValueError("all tensors must be on the same CUDA device")
    return dev


def _cache_views(kv_buffer: torch.Tensor, kv_scales: torch.Tensor):
    """Accept [pages, 64, 384] / [pages, 64, 1, 384] (and the same for scales)."""
    if kv_buffer.dtype != torch.uint8 or kv_scales.dtype != torch.uint8:
        raise ValueError("kv_buffer and kv_scales must be uint8")
    if not kv_buffer.is_contiguous() or not kv_scales.is_contiguous():
        raise ValueError("kv_buffer and kv_scales must be contiguous")
    if kv_buffer.numel() % (PAGE_SIZE * TOKEN_BYTES) or kv_buffer.shape[-1] != TOKEN_BYTES:
        raise ValueError(f"kv_buffer must be [num_pages, {PAGE_SIZE}, {TOKEN_BYTES}] uint8")
    num_pages = kv_buffer.numel() // (PAGE_SIZE * TOKEN_BYTES)
    if kv_scales.numel() != num_pages * PAGE_SIZE * SCALE_BYTES or kv_scales.shape[-1] != SCALE_BYTES:
        raise ValueError(f"kv_scales must be [num_pages, {PAGE_SIZE}, {SCALE_BYTES}] uint8")
    return num_pages


def alloc_mxfp4_cache(num_pages: int, device, zero: bool = True):
    """A paged MXFP4 latent cache: ``(kv_buffer [P, 64, 384] u8, kv_scales [P, 64, 16] u8)``."""
    make = torch.zeros if zero else torch.empty
    return (make(num_pages, PAGE_SIZE, TOKEN_BYTES, dtype=torch.uint8, device=device),
            make(num_pages, PAGE_SIZE, SCALE_BYTES, dtype=torch.uint8, device=device))


def num_kv_splits_for(batch: int, num_heads: int, num_kv_splits: int | None = None) -> int:
    """The split count the decode uses (``None``/0 = automatic)."""
    return int(_lib.load().kimi_mla_decode_num_splits(batch, num_heads, int(num_kv_splits or 0)))


def workspace_bytes(batch: int, num_heads: int, num_kv_splits: int | None = None) -> int:
    return int(_lib.load().kimi_mla_decode_workspace_size(batch, num_heads, int(num_kv_splits or 0)))


def alloc_workspace(batch: int, num_heads: int, num_kv_splits: int | None, device) -> torch.Tensor:
    """Preallocate the split-K workspace (for CUDA-graph capture: allocate once,
    pass it to every :func:`mla_decode_fwd` call of that shape)."""
    n = workspace_bytes(batch, num_heads, num_kv_splits)
    return torch.empty(max(n, 256), dtype=torch.uint8, device=device)


_ws_cache: dict = {}


def _default_workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    key = (device.type, device.index)
    buf = _ws_cache.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _ws_cache[key] = buf
    return buf


def _run_decode(entry: str, q, kv_buffer, kv_scales, o, qo_indptr, kv_indptr, kv_indices, kv_last_page_len,
                max_seqlen_q, page_size, nhead_kv, sm_scale, logit_cap, num_kv_splits, workspace,
                status=None, timeout_ns=0):
    """Checks the arguments, fills the C-ABI params and calls ``entry``."""
    dev = _require_cuda(q, kv_buffer, kv_scales, o, kv_indptr, kv_indices)
    if status is not None:
        _require_status_word(status, dev)
    if max_seqlen_q != 1:
        raise ValueError("mla_decode_fwd supports one query token per sequence (max_seqlen_q == 1)")
    if page_size != PAGE_SIZE:
        raise ValueError(f"page_size must be {PAGE_SIZE}")
    if nhead_kv != 1:
        raise ValueError("MLA has one latent KV head (nhead_kv == 1)")
    if q.dtype != torch.bfloat16 or o.dtype != torch.bfloat16:
        raise ValueError("q and o must be bfloat16")
    if q.dim() != 3 or q.shape[2] != QK_DIM or q.stride(2) != 1:
        raise ValueError(f"q must be [batch, heads, {QK_DIM}] with a contiguous last dim")
    batch, heads = q.shape[0], q.shape[1]
    if o.dim() != 3 or tuple(o.shape) != (batch, heads, KV_LORA_RANK) or o.stride(2) != 1:
        raise ValueError(f"o must be [batch, heads, {KV_LORA_RANK}] with a contiguous last dim")
    if qo_indptr is not None and qo_indptr.numel() != batch + 1:
        raise ValueError("qo_indptr must have batch + 1 entries")
    for name, t in (("kv_indptr", kv_indptr), ("kv_indices", kv_indices), ("kv_last_page_len", kv_last_page_len)):
        if t is not None and (t.dtype != torch.int32 or not t.is_contiguous()):
            raise ValueError(f"{name} must be a contiguous int32 tensor")
    if kv_indptr.numel() != batch + 1:
        raise ValueError("kv_indptr must have batch + 1 entries")
    if kv_last_page_len is not None and kv_last_page_len.numel() != batch:
        raise ValueError("kv_last_page_len must have batch entries")
    num_pages = _cache_views(kv_buffer, kv_scales)
    scale = (1.0 / math.sqrt(QK_DIM)) if sm_scale is None else float(sm_scale)
    lib = _lib.load()
    splits_req = int(num_kv_splits or 0)
    need = int(lib.kimi_mla_decode_workspace_size(batch, heads, splits_req))
    if need:
        if workspace is None:
            workspace = _default_workspace(need, dev)
        elif workspace.device != dev or workspace.numel() * workspace.element_size() < need:
            raise ValueError(f"workspace must hold at least {need} bytes on {dev}")
    p = _lib.KimiMlaDecodeParams(
        q=q.data_ptr(), q_stride_b=q.stride(0), q_stride_h=q.stride(1),
        kv_buffer=kv_buffer.data_ptr(), kv_scales=kv_scales.data_ptr(), num_pages=num_pages,
        kv_indptr=kv_indptr.data_ptr(), kv_indices=kv_indices.data_ptr() if kv_indices.numel() else None,
        kv_last_page_len=_ptr(kv_last_page_len),
        o=o.data_ptr(), o_stride_b=o.stride(0), o_stride_h=o.stride(1),
        batch=batch, num_heads=heads, num_kv_splits=splits_req,
        sm_scale=scale, logit_cap=float(logit_cap), status=_ptr(status), timeout_ns=int(timeout_ns))
    if p.kv_indices is None and batch:
        # an all-empty batch still needs a valid pointer; the kernel never reads past kv_indptr
        p.kv_indices = kv_indptr.data_ptr()
    ws_ptr = workspace.data_ptr() if (need and workspace is not None) else None
    ws_bytes = workspace.numel() * workspace.element_size() if (need and workspace is not None) else 0
    with torch.cuda.device(dev):
        status = getattr(lib, entry)(ctypes.byref(p), ws_ptr, ws_bytes, _stream_handle(dev))
    _lib.check(status, entry)
    return o


def mla_decode_fwd(q: torch.Tensor, kv_buffer: torch.Tensor, kv_scales: torch.Tensor, o: torch.Tensor,
                   qo_indptr: torch.Tensor | None, kv_indptr: torch.Tensor, kv_indices: torch.Tensor,
                   kv_last_page_len: torch.Tensor | None, max_seqlen_q: int = 1, page_size: int = PAGE_SIZE,
                   nhead_kv: int = 1, sm_scale: float | None = None, logit_cap: float = 0.0,
                   num_kv_splits: int | None = None, workspace: torch.Tensor | None = None,
                   status: torch.Tensor | None = None, timeout_ns: int = 0) -> torch.Tensor:
    """Absorbed-MLA decode over the paged MXFP4 latent cache; writes ``o``.

    q            bf16 [batch, num_heads, 576] (rows may be strided; last dim contiguous)
    kv_buffer    uint8 [num_pages, 64, 384] (nibbles of the 512-dim latent, then bf16 RoPE)
    kv_scales    uint8 [num_pages, 64, 16]  (e8m0, one per 32 latent elements)
    o            bf16 [batch, num_heads, 512], any (batch, head) strides
    kv_indptr    int32 [batch + 1] page offsets; kv_indices int32 page ids;
    kv_last_page_len int32 [batch] tokens in each last page (None = full pages)
    sm_scale     softmax scale (default 1/sqrt(576))
    num_kv_splits equal split-K ranges per sequence (the reference's meaning),
                 or None / 0 for the balanced schedule over all SMs;
                 workspace optional uint8 buffer of at least :func:`workspace_bytes`
    status       optional int32 [1] device word: the kernels OR KIMI_DEVICE_* bits
                 into it when a bounded device wait gives up or a page id lies
                 outside the cache (read it with :func:`device_status`)
    timeout_ns   bound of each device-side wait (0 = the library default, 2 s)
    """
    return _run_decode("kimi_mla_decode", q, kv_buffer, kv_scales, o, qo_indptr, kv_indptr, kv_indices,
                       kv_last_page_len, max_seqlen_q, page_size, nhead_kv, sm_scale, logit_cap, num_kv_splits,
                       workspace, status, timeout_ns)


def mla_decode_partial(q, kv_buffer, kv_scales, o, qo_indptr, kv_indptr, kv_indices, kv_last_page_len,
                       max_seqlen_q: int = 1, page_size: int = PAGE_SIZE, nhead_kv: int = 1,
                       sm_scale: float | None = None, logit_cap: float = 0.0, num_kv_splits: int | None = None,
                       workspace: torch.Tensor | None = None, status: torch.Tensor | None = None,
                       timeout_ns: int = 0) -> torch.Tensor:
    """The split-K attention launch of :func:`mla_decode_fwd` alone (the
    archive's ``_mla_decode_split_kv``); pair it with :func:`mla_decode_merge`
    on the same arguments and workspace."""
    return _run_decode("kimi_mla_decode_partial", q, kv_buffer, kv_scales, o, qo_indptr, kv_indptr, kv_indices,
                       kv_last_page_len, max_seqlen_q, page_size, nhead_kv, sm_scale, logit_cap, num_kv_splits,
                       workspace, status, timeout_ns)


def mla_decode_merge(q, kv_buffer, kv_scales, o, qo_indptr, kv_indptr, kv_indices, kv_last_page_len,
                     max_seqlen_q: int = 1, page_size: int = PAGE_SIZE, nhead_kv: int = 1,
                     sm_scale: float | None = None, logit_cap: float = 0.0, num_kv_splits: int | None = None,
                     workspace: torch.Tensor | None = None) -> torch.Tensor:
    """The log-sum-exp merge launch of :func:`mla_decode_fwd` alone (the
    archive's ``_mla_reduce``), after :func:`mla_decode_partial`."""
    return _run_decode("kimi_mla_decode_merge", q, kv_buffer, kv_scales, o, qo_indptr, kv_indptr, kv_indices,
                       kv_last_page_len, max_seqlen_q, page_size, nhead_kv, sm_scale, logit_cap, num_kv_splits,
                       workspace)


def _require_status_word(status: torch.Tensor, dev: torch.device) -> None:
    if status.dtype != torch.int32 or status.numel() != 1 or status.device != dev:
        raise ValueError(f"status must be an int32 tensor of one element on {dev}")


def device_status(status: torch.Tensor, clear: bool = False) -> int:
    """The KIMI_DEVICE_* bits in a decode status word (0 = none), read after
    the work queued on the current stream (this waits for it).  ``clear``
    resets the word afterwards."""
    dev = _require_cuda(status)
    _require_status_word(status, dev)
    with torch.cuda.device(dev):
        st = _lib.load().kimi_device_status(status.data_ptr(), int(bool(clear)), _stream_handle(dev))
    if st >= _lib.KIMI_ERR_CUDA_BASE or st < 0:
        _lib.check(st, "kimi_device_status")
    return int(st)


def check_device_status(status: torch.Tensor, clear: bool = False) -> None:
    """Raise ``RuntimeError`` when a decode recorded a device-side failure in
    ``status`` (a wait that gave up, or a page id outside the cache)."""
    st = device_status(status, clear)
    if st:
        raise RuntimeError(f"MLA decode reported a device-side failure: {_lib.status_text(st)} (bits {st:#x})")


def mla_reduce(partial_o: torch.Tensor, partial_lse: torch.Tensor, o: torch.Tensor) -> torch.Tensor:
    """Merge split partials: partial_o f32 [B, S, H, 512], partial_lse f32 [B, S, H]
    (natural log, -inf = empty split) -> bf16 ``o`` [B, H, 512] (any strides)."""
    dev = _require_cuda(partial_o, partial_lse, o)
    b, s, h, d = partial_o.shape
    if d != KV_LORA_RANK or tuple(partial_lse.shape) != (b, s, h):
        raise ValueError("partial_o must be [B, S, H, 512] and partial_lse [B, S, H]")
    if partial_o.dtype != torch.float32 or partial_lse.dtype != torch.float32:
        raise ValueError("partials must be float32")
    if not partial_o.is_contiguous() or not partial_lse.is_contiguous():
        raise ValueError("partials must be contiguous")
    if o.dtype != torch.bfloat16 or tuple(o.shape) != (b, h, KV_LORA_RANK) or o.stride(2) != 1:
        raise ValueError("o must be bf16 [B, H, 512] with a contiguous last dim")
    p = _lib.KimiMlaReduceParams(partial_o=partial_o.data_ptr(), partial_lse=partial_lse.data_ptr(),
                                 o=o.data_ptr(), o_stride_b=o.stride(0), o_stride_h=o.stride(1),
                                 batch=b, num_heads=h, num_splits=s)
    with torch.cuda.device(dev):
        status = _lib.load().kimi_mla_reduce(ctypes.byref(p), _stream_handle(dev))
    _lib.check(status, "kimi_mla_reduce")
    return o


def mxfp4_kv_append(kv_c: torch.Tensor, k_pe: torch.Tensor, kv_buffer: torch.Tensor, kv_scales: torch.Tensor,
                    slot_mapping: torch.Tensor, legacy_rule: bool = False) -> None:
    """Quantise ``kv_c`` (bf16 [n, 512]) to MXFP4 and write it, with ``k_pe``
    (bf16 [n, 64]), into the paged cache at ``slot_mapping`` (int64 [n],
    page * 64 + row; negative = skip)."""
    dev = _require_cuda(kv_c, k_pe, kv_buffer, kv_scales, slot_mapping)
    num_pages = _cache_views(kv_buffer, kv_scales)
    if kv_c.dtype != torch.bfloat16 or k_pe.dtype != torch.bfloat16:
        raise ValueError("kv_c and k_pe must be bfloat16")
    if kv_c.dim() != 2 or kv_c.shape[1] != KV_LORA_RANK or kv_c.stride(1) != 1:
        raise ValueError("kv_c must be [n, 512] with a contiguous last dim")
    if k_pe.dim() != 2 or k_pe.shape[1] != ROPE_DIM or k_pe.stride(1) != 1 or k_pe.shape[0] != kv_c.shape[0]:
        raise ValueError("k_pe must be [n, 64] with a contiguous last dim")
    if slot_mapping.dtype != torch.int64 or slot_mapping.numel() != kv_c.shape[0] or not slot_mapping.is_contiguous():
        raise ValueError("slot_mapping must be a contiguous int64 tensor with n entries")
    p = _lib.KimiKvAppendParams(kv_c=kv_c.data_ptr(), kv_c_stride=kv_c.stride(0), k_pe=k_pe.data_ptr(),
                                k_pe_stride=k_pe.stride(0), slot_mapping=slot_mapping.data_ptr(),
                                kv_buffer=kv_buffer.data_ptr(), kv_scales=kv_scales.data_ptr(),
                                num_pages=num_pages, num_tokens=kv_c.shape[0], legacy_rule=int(bool(legacy_rule)))
    with torch.cuda.device(dev):
        status = _lib.load().kimi_mxfp4_kv_append(ctypes.byref(p), _stream_handle(dev))
    _lib.check(status, "kimi_mxfp4_kv_append")


def q_absorb_rope_append(q_nope: torch.Tensor, q_pe: torch.Tensor, w_uk: torch.Tensor, kv_c: torch.Tensor,
                         k_pe: torch.Tensor, positions: torch.Tensor, cos_cache: torch.Tensor,
                         sin_cache: torch.Tensor, kv_buffer: torch.Tensor, kv_scales: torch.Tensor,
                         slot_mapping: torch.Tensor, q_out: torch.Tensor | None = None, is_neox: bool = False,
                         legacy_rule: bool = False, status: torch.Tensor | None = None) -> torch.Tensor:
    """The decode step before attention in one launch (the reference's
    ``fused_kv_bmm``, patches/atom-optimizations.patch:468-639):

    * ``q_out[t, h, :512] = q_nope[t, h] @ w_uk[h]`` (q absorbed by W_UK);
    * ``q_out[t, h, 512:] = rope(q_pe[t, h], positions[t])``;
    * the cache gets MXFP4(``kv_c[t]``) and ``rope(k_pe[t], positions[t])``
      at ``slot_mapping[t]``.

    Shapes: q_nope bf16 [T, H, 128], q_pe bf16 [T, H, 64] (both may be views
    of one [T, H, 192] projection), w_uk bf16 [H, 128, 512] contiguous, kv_c
    bf16 [T, 512], k_pe bf16 [T, 64] before RoPE, positions int64 [T],
    cos_cache / sin_cache float32 [max_position, 32], slot_mapping int64
    [T].  ``q_out`` (bf16 [T, H, 576], allocated when None) is returned and is
    the decode's ``q``.  ``is_neox`` selects the rotary pairing
    (x[i], x[i+32]) instead of (x[2i], x[2i+1]).
    """
    dev = _require_cuda(q_nope, q_pe, w_uk, kv_c, k_pe, positions, cos_cache, sin_cache, kv_buffer, kv_scales,
                        slot_mapping)
    num_pages = _cache_views(kv_buffer, kv_scales)
    for name, t in (("q_nope", q_nope), ("q_pe", q_pe), ("w_uk", w_uk), ("kv_c", kv_c), ("k_pe", k_pe)):
        if t.dtype != torch.bfloat16:
            raise ValueError(f"{name} must be bfloat16")
    if q_nope.dim() != 3 or q_nope.shape[2] != 128 or q_nope.stride(2) != 1:
        raise ValueError("q_nope must be [T, H, 128] with a contiguous last dim")
    T, H = q_nope.shape[0], q_nope.shape[1]
    if q_pe.shape != (T, H, ROPE_DIM) or q_pe.stride(2) != 1:
        raise ValueError("q_pe must be [T, H, 64] with a contiguous last dim")
    if w_uk.shape != (H, 128, KV_LORA_RANK) or not w_uk.is_contiguous():
        raise ValueError("w_uk must be a contiguous [H, 128, 512] tensor")
    if kv_c.shape != (T, KV_LORA_RANK) or kv_c.stride(1) != 1 or k_pe.shape != (T, ROPE_DIM) or k_pe.stride(1) != 1:
        raise ValueError("kv_c must be [T, 512] and k_pe [T, 64], contiguous in the last dim")
    for name, t in (("positions", positions), ("slot_mapping", slot_mapping)):
        if t.dtype != torch.int64 or t.numel() != T or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous int64 tensor with T entries")
    if (cos_cache.dtype != torch.float32 or sin_cache.dtype != torch.float32 or cos_cache.dim() != 2
            or cos_cache.shape[1] != 32 or sin_cache.shape != cos_cache.shape or not cos_cache.is_contiguous()
            or not sin_cache.is_contiguous()):
        raise ValueError("cos_cache and sin_cache must be contiguous float32 [max_position, 32]")
    if q_out is None:
        q_out = torch.empty(T, H, QK_DIM, dtype=torch.bfloat16, device=dev)
    if q_out.dtype != torch.bfloat16 or q_out.shape != (T, H, QK_DIM) or q_out.stride(2) != 1:
        raise ValueError("q_out must be a bf16 [T, H, 576] tensor with a contiguous last dim")
    p = _lib.KimiQAbsorbParams(
        q_nope=q_nope.data_ptr(), q_nope_stride_t=q_nope.stride(0), q_nope_stride_h=q_nope.stride(1),
        q_pe=q_pe.data_ptr(), q_pe_stride_t=q_pe.stride(0), q_pe_stride_h=q_pe.stride(1), w_uk=w_uk.data_ptr(),
        kv_c=kv_c.data_ptr(), kv_c_stride=kv_c.stride(0), k_pe=k_pe.data_ptr(), k_pe_stride=k_pe.stride(0),
        positions=positions.data_ptr(), cos_cache=cos_cache.data_ptr(), sin_cache=sin_cache.data_ptr(),
        max_position=cos_cache.shape[0], slot_mapping=slot_mapping.data_ptr(), kv_buffer=kv_buffer.data_ptr(),
        kv_scales=kv_scales.data_ptr(), num_pages=num_pages, q_out=q_out.data_ptr(),
        q_out_stride_t=q_out.stride(0), q_out_stride_h=q_out.stride(1), num_tokens=T, num_heads=H,
        is_neox=int(bool(is_neox)), legacy_rule=int(bool(legacy_rule)))
    if status is not None:
        _require_status_word(status, dev)
        p.status = status.data_ptr()
    with torch.cuda.device(dev):
        st = _lib.load().kimi_mla_q_absorb_rope_append(ctypes.byref(p), _stream_handle(dev))
    _lib.check(st, "kimi_mla_q_absorb_rope_append")
    return q_out


def v_up_proj_and_o_proj(o: torch.Tensor, w_uv: torch.Tensor, w_o: torch.Tensor, out: torch.Tensor | None = None,
                         x: torch.Tensor | None = None, status: torch.Tensor | None = None) -> torch.Tensor:
    """The decode step after attention (the reference's
    ``_v_up_proj_and_o_proj(o, heads_first=True)``,
    patches/atom-optimizations.patch:131-143 and :297-302):

    * ``x[t, h*128:(h+1)*128] = bf16(o[h, t] @ w_uv[h])`` (fp32 accumulation);
    * ``out[t] = bf16(x[t] @ w_o.T)`` (fp32 accumulation).

    ``o`` is the decode's heads-first output bf16 [H, T, 512] (a slice of the
    padded heads, latent dim contiguous; any head and token strides that are
    multiples of 8 elements, so the transposed view of a token-major
    [T, H, 512] tensor works too), ``w_uv`` bf16 [H, 512, 128] and
    ``w_o`` bf16 [hidden, H * 128] contiguous (H <= 8, hidden % 64 == 0).
    ``out`` (bf16 [T, hidden], last dim contiguous, allocated when None) is
    returned: this rank's partial of the tensor-parallel all-reduce, so it
    may be a :class:`kimi_b200.tp.PeerPartials` ``local`` buffer.  ``x`` is a
    bf16 [T, H * 128] contiguous scratch (allocated when None) that holds the
    up-projection afterwards.  ``status``: optional int32 [1] device word that
    gets ``DEVICE_VUP_WAIT`` when a wait gave up (read it with
    :func:`device_status`).
    """
    dev = _require_cuda(o, w_uv, w_o)
    for name, t in (("o", o), ("w_uv", w_uv), ("w_o", w_o)):
        if t.dtype != torch.bfloat16:
            raise ValueError(f"{name} must be bfloat16")
    if o.dim() != 3 or o.shape[2] != KV_LORA_RANK or o.stride(2) != 1:
        raise ValueError("o must be heads-first [H, T, 512] with a contiguous last dim")
    H, T = o.shape[0], o.shape[1]
    if w_uv.shape != (H, KV_LORA_RANK, 128) or not w_uv.is_contiguous():
        raise ValueError("w_uv must be a contiguous [H, 512, 128] tensor")
    if w_o.dim() != 2 or w_o.shape[1] != H * 128 or not w_o.is_contiguous():
        raise ValueError("w_o must be a contiguous [hidden, H * 128] tensor")
    hidden = w_o.shape[0]
    if out is None:
        out = torch.empty(T, hidden, dtype=torch.bfloat16, device=dev)
    if out.dtype != torch.bfloat16 or out.dim() != 2 or out.shape != (T, hidden) or out.stride(1) != 1:
        raise ValueError("out must be a bf16 [T, hidden] tensor with a contiguous last dim")
    if x is None:
        x = torch.empty(T, H * 128, dtype=torch.bfloat16, device=dev)
    if x.dtype != torch.bfloat16 or x.shape != (T, H * 128) or not x.is_contiguous():
        raise ValueError("x must be a contiguous bf16 [T, H * 128] tensor")
    p = _lib.KimiVUpOProjParams(o=o.data_ptr(), o_stride_h=o.stride(0), o_stride_t=o.stride(1), w_uv=w_uv.data_ptr(),
                                w_o=w_o.data_ptr(), x=x.data_ptr(), out=out.data_ptr(), out_stride=out.stride(0),
                                num_tokens=T, num_heads=H, hidden=hidden)
    if status is not None:
        _require_status_word(status, dev)
        p.status = status.data_ptr()
    with torch.cuda.device(dev):
        st = _lib.load().kimi_mla_v_up_o_proj(ctypes.byref(p), _stream_handle(dev))
    _lib.check(st, "kimi_mla_v_up_o_proj")
    return out


def mxfp4_quantize(x: torch.Tensor, legacy_rule: bool = False):
    """bf16 [rows, cols] (cols % 32 == 0) -> (nibbles u8 [rows, cols/2], scales u8 [rows, cols/32])."""
    dev = _require_cuda(x)
    if x.dtype != torch.bfloat16 or x.dim() != 2 or x.stride(1) != 1:
        raise ValueError("x must be a bf16 [rows, cols] tensor with a contiguous last dim")
    rows, cols = x.shape
    if cols % 32:
        raise ValueError("cols must be a multiple of 32")
    nib = torch.empty(rows, cols // 2, dtype=torch.uint8, device=dev)
    sc = torch.empty(rows, cols // 32, dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        status = _lib.load().kimi_mxfp4_quantize(x.data_ptr(), rows, cols, x.stride(0), nib.data_ptr(),
                                                 sc.data_ptr(), int(bool(legacy_rule)), _stream_handle(dev))
    _lib.check(status, "kimi_mxfp4_quantize")
    return nib, sc
