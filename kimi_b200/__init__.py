"""kimi_b200 -- B200-native (sm_100a) MXFP4 absorbed-MLA decode.

The hot path of the ianye23301/kimi serving work rebuilt as hand-written
CUDA behind a C ABI (include/kimi_mla.h, ``libkimi_mla.so``), with a thin
PyTorch host layer that keeps the reference's operator interface.
"""
from .mla import (  # noqa: F401
    KV_LORA_RANK,
    PAGE_SIZE,
    QK_DIM,
    ROPE_DIM,
    SCALE_BYTES,
    TOKEN_BYTES,
    alloc_mxfp4_cache,
    alloc_workspace,
    check_device_status,
    device_status,
    mla_decode_fwd,
    mla_decode_merge,
    mla_decode_partial,
    mla_reduce,
    mxfp4_kv_append,
    mxfp4_quantize,
    num_kv_splits_for,
    q_absorb_rope_append,
    v_up_proj_and_o_proj,
    workspace_bytes,
)

__all__ = [
    "KV_LORA_RANK", "PAGE_SIZE", "QK_DIM", "ROPE_DIM", "SCALE_BYTES", "TOKEN_BYTES",
    "alloc_mxfp4_cache", "alloc_workspace", "check_device_status", "device_status", "mla_decode_fwd", "mla_decode_merge", "mla_decode_partial",
    "mla_reduce", "mxfp4_kv_append",
    "mxfp4_quantize", "num_kv_splits_for", "q_absorb_rope_append", "v_up_proj_and_o_proj",
    "workspace_bytes",
]
