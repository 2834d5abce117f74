"""aspida_b200 — B200 (sm_100a) attention library for the Aspida engine.

The compute lives in libaspida_attn.so (CUDA, C ABI in include/aspida_attn.h);
this package is the host-side binding that mirrors the reference's GPU
attention interface. Importing it loads the library and fails if it is absent.
"""
from . import _lib

_lib.load()

from .attention import (  # noqa: E402
    GPUError, RopeParams, KVCache, Workspace, fattn_new, fattn_free, fattn_snapshot,
    fattn_restore, prefix_reset, last_error, device_status, debug_fail_allocs, fattn_kv, prep,
    decode, decode_partial, decode_paged, decode_fused, decode_q8, quantize_q8, decode_fp8, quantize_fp8, prefill_q8_gated, prep_paged, prefill_paged, prefill, prefill_batch, merge, decode_workspace_size, ptr_table, step_host,
    ASPIDA_OK, ASPIDA_ERR_ARG, ASPIDA_ERR_HANDLE, ASPIDA_ERR_NOMEM, ASPIDA_ERR_UNSUPPORTED,
    ASPIDA_ERR_WORKSPACE, ASPIDA_ERR_DEVICE,
)

LIB_PATH = _lib.LIB_PATH
