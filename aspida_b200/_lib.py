"""ctypes binding of libaspida_attn.so (the C ABI declared in include/aspida_attn.h).

The shared library is built in-tree by ``aspida_b200/csrc/Makefile``; there is
no CPU fallback, so importing this module fails loudly when it is missing.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
# ASPIDA_ATTN_LIB overrides the in-tree library (e.g. to load an alternative build)
LIB_PATH = os.environ.get("ASPIDA_ATTN_LIB") or os.path.join(_HERE, "libaspida_attn.so")

i32, f32, sz, vp = C.c_int, C.c_float, C.c_size_t, C.c_void_p
pp = C.POINTER(C.c_void_p)
ip = C.POINTER(C.c_int)

# name -> (restype, argtypes); mirrors include/aspida_attn.h one to one.
SIGNATURES = {
    "aspida_gpu_fattn_new": (i32, [i32, i32, i32]),
    "aspida_gpu_fattn_free": (None, [i32]),
    "aspida_gpu_fattn_snapshot": (i32, [i32, i32, i32]),
    "aspida_gpu_fattn_restore": (i32, [i32, i32]),
    "aspida_gpu_prefix_reset": (None, []),
    "aspida_gpu_last_error": (i32, []),
    "aspida_gpu_fattn_kv": (i32, [i32, pp, pp, ip, ip]),
    "aspida_attn_device_status": (i32, []),
    "aspida_attn_device_status_where": (i32, []),
    "aspida_attn_debug_fail_allocs": (None, [i32]),
    "aspida_attn_prep": (i32, [vp, vp, vp, i32, i32, i32, i32, vp, vp, f32, vp, i32, vp, vp,
                               i32, i32, i32, f32, f32, f32, i32, f32, f32, vp, i32, i32, i32,
                               vp]),
    "aspida_attn_prep_paged": (i32, [vp, vp, vp, i32, i32, i32, i32, vp, vp, f32, vp, i32, vp,
                                     vp, vp, i32, i32, i32, vp, i32, f32, f32, f32, i32, f32, f32,
                                     vp, i32, i32, i32, vp]),
    "aspida_attn_prefill_paged": (i32, [vp, vp, vp, vp, i32, i32, vp, vp, i32, i32, i32, i32, i32,
                                        i32, f32, i32, f32, vp]),
    "aspida_attn_decode_workspace_size": (sz, [i32, i32, i32, i32, i32, i32]),
    "aspida_attn_decode": (i32, [vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, f32, i32, f32,
                                 i32, i32, vp, sz, vp]),
    "aspida_attn_decode_paged": (i32, [vp, vp, vp, vp, vp, i32, i32, vp, vp, i32, i32, i32, i32,
                                       f32, i32, f32, i32, i32, vp, sz, vp]),
    "aspida_attn_decode_partial": (i32, [vp, vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, i32,
                                         f32, f32, i32, i32, vp, sz, vp]),
    "aspida_attn_decode_fused": (i32, [vp, vp, vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, vp,
                                       vp, f32, i32, f32, f32, f32, i32, f32, f32, vp, i32, i32,
                                       i32, f32, i32, f32, i32, i32, vp, sz, vp]),
    "aspida_attn_decode_q8": (i32, [vp, vp, vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, f32,
                                    i32, f32, i32, i32, vp, sz, vp]),
    "aspida_attn_quantize_q8": (i32, [vp, vp, vp, C.c_longlong, vp]),
    "aspida_attn_decode_fp8": (i32, [vp, vp, vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, f32,
                                     i32, f32, i32, i32, vp, sz, vp]),
    "aspida_attn_quantize_fp8": (i32, [vp, vp, vp, C.c_longlong, vp]),
    "aspida_attn_prefill_q8_gated": (i32, [vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32,
                                           vp]),
    "aspida_attn_peer_buffer_size": (sz, [i32, i32, i32]),
    "aspida_attn_peer_alloc": (i32, [sz, vp, vp]),
    "aspida_attn_peer_open": (i32, [vp, vp]),
    "aspida_attn_peer_close": (i32, [vp]),
    "aspida_attn_peer_free": (i32, [vp]),
    "aspida_attn_exchange_merge": (i32, [vp, vp, i32, i32, C.c_ulonglong, vp, vp, i32, i32, vp]),
    "aspida_attn_exchange_merge_ex": (i32, [vp, vp, i32, i32, C.c_ulonglong, vp, vp, i32, i32,
                                            vp, C.c_longlong, vp]),
    "aspida_attn_merge": (i32, [vp, vp, vp, vp, vp, i32, i32, i32, vp]),
    "aspida_attn_merge_strided": (i32, [vp, vp, vp, vp, vp, i32, i32, i32, C.c_long, vp]),
    "aspida_attn_decode_noalloc": (i32, [vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, f32, i32,
                                         f32, i32, i32, vp]),
    "aspida_attn_prefill": (i32, [vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, f32, i32, f32,
                                  vp]),
    "aspida_attn_prefill_batch": (i32, [i32, vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, f32,
                                        i32, f32, vp]),
    "aspida_attn_prefill_gated": (i32, [vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, vp]),
    "aspida_attn_step_host": (i32, [vp, i32, vp, vp, vp, vp, vp, i32, i32, i32, f32, i32, f32,
                                    i32, f32, i32, vp]),
}

_lib = None


def load() -> C.CDLL:
    """Load the library once; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `make -C aspida_b200/csrc` "
            "(or __graft_entry__.build()); there is no CPU fallback")
    lib = C.CDLL(LIB_PATH, mode=C.RTLD_GLOBAL)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def exported_symbols() -> list[str]:
    return sorted(SIGNATURES)
