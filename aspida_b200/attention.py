"""Host-side mirror of the reference's GPU attention binding.

Names follow the Ada binding ``LLM_Qwen_GPU`` (src/llm/llm_qwen_gpu.ads:116-170:
``Fattn_New``, ``Fattn_Free``, ``Fattn_Snapshot``, ``Fattn_Restore``,
``Prefix_Reset``) and the RoPE record ``LLM_RoPE.RoPE_Params``
(src/llm/llm_rope.ads:17-41). Every call goes through the C ABI of
libaspida_attn.so; device buffers are torch tensors used as plain memory
(torch supplies allocation and streams, not the attention math).

Errors: a non-zero status raises :class:`GPUError` carrying the code, the
Python counterpart of the binding's ``Check_GPU`` raising ``GPU_Error``
(src/llm/llm_qwen_gpu.adb:673-683). The lifecycle calls keep the shim's
conventions (``fattn_new`` returns -1 on failure, ``fattn_free`` ignores an
unknown handle).
"""
from __future__ import annotations

import array
import ctypes as C
import math
from dataclasses import dataclass, field
from typing import Optional, Sequence

import torch

from . import _lib

ASPIDA_OK = 0
ASPIDA_ERR_ARG = -1
ASPIDA_ERR_HANDLE = -2
ASPIDA_ERR_NOMEM = -3
ASPIDA_ERR_UNSUPPORTED = -4
ASPIDA_ERR_WORKSPACE = -5
ASPIDA_ERR_DEVICE = -6


class GPUError(RuntimeError):
    def __init__(self, code: int, what: str = ""):
        super().__init__(f"aspida attention error {code}{': ' + what if what else ''}")
        self.code = code


def _lib_():
    return _lib.load()


def _check(rc: int, what: str = "") -> None:
    if rc != 0:
        raise GPUError(rc, what)


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream(stream) -> Optional[int]:
    if stream is None:
        stream = torch.cuda.current_stream()
    return stream.cuda_stream if hasattr(stream, "cuda_stream") else stream


# ---------------------------------------------------------------------------
# RoPE parameters (LLM_RoPE.RoPE_Params)
# ---------------------------------------------------------------------------
@dataclass
class RopeParams:
    dim: int                      # rotated dims per head (rd)
    freq_base: float = 10000.0
    sections: Sequence[int] = field(default_factory=lambda: ())  # () = all pairs at pos
    use_ff: bool = False
    freq_factors: Optional[torch.Tensor] = None   # dev f32 [dim/2]
    interleaved: bool = False
    freq_scale: float = 1.0
    yarn_on: bool = False
    corr_low: float = 0.0
    corr_high: float = 0.0
    m_scale: float = 1.0

    @property
    def sec_total(self) -> int:
        """Pairs covered by the sections (Sections_Total, llm_fullattn.adb:249)."""
        if not self.sections:
            return self.dim // 2
        return sum(max(0, int(s)) for s in self.sections)


# ---------------------------------------------------------------------------
# KV-state lifecycle
# ---------------------------------------------------------------------------
def fattn_new(max_len: int, kvd: int, nq: int) -> int:
    return _lib_().aspida_gpu_fattn_new(max_len, kvd, nq)


def fattn_free(handle: int) -> None:
    _lib_().aspida_gpu_fattn_free(handle)


def fattn_snapshot(handle: int, rows: int, slot: int = -1) -> int:
    return _lib_().aspida_gpu_fattn_snapshot(handle, rows, slot)


def fattn_restore(handle: int, slot: int) -> int:
    return _lib_().aspida_gpu_fattn_restore(handle, slot)


def prefix_reset() -> None:
    _lib_().aspida_gpu_prefix_reset()


def last_error() -> int:
    return _lib_().aspida_gpu_last_error()


def device_status() -> int:
    return _lib_().aspida_attn_device_status()


def debug_fail_allocs(n: int) -> None:
    _lib_().aspida_attn_debug_fail_allocs(n)


class _DevArray:
    """__cuda_array_interface__ over library-owned device memory."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {
            "shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
            "version": 3, "strides": None,
        }


def fattn_kv(handle: int):
    """(K, V) fp16 tensor views [max_len, kvd] of a state's device caches."""
    k, v = C.c_void_p(), C.c_void_p()
    ml, kvd = C.c_int(), C.c_int()
    _check(_lib_().aspida_gpu_fattn_kv(handle, C.byref(k), C.byref(v), C.byref(ml), C.byref(kvd)),
           "fattn_kv")
    dev = torch.device("cuda", torch.cuda.current_device())
    K = torch.as_tensor(_DevArray(k.value, (ml.value, kvd.value), "<f2"), device=dev)
    V = torch.as_tensor(_DevArray(v.value, (ml.value, kvd.value), "<f2"), device=dev)
    return K, V


class KVCache:
    """A resident KV state (one generation x one layer) owned by a handle."""

    def __init__(self, max_len: int, nkv: int, hd: int, nq: int):
        self.max_len, self.nkv, self.hd, self.nq = max_len, nkv, hd, nq
        self.handle = fattn_new(max_len, nkv * hd, nq)
        if self.handle < 0:
            raise GPUError(last_error() or ASPIDA_ERR_NOMEM, "fattn_new")
        self.K, self.V = fattn_kv(self.handle)

    def free(self) -> None:
        if self.handle >= 0:
            self.K = self.V = None
            fattn_free(self.handle)
            self.handle = -1

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


# ---------------------------------------------------------------------------
# Compute entry points
# ---------------------------------------------------------------------------
def prep(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, K: torch.Tensor, V: torch.Tensor,
         pos_start: int, nq: int, nkv: int, hd: int, rope: RopeParams,
         q_norm: Optional[torch.Tensor] = None, k_norm: Optional[torch.Tensor] = None,
         eps: float = 1e-6, q_out_dtype=torch.float32, stream=None) -> torch.Tensor:
    """QK-norm (optional) + partial RoPE + fp16 K/V append for P tokens.

    q [P, nq*hd], k/v [P, nkv*hd] f32 on the device; K/V the fp16 cache
    [max_len, nkv*hd]. Returns the rotated queries in ``q_out_dtype``."""
    P = q.shape[0]
    q_out = torch.empty((P, nq * hd), dtype=q_out_dtype, device=q.device)
    ff = rope.freq_factors if rope.use_ff else None
    rc = _lib_().aspida_attn_prep(
        _ptr(q), _ptr(k), _ptr(v), P, nq, nkv, hd, _ptr(q_norm), _ptr(k_norm), eps,
        _ptr(q_out), int(q_out_dtype == torch.float16), _ptr(K), _ptr(V), K.shape[0], pos_start,
        rope.dim, rope.freq_base, rope.freq_scale, rope.m_scale, int(rope.yarn_on),
        rope.corr_low, rope.corr_high, _ptr(ff), int(rope.use_ff), int(rope.interleaved),
        rope.sec_total, _stream(stream))
    _check(rc, "prep")
    return q_out


def prep_paged(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, K_pool: torch.Tensor,
               V_pool: torch.Tensor, block_table: torch.Tensor, block_size: int, nq: int,
               nkv: int, hd: int, rope: RopeParams, *, pos_start: int = 0,
               pos: Optional[torch.Tensor] = None, q_norm: Optional[torch.Tensor] = None,
               k_norm: Optional[torch.Tensor] = None, eps: float = 1e-6,
               q_out_dtype=torch.float32, stream=None) -> torch.Tensor:
    """prep() appending into paged pools K_pool/V_pool [blocks*block_size,
    nkv*hd]. pos None: P tokens of one sequence at pos_start.. through the
    block_table int32 [max_blocks]; pos int32 [P]: a decode batch, row t at
    pos[t] through block_table row t ([P, max_blocks])."""
    P = q.shape[0]
    q_out = torch.empty((P, nq * hd), dtype=q_out_dtype, device=q.device)
    ff = rope.freq_factors if rope.use_ff else None
    rc = _lib_().aspida_attn_prep_paged(
        _ptr(q), _ptr(k), _ptr(v), P, nq, nkv, hd, _ptr(q_norm), _ptr(k_norm), eps,
        _ptr(q_out), int(q_out_dtype == torch.float16), _ptr(K_pool), _ptr(V_pool),
        _ptr(block_table), block_table.shape[-1], block_size, pos_start, _ptr(pos),
        rope.dim, rope.freq_base, rope.freq_scale, rope.m_scale, int(rope.yarn_on),
        rope.corr_low, rope.corr_high, _ptr(ff), int(rope.use_ff), int(rope.interleaved),
        rope.sec_total, _stream(stream))
    _check(rc, "prep_paged")
    return q_out


def ptr_table(tensors: Sequence[torch.Tensor], device) -> torch.Tensor:
    return torch.tensor([t.data_ptr() for t in tensors], dtype=torch.int64, device=device)


def decode_workspace_size(B: int, nq: int, nkv: int, hd: int, max_kv_len: int,
                          chunk: int = 0) -> int:
    return _lib_().aspida_attn_decode_workspace_size(B, nq, nkv, hd, max_kv_len, chunk)


class Workspace:
    """Grow-only device scratch for the decode entry points."""

    def __init__(self):
        self.buf: Optional[torch.Tensor] = None

    def get(self, nbytes: int, device) -> torch.Tensor:
        if self.buf is None or self.buf.numel() < nbytes or self.buf.device != device:
            self.buf = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=device)
        return self.buf


_default_ws = {}


def _ws(ws: Optional[Workspace], device) -> Workspace:
    if ws is not None:
        return ws
    key = (device.type, device.index)
    if key not in _default_ws:
        _default_ws[key] = Workspace()
    return _default_ws[key]


def decode(q: torch.Tensor, K_tab: torch.Tensor, V_tab: torch.Tensor, pos: torch.Tensor,
           nq: int, nkv: int, hd: int, *, gate: Optional[torch.Tensor] = None,
           max_len: Optional[torch.Tensor] = None, scale: Optional[float] = None,
           window: int = 0, softcap: float = 0.0, max_kv_len: int, chunk: int = 0,
           out: Optional[torch.Tensor] = None, workspace: Optional[Workspace] = None,
           stream=None) -> torch.Tensor:
    """Batched GQA decode. q [B, nq*hd] f32; K_tab/V_tab int64 [B] device
    pointer tables of fp16 caches [rows, nkv*hd]; pos int32 [B]."""
    B = q.shape[0]
    if scale is None:
        scale = 1.0 / math.sqrt(hd)
    if out is None:
        out = torch.empty((B, nq * hd), dtype=torch.float32, device=q.device)
    nbytes = decode_workspace_size(B, nq, nkv, hd, max_kv_len, chunk)
    wsb = _ws(workspace, q.device).get(nbytes, q.device)
    rc = _lib_().aspida_attn_decode(
        _ptr(q), _ptr(gate), _ptr(K_tab), _ptr(V_tab), _ptr(pos), _ptr(max_len), _ptr(out), B,
        nq, nkv, hd, scale, window, softcap, max_kv_len, chunk, _ptr(wsb), wsb.numel(),
        _stream(stream))
    _check(rc, "decode")
    return out


def quantize_q8(x: torch.Tensor, q: Optional[torch.Tensor] = None,
                scales: Optional[torch.Tensor] = None, stream=None):
    """Q8_0-quantise f32 x [..., n] (n a multiple of 32) into int8 q [..., n]
    and fp16 scales [..., n/32] (k_to_q8, gpu/fattn_kvhalf.cu:143-152).
    q / scales may be views into a cache (rows being appended)."""
    if x.dtype != torch.float32 or not x.is_contiguous() or x.shape[-1] % 32:
        raise ValueError("x must be contiguous f32 with a last dim divisible by 32")
    if q is None:
        q = torch.empty(x.shape, dtype=torch.int8, device=x.device)
    if scales is None:
        scales = torch.empty((*x.shape[:-1], x.shape[-1] // 32), dtype=torch.float16,
                             device=x.device)
    if q.numel() != x.numel() or scales.numel() * 32 != x.numel() or not q.is_contiguous() \
            or not scales.is_contiguous():
        raise ValueError("q / scales do not match x")
    rc = _lib_().aspida_attn_quantize_q8(_ptr(x), _ptr(q), _ptr(scales), x.numel() // 32,
                                         _stream(stream))
    _check(rc, "quantize_q8")
    return q, scales


def decode_q8(q: torch.Tensor, K_tab: torch.Tensor, V_tab: torch.Tensor, Ks_tab: torch.Tensor,
              Vs_tab: torch.Tensor, pos: torch.Tensor, nq: int, nkv: int, hd: int, *,
              gate: Optional[torch.Tensor] = None, max_len: Optional[torch.Tensor] = None,
              scale: Optional[float] = None, window: int = 0, softcap: float = 0.0,
              max_kv_len: int, chunk: int = 0, out: Optional[torch.Tensor] = None,
              workspace: Optional[Workspace] = None, stream=None) -> torch.Tensor:
    """Batched GQA decode over Q8_0 caches: K_tab/V_tab pointer tables of int8
    caches [rows, nkv*hd], Ks_tab/Vs_tab of fp16 scales [rows, nkv*hd/32]."""
    B = q.shape[0]
    if scale is None:
        scale = 1.0 / math.sqrt(hd)
    if out is None:
        out = torch.empty((B, nq * hd), dtype=torch.float32, device=q.device)
    nbytes = decode_workspace_size(B, nq, nkv, hd, max_kv_len, chunk)
    wsb = _ws(workspace, q.device).get(nbytes, q.device)
    rc = _lib_().aspida_attn_decode_q8(
        _ptr(q), _ptr(gate), _ptr(K_tab), _ptr(V_tab), _ptr(Ks_tab), _ptr(Vs_tab), _ptr(pos),
        _ptr(max_len), _ptr(out), B, nq, nkv, hd, scale, window, softcap, max_kv_len, chunk,
        _ptr(wsb), wsb.numel(), _stream(stream))
    _check(rc, "decode_q8")
    return out


def quantize_fp8(x: torch.Tensor, q: Optional[torch.Tensor] = None,
                 scales: Optional[torch.Tensor] = None, stream=None):
    """fp8 (e4m3) quantisation of f32 x [..., n] (n a multiple of 32) into
    uint8 codes q [..., n] and fp16 scales [..., n/32] (per 32-value block,
    s = fp16(max|v| / 448), code = e4m3(v / s), saturating)."""
    if x.dtype != torch.float32 or not x.is_contiguous() or x.shape[-1] % 32:
        raise ValueError("x must be contiguous f32 with a last dim divisible by 32")
    if q is None:
        q = torch.empty(x.shape, dtype=torch.uint8, device=x.device)
    if scales is None:
        scales = torch.empty((*x.shape[:-1], x.shape[-1] // 32), dtype=torch.float16,
                             device=x.device)
    if q.numel() != x.numel() or scales.numel() * 32 != x.numel() or not q.is_contiguous() \
            or not scales.is_contiguous():
        raise ValueError("q / scales do not match x")
    rc = _lib_().aspida_attn_quantize_fp8(_ptr(x), _ptr(q), _ptr(scales), x.numel() // 32,
                                          _stream(stream))
    _check(rc, "quantize_fp8")
    return q, scales


def decode_fp8(q: torch.Tensor, K_tab: torch.Tensor, V_tab: torch.Tensor, Ks_tab: torch.Tensor,
               Vs_tab: torch.Tensor, pos: torch.Tensor, nq: int, nkv: int, hd: int, *,
               gate: Optional[torch.Tensor] = None, max_len: Optional[torch.Tensor] = None,
               scale: Optional[float] = None, window: int = 0, softcap: float = 0.0,
               max_kv_len: int, chunk: int = 0, out: Optional[torch.Tensor] = None,
               workspace: Optional[Workspace] = None, stream=None) -> torch.Tensor:
    """Batched GQA decode over fp8 (e4m3) caches: K_tab/V_tab pointer tables of
    uint8 code caches [rows, nkv*hd], Ks_tab/Vs_tab of fp16 block scales
    [rows, nkv*hd/32] (quantize_fp8's layout)."""
    B = q.shape[0]
    if scale is None:
        scale = 1.0 / math.sqrt(hd)
    if out is None:
        out = torch.empty((B, nq * hd), dtype=torch.float32, device=q.device)
    nbytes = decode_workspace_size(B, nq, nkv, hd, max_kv_len, chunk)
    wsb = _ws(workspace, q.device).get(nbytes, q.device)
    rc = _lib_().aspida_attn_decode_fp8(
        _ptr(q), _ptr(gate), _ptr(K_tab), _ptr(V_tab), _ptr(Ks_tab), _ptr(Vs_tab), _ptr(pos),
        _ptr(max_len), _ptr(out), B, nq, nkv, hd, scale, window, softcap, max_kv_len, chunk,
        _ptr(wsb), wsb.numel(), _stream(stream))
    _check(rc, "decode_fp8")
    return out


def prefill_q8_gated(q: torch.Tensor, K8: torch.Tensor, V8: torch.Tensor, Ks: torch.Tensor,
                     Vs: torch.Tensor, nq: int, nkv: int, hd: int, pos_start: int = 0, *,
                     gate: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
                     stream=None) -> torch.Tensor:
    """Gated causal prefill over Q8_0 caches (k_gqa_kv<..., 2> semantics):
    q f32 [P, nq*hd]; K8/V8 int8 [rows, nkv*hd]; Ks/Vs fp16 [rows, nkv*hd/32]."""
    P = q.shape[0]
    if out is None:
        out = torch.empty((P, nq * hd), dtype=torch.float32, device=q.device)
    rc = _lib_().aspida_attn_prefill_q8_gated(
        _ptr(q), _ptr(gate), _ptr(K8), _ptr(V8), _ptr(Ks), _ptr(Vs), _ptr(out), nq, nkv, hd, P,
        pos_start, _stream(stream))
    _check(rc, "prefill_q8_gated")
    return out


def decode_fused(q_raw: torch.Tensor, k_raw: torch.Tensor, v_raw: torch.Tensor,
                 K_tab: torch.Tensor, V_tab: torch.Tensor, pos: torch.Tensor, nq: int, nkv: int,
                 hd: int, rope: RopeParams, *, q_norm: Optional[torch.Tensor] = None,
                 k_norm: Optional[torch.Tensor] = None, eps: float = 1e-6,
                 gate: Optional[torch.Tensor] = None, max_len: Optional[torch.Tensor] = None,
                 scale: Optional[float] = None, window: int = 0, softcap: float = 0.0,
                 max_kv_len: int, chunk: int = 0, out: Optional[torch.Tensor] = None,
                 workspace: Optional[Workspace] = None, stream=None) -> torch.Tensor:
    """prep + decode in one launch: raw queries and the new raw K/V rows
    [B, nkv*hd] (appended at pos into the fp16 caches of the tables)."""
    B = q_raw.shape[0]
    if scale is None:
        scale = 1.0 / math.sqrt(hd)
    if out is None:
        out = torch.empty((B, nq * hd), dtype=torch.float32, device=q_raw.device)
    nbytes = decode_workspace_size(B, nq, nkv, hd, max_kv_len, chunk)
    wsb = _ws(workspace, q_raw.device).get(nbytes, q_raw.device)
    ff = rope.freq_factors if rope.use_ff else None
    rc = _lib_().aspida_attn_decode_fused(
        _ptr(q_raw), _ptr(k_raw), _ptr(v_raw), _ptr(gate), _ptr(K_tab), _ptr(V_tab), _ptr(pos),
        _ptr(max_len), _ptr(out), B, nq, nkv, hd, _ptr(q_norm), _ptr(k_norm), eps, rope.dim,
        rope.freq_base, rope.freq_scale, rope.m_scale, int(rope.yarn_on), rope.corr_low,
        rope.corr_high, _ptr(ff), int(rope.use_ff), int(rope.interleaved), rope.sec_total,
        scale, window, softcap, max_kv_len, chunk, _ptr(wsb), wsb.numel(), _stream(stream))
    _check(rc, "decode_fused")
    return out


def decode_partial(q: torch.Tensor, K_tab: torch.Tensor, V_tab: torch.Tensor,
                   kv_lo: torch.Tensor, kv_hi: torch.Tensor, nq: int, nkv: int, hd: int, *,
                   scale: Optional[float] = None, softcap: float = 0.0, max_kv_len: int,
                   chunk: int = 0, workspace: Optional[Workspace] = None, stream=None):
    """Split-KV partial (m, l, o) over keys [kv_lo[b], kv_hi[b]) of each cache."""
    B = q.shape[0]
    if scale is None:
        scale = 1.0 / math.sqrt(hd)
    m = torch.empty((B, nq), dtype=torch.float32, device=q.device)
    l = torch.empty((B, nq), dtype=torch.float32, device=q.device)
    o = torch.empty((B, nq, hd), dtype=torch.float32, device=q.device)
    nbytes = decode_workspace_size(B, nq, nkv, hd, max_kv_len, chunk)
    wsb = _ws(workspace, q.device).get(nbytes, q.device)
    rc = _lib_().aspida_attn_decode_partial(
        _ptr(q), _ptr(K_tab), _ptr(V_tab), _ptr(kv_lo), _ptr(kv_hi), _ptr(m), _ptr(l), _ptr(o),
        B, nq, nkv, hd, scale, softcap, max_kv_len, chunk, _ptr(wsb), wsb.numel(),
        _stream(stream))
    _check(rc, "decode_partial")
    return m, l, o


def merge(m: torch.Tensor, l: torch.Tensor, o: torch.Tensor,
          gate: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
          stream=None) -> torch.Tensor:
    """Merge S partials: m, l [S, rows]; o [S, rows, hd] -> out [rows, hd]."""
    S, rows, hd = o.shape
    if out is None:
        out = torch.empty((rows, hd), dtype=torch.float32, device=o.device)
    rc = _lib_().aspida_attn_merge(_ptr(m), _ptr(l), _ptr(o), _ptr(gate), _ptr(out), S, rows, hd,
                                   _stream(stream))
    _check(rc, "merge")
    return out


def _int32_host(xs):
    """A host int32 array for an ABI argument: (object to keep alive, address).
    Accepts a CPU int32 tensor or an array.array('i') as is; otherwise builds
    an array.array (a few microseconds for a batch, where a ctypes array of
    Python ints costs several times that on every decode step)."""
    if isinstance(xs, torch.Tensor):
        if xs.dtype != torch.int32 or xs.is_cuda or not xs.is_contiguous():
            xs = xs.to(device="cpu", dtype=torch.int32).contiguous()
        return xs, xs.data_ptr()
    if not (isinstance(xs, array.array) and xs.typecode == "i"):
        xs = array.array("i", xs)
    return xs, xs.buffer_info()[0]


def step_host(handles: Sequence[int], q, k, v, pos, out, nq: int, nkv: int, hd: int, *,
              scale: Optional[float] = None, window: int = 0, softcap: float = 0.0,
              rope_dim: int = 0, rope_base: float = 10000.0, interleaved: bool = False,
              stream=None) -> None:
    """Host-buffer decode step (q/k/v/pos/out are host tensors, ideally pinned)."""
    B = len(handles)
    if scale is None:
        scale = 1.0 / math.sqrt(hd)
    h, hp = _int32_host(handles)
    pa, pp = _int32_host(pos)
    rc = _lib_().aspida_attn_step_host(
        hp, B, q.data_ptr(), k.data_ptr(), v.data_ptr(), pp, out.data_ptr(),
        nq, nkv, hd, scale, window, softcap, rope_dim, rope_base, int(interleaved),
        _stream(stream))
    del h, pa
    _check(rc, "step_host")


def prefill(q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, nq: int, nkv: int, hd: int,
            pos_start: int = 0, *, gate: Optional[torch.Tensor] = None,
            scale: Optional[float] = None, window: int = 0, softcap: float = 0.0,
            out_dtype=torch.float16, out: Optional[torch.Tensor] = None,
            stream=None) -> torch.Tensor:
    """Causal prefill: q fp16 [P, nq*hd] at positions pos_start.., K/V fp16
    caches [>= pos_start+P, nkv*hd]. Returns [P, nq*hd] in ``out_dtype``."""
    P = q.shape[0]
    if scale is None:
        scale = 1.0 / math.sqrt(hd)
    if out is None:
        out = torch.empty((P, nq * hd), dtype=out_dtype, device=q.device)
    rc = _lib_().aspida_attn_prefill(
        _ptr(q), _ptr(K), _ptr(V), _ptr(gate), _ptr(out), int(out.dtype == torch.float32), nq,
        nkv, hd, P, pos_start, scale, window, softcap, _stream(stream))
    _check(rc, "prefill")
    return out


def prefill_paged(q: torch.Tensor, K_pool: torch.Tensor, V_pool: torch.Tensor,
                  block_table: torch.Tensor, block_size: int, nq: int, nkv: int, hd: int,
                  pos_start: int = 0, *, gate: Optional[torch.Tensor] = None,
                  scale: Optional[float] = None, window: int = 0, softcap: float = 0.0,
                  out_dtype=torch.float16, out: Optional[torch.Tensor] = None,
                  stream=None) -> torch.Tensor:
    """prefill() over paged pools [blocks*block_size, nkv*hd] through
    block_table int32 [max_blocks]; block_size a multiple of 128 (hd <= 128)
    or 64 (hd 256)."""
    P = q.shape[0]
    if scale is None:
        scale = 1.0 / math.sqrt(hd)
    if out is None:
        out = torch.empty((P, nq * hd), dtype=out_dtype, device=q.device)
    nblocks = K_pool.shape[0] // block_size
    rc = _lib_().aspida_attn_prefill_paged(
        _ptr(q), _ptr(K_pool), _ptr(V_pool), _ptr(block_table), nblocks, block_size, _ptr(gate),
        _ptr(out), int(out.dtype == torch.float32), nq, nkv, hd, P, pos_start, scale, window,
        softcap, _stream(stream))
    _check(rc, "prefill_paged")
    return out


def prefill_batch(qs, Ks, Vs, nq: int, nkv: int, hd: int, pos_starts=None, *,
                  gates=None, outs=None, scale: Optional[float] = None, window: int = 0,
                  softcap: float = 0.0, out_dtype=torch.float16, stream=None):
    """Prefill several sequences in one launch (each its own q/K/V/out)."""
    n = len(qs)
    if scale is None:
        scale = 1.0 / math.sqrt(hd)
    if pos_starts is None:
        pos_starts = [0] * n
    if outs is None:
        outs = [torch.empty((q.shape[0], nq * hd), dtype=out_dtype, device=q.device) for q in qs]
    arr = lambda ts: (C.c_void_p * n)(*[None if t is None else t.data_ptr() for t in ts])
    qa, ka, va, oa = arr(qs), arr(Ks), arr(Vs), arr(outs)
    ga = arr(gates) if gates is not None else None
    Pa = (C.c_int * n)(*[q.shape[0] for q in qs])
    pa = (C.c_int * n)(*pos_starts)
    rc = _lib_().aspida_attn_prefill_batch(
        n, C.addressof(qa), C.addressof(ka), C.addressof(va),
        None if ga is None else C.addressof(ga), C.addressof(oa), C.addressof(Pa),
        C.addressof(pa), int(outs[0].dtype == torch.float32), nq, nkv, hd, scale, window,
        softcap, _stream(stream))
    _check(rc, "prefill_batch")
    return outs


def decode_paged(q: torch.Tensor, K_pool: torch.Tensor, V_pool: torch.Tensor,
                 block_table: torch.Tensor, block_size: int, pos: torch.Tensor, nq: int,
                 nkv: int, hd: int, *, gate: Optional[torch.Tensor] = None,
                 scale: Optional[float] = None, window: int = 0, softcap: float = 0.0,
                 max_kv_len: int, chunk: int = 0, out: Optional[torch.Tensor] = None,
                 workspace: Optional[Workspace] = None, stream=None) -> torch.Tensor:
    """Decode over a paged KV pool: K_pool/V_pool fp16 [blocks*block_size,
    nkv*hd]; block_table int32 [B, max_blocks] of block ids."""
    B = q.shape[0]
    if scale is None:
        scale = 1.0 / math.sqrt(hd)
    if out is None:
        out = torch.empty((B, nq * hd), dtype=torch.float32, device=q.device)
    nbytes = decode_workspace_size(B, nq, nkv, hd, max_kv_len, chunk)
    wsb = _ws(workspace, q.device).get(nbytes, q.device)
    rc = _lib_().aspida_attn_decode_paged(
        _ptr(q), _ptr(gate), _ptr(K_pool), _ptr(V_pool), _ptr(block_table), block_table.shape[1],
        block_size, _ptr(pos), _ptr(out), B, nq, nkv, hd, scale, window, softcap, max_kv_len,
        chunk, _ptr(wsb), wsb.numel(), _stream(stream))
    _check(rc, "decode_paged")
    return out
