"""CPU oracle — TEST INFRASTRUCTURE ONLY.

numpy front end of liboracle_attn.so (attn_oracle.cpp), the C++ restatement
of the reference's Ada attention loops. Only tests/, __graft_entry__.smoke()
and bench.py's CPU-baseline legs use it, as the checker; the product path in
aspida_b200/ never imports it.

Parity is pinned against fixtures produced by the reference's own fp32
kernels (oracle/ref_harness.cu, tests/golden/make_golden.py) and against the
reference's known-answer tests restated in tests/test_oracle.py.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle_attn.so")

_lib = None


def build() -> None:
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def load():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        lib = C.CDLL(LIB_PATH)
        vp, i32, f32 = C.c_void_p, C.c_int, C.c_float
        lib.oracle_rmsnorm.argtypes = [vp, vp, vp, i32, f32]
        lib.oracle_rope_apply_sections.argtypes = [vp, vp, i32, f32, vp, vp, i32, vp, i32, f32,
                                                   i32, f32, f32, f32]
        lib.oracle_norm_rope.argtypes = [vp, vp, f32, vp, i32, i32, i32, f32, i32, i32, vp, i32,
                                         f32, i32, f32, f32, f32]
        lib.oracle_decode_batch.argtypes = [vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, f32, i32,
                                            f32, i32]
        lib.oracle_prefill.argtypes = [vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, f32, i32, f32,
                                       vp, i32, i32]
        lib.oracle_merge.argtypes = [vp, vp, vp, vp, vp, i32, i32, i32]
        for fn in ("oracle_rmsnorm", "oracle_rope_apply_sections", "oracle_norm_rope",
                   "oracle_decode_batch", "oracle_prefill", "oracle_merge"):
            getattr(lib, fn).restype = None
        _lib = lib
    return _lib


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _p(a):
    return None if a is None else a.ctypes.data


def rmsnorm(x, w, eps=1e-6):
    x, w = _f32(x), _f32(w)
    out = np.empty_like(x)
    load().oracle_rmsnorm(_p(x), _p(w), _p(out), x.size, eps)
    return out


def rope_apply_sections(x, base, sections, sec_pos, *, ff=None, interleaved=False,
                        freq_scale=1.0, yarn_on=False, corr_lo=0.0, corr_hi=0.0, m_scale=1.0):
    """LLM_RoPE.Apply_Sections on one head vector of length dim."""
    x = _f32(x)
    out = np.empty_like(x)
    sec = np.ascontiguousarray(sections, dtype=np.int32)
    sp = np.ascontiguousarray(sec_pos, dtype=np.int32)
    ffa = _f32(ff) if ff is not None else None
    load().oracle_rope_apply_sections(_p(x), _p(out), x.size, base, _p(sec), _p(sp),
                                      int(ff is not None), _p(ffa), int(interleaved), freq_scale,
                                      int(yarn_on), corr_lo, corr_hi, m_scale)
    return out


def rope_apply(x, base, pos, **kw):
    """LLM_RoPE.Apply: all pairs at `pos` (sections covering dim/2)."""
    d = np.asarray(x).size
    return rope_apply_sections(x, base, [d // 2, 0, 0, 0], [pos] * 4, **kw)


def norm_rope(x, norm_w, hd, rd, pos, base, *, eps=1e-6, sec_total=None, ff=None,
              interleaved=False, freq_scale=1.0, yarn_on=False, corr_lo=0.0, corr_hi=0.0,
              m_scale=1.0):
    """Norm_Rope of LLM_FullAttn for one head (norm_w None = no RMSNorm)."""
    x = _f32(x)
    out = np.empty(hd, np.float32)
    nw = _f32(norm_w) if norm_w is not None else None
    ffa = _f32(ff) if ff is not None else None
    load().oracle_norm_rope(_p(x), _p(nw), eps, _p(out), hd, rd, pos, base,
                            rd // 2 if sec_total is None else sec_total, int(ff is not None),
                            _p(ffa), int(interleaved), freq_scale, int(yarn_on), corr_lo,
                            corr_hi, m_scale)
    return out


def rope_rows(x, nheads, hd, positions, base, *, rd=None, interleaved=False, sec_total=None):
    """Rotate rows x[t] ([nheads*hd] each) at positions[t] (no norm)."""
    x = _f32(x)
    rd = hd if rd is None else rd
    out = np.empty_like(x)
    for t, p in enumerate(positions):
        for h in range(nheads):
            out[t, h * hd:(h + 1) * hd] = norm_rope(x[t, h * hd:(h + 1) * hd], None, hd, rd, int(p),
                                                    base, interleaved=interleaved,
                                                    sec_total=sec_total)
    return out


def decode_batch(q, K_list, V_list, pos, nq, nkv, hd, *, gate=None, scale=None, window=0,
                 softcap=0.0, threads=0):
    """q [B, nq*hd]; K_list/V_list: B arrays [rows, nkv*hd] (f32); pos [B]."""
    q = _f32(q)
    B = q.shape[0]
    Ks = [_f32(k) for k in K_list]
    Vs = [_f32(v) for v in V_list]
    kp = (C.c_void_p * B)(*[k.ctypes.data for k in Ks])
    vp_ = (C.c_void_p * B)(*[v.ctypes.data for v in Vs])
    posa = np.ascontiguousarray(pos, dtype=np.int32)
    g = _f32(gate) if gate is not None else None
    out = np.empty((B, nq * hd), np.float32)
    if scale is None:
        scale = 1.0 / np.sqrt(np.float32(hd))
    threads = threads or os.cpu_count() or 1
    load().oracle_decode_batch(_p(q), _p(g), C.cast(kp, C.c_void_p), C.cast(vp_, C.c_void_p),
                               _p(posa), _p(out), B, nq, nkv, hd, float(scale), window, softcap,
                               threads)
    return out


def prefill(q, K, V, pos_start, nq, nkv, hd, *, gate=None, scale=None, window=0, softcap=0.0,
            rows=None, threads=0):
    """q [P, nq*hd]; K/V [pos_start+P, nkv*hd]. rows: optional token subset.
    Returns [P, nq*hd] (rows not in the subset are left as NaN)."""
    q, K, V = _f32(q), _f32(K), _f32(V)
    P = q.shape[0]
    out = np.full((P, nq * hd), np.nan, np.float32)
    g = _f32(gate) if gate is not None else None
    if scale is None:
        scale = 1.0 / np.sqrt(np.float32(hd))
    ra = np.ascontiguousarray(rows, dtype=np.int32) if rows is not None else None
    if ra is not None and ra.size and (ra.min() < 0 or ra.max() >= P):
        raise ValueError("rows must lie in [0, P)")
    threads = threads or os.cpu_count() or 1
    load().oracle_prefill(_p(q), _p(g), _p(K), _p(V), _p(out), P, pos_start, nq, nkv, hd,
                          float(scale), window, softcap, _p(ra), 0 if ra is None else ra.size,
                          threads)
    return out


def merge(m, l, o, gate=None):
    """m, l [S, rows]; o [S, rows, hd] -> [rows, hd]."""
    m, l, o = _f32(m), _f32(l), _f32(o)
    S, rows, hd = o.shape
    g = _f32(gate) if gate is not None else None
    out = np.empty((rows, hd), np.float32)
    load().oracle_merge(_p(m), _p(l), _p(o), _p(g), _p(out), S, rows, hd)
    return out


def quantize_q8(x):
    """Q8_0 quantisation of k_to_q8 (gpu/fattn_kvhalf.cu:143-152), in numpy:
    per 32-value block d = max|v| / 127 (f32 division), id = 1/d (0 for an
    all-zero block), q = clamp(rint(v * id), -127, 127) (lrintf: nearest,
    ties to even), scale = fp16(d). Returns (int8 q, fp16 scales)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    blocks = x.reshape(-1, 32)
    amax = np.max(np.abs(blocks), axis=1)
    d = (amax / np.float32(127)).astype(np.float32)
    with np.errstate(divide="ignore"):
        idv = np.where(d > 0, np.float32(1) / d, np.float32(0)).astype(np.float32)
    qv = np.clip(np.rint(blocks * idv[:, None]), -127, 127).astype(np.int8)
    return qv.reshape(x.shape), d.astype(np.float16).reshape(*x.shape[:-1], x.shape[-1] // 32)


def dequantize_q8(q, scales):
    """Values the reference's KVMODE 2 tile load computes
    (gpu/fattn_kvhalf.cu:88-92): float(int8) * float(fp16 scale), in f32."""
    q = np.asarray(q)
    s = np.asarray(scales).astype(np.float32)
    return (q.astype(np.float32).reshape(-1, 32) * s.reshape(-1, 1)).reshape(q.shape)


def _e4m3_table():
    """Values of the 127 non-negative finite e4m3 codes 0x00..0x7e (OCP FP8
    E4M3: 4 exponent bits, bias 7, 3 mantissa bits, subnormals, no infinity;
    0x7f is NaN)."""
    vals = np.empty(127, np.float64)
    for c in range(127):
        e, m = c >> 3, c & 7
        vals[c] = (m / 8.0) * 2.0 ** -6 if e == 0 else (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return vals


_E4M3 = _e4m3_table()


def e4m3_encode(x):
    """f32 -> e4m3 codes (uint8): round to nearest, ties to the even code,
    saturating at +-448, the sign kept (a negative value that rounds to zero
    gives -0, 0x80) - cvt.rn.satfinite.e4m3x2.f32 semantics."""
    x = np.asarray(x, np.float32).astype(np.float64)
    a = np.minimum(np.abs(x), 448.0)
    hi = np.clip(np.searchsorted(_E4M3, a, side="left"), 0, 126)
    lo = np.clip(hi - 1, 0, 126)
    dlo, dhi = a - _E4M3[lo], _E4M3[hi] - a
    pick_hi = (dhi < dlo) | ((dhi == dlo) & (hi % 2 == 0))
    code = np.where(pick_hi, hi, lo).astype(np.uint8)
    return np.where(np.signbit(x), code | 0x80, code).astype(np.uint8)


def e4m3_decode(codes):
    c = np.asarray(codes, np.uint8)
    v = _E4M3[np.minimum(c & 0x7F, 126)].astype(np.float32)
    return np.where(c & 0x80, -v, v).astype(np.float32)


def quantize_fp8(x):
    """fp8 (e4m3) block quantisation of aspida_attn_quantize_fp8, in numpy: per
    32-value block s = fp16(max|v| / 448) (f32 division), code = e4m3(v / s)
    (f32 division, nearest-even, saturating), zeros when s = 0. Returns
    (uint8 codes, fp16 scales)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    blocks = x.reshape(-1, 32)
    amax = np.max(np.abs(blocks), axis=1)
    s16 = (amax / np.float32(448)).astype(np.float32).astype(np.float16)
    s = s16.astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        y = np.where(s[:, None] > 0, blocks / s[:, None], np.float32(0)).astype(np.float32)
    codes = e4m3_encode(y)
    return codes.reshape(x.shape), s16.reshape(*x.shape[:-1], x.shape[-1] // 32)


def dequantize_fp8(codes, scales):
    """Values the fp8 decode reads: float(e4m3 code) * float(fp16 scale), f32."""
    v = e4m3_decode(codes).reshape(-1, 32)
    s = np.asarray(scales).astype(np.float32).reshape(-1, 1)
    return (v * s).reshape(np.asarray(codes).shape)
