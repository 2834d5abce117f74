// common.cuh — shared helpers for the sm_100a attention kernels:
// status codes, the device-side status word, and thin inline-PTX wrappers
// (mbarrier, bulk async copy, ldmatrix, mma.sync, movmatrix).
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/aspida_attn.h"

namespace aspida {

// ---------------------------------------------------------------------------
// Host-side status bookkeeping (kv_state.cu owns the storage).
// ---------------------------------------------------------------------------
int record_status(int status);                 // remembers non-zero, returns it
inline int cuda_status(cudaError_t e) { return e == cudaSuccess ? 0 : record_status((int)e); }
int num_sms();                                 // SM count of the current device

// Device-side status word: a kernel whose bounded wait ran out writes a
// non-zero code here and returns early; aspida_attn_device_status() reads it.
struct DeviceStatus { int code; int where; };
DeviceStatus* device_status_ptr();             // per-device compiled-in word (no allocation)

constexpr int kDevTimeoutMbar = 1;             // mbarrier wait ran out

// ---------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n"
      "selp.u32 %0, 1, 0, p;\n"
      "}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: polls try_wait (which itself suspends briefly in hardware)
// without sleeping for the first 2^16 polls, so hand-offs on a busy pipeline
// cost no added latency; then backs off with __nanosleep. Returns false when
// the limit (on the order of seconds) is exhausted.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  for (uint32_t it = 0; it < (1u << 16); ++it)
    if (mbar_try_wait(bar, parity)) return true;
  uint32_t ns = 64;
  for (uint32_t it = 0; it < (1u << 22); ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    __nanosleep(ns);
    if (ns < 1024) ns <<= 1;
  }
  return false;
}

// Bulk (non-tensor) async copy global -> shared, completion counted on `bar`.
// Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                            uint32_t& r3, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                                  uint32_t& r3, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// D = A(16x16, row) * B(16x8, col) + D, f16 inputs, f32 accumulate.
__device__ __forceinline__ void mma_16816(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// 8x8 b16 transpose across the warp (fragment layout: row lane/4, cols 2*(lane%4)+{0,1}).
// RoPE angle of pair i at position pos_eff (LLM_RoPE.Apply_Sections,
// src/llm/llm_rope.adb:84-200, and k_fattn_prep, gpu/gpu_matvec.cu:1449-1503):
// theta = pos/base^(2i/rd), x freq_scale or the YaRN blend, / ff[i]. Shared
// by the prep kernel and the fused decode so both rotate identically.
__device__ __forceinline__ float rope_angle(int i, int pos_eff, int rd, float base,
                                            float freq_scale, int yarn_on, float corr_lo,
                                            float corr_hi, const float* ff, int use_ff) {
  float extrap = (float)pos_eff / powf(base, (float)(2 * i) / (float)rd);
  float th;
  if (yarn_on) {
    float interp = freq_scale * extrap;
    float y = ((float)i - corr_lo) / fmaxf(0.001f, corr_hi - corr_lo);
    float ramp = 1.0f - fminf(1.0f, fmaxf(0.0f, y));
    th = interp * (1.0f - ramp) + extrap * ramp;
  } else {
    th = extrap * freq_scale;
  }
  if (use_ff) th = th / ff[i];
  return th;
}

// RoPE parameters of the pre-attention step (LLM_RoPE.Apply_Sections,
// src/llm/llm_rope.adb:84-200; k_fattn_prep, gpu/gpu_matvec.cu:1449-1503).
struct RopeArgs {
  const float* ff;          // per-pair frequency divisors, or null
  float base, freq_scale, m_scale, corr_lo, corr_hi;
  int rd, yarn_on, use_ff, interleaved, sec_total;
};

// One warp normalises one head row: sh[d] <- x[d] / rms * w[d] (or x[d]
// without weights), rms = sqrt(sum x^2 / hd + eps). The sum is reduced in a
// fixed order (lane-strided partial sums, then a butterfly), so every user
// of this helper - the prep kernel and the fused decode's appends - writes
// bit-identical rows. sh: hd floats of shared memory owned by the warp.
__device__ __forceinline__ void warp_norm_row(const float* __restrict__ x,
                                              const float* __restrict__ w, float eps, int hd,
                                              float* sh, int lane) {
  float ss = 0.f;
  if (hd <= 256) {
    // every load issued before any is used: one memory round trip per row,
    // which matters when x is pinned host memory read over PCIe
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = lane + 32 * j < hd ? x[lane + 32 * j] : 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (lane + 32 * j < hd) {
        sh[lane + 32 * j] = v[j];
        ss = __fadd_rn(ss, __fmul_rn(v[j], v[j]));
      }
    }
  } else {
    for (int d = lane; d < hd; d += 32) {
      const float v = x[d];
      sh[d] = v;
      ss = __fadd_rn(ss, __fmul_rn(v, v));
    }
  }
  if (w) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
    const float rms = sqrtf(ss / (float)hd + eps);
    for (int d = lane; d < hd; d += 32) sh[d] = __fmul_rn(sh[d] / rms, w[d]);
  }
  __syncwarp();
}

// Rotation of pair i (0 <= i < rd/2) of a normalised row: the pair's two
// dims d1 < d2 (NeoX: i, i + rd/2; interleaved: 2i, 2i + 1) and their
// rotated values. Pairs i >= sec_total rotate at position 0 (the reference's
// section quirk). One angle per pair.
__device__ __forceinline__ void rope_pair(const float* sh, int i, int pos, const RopeArgs& r,
                                          int& d1, int& d2, float& o1, float& o2) {
  if (r.interleaved) { d1 = 2 * i; d2 = d1 + 1; }
  else { d1 = i; d2 = i + r.rd / 2; }
  const int pos_eff = i < r.sec_total ? pos : 0;
  const float th = rope_angle(i, pos_eff, r.rd, r.base, r.freq_scale, r.yarn_on, r.corr_lo,
                              r.corr_hi, r.ff, r.use_ff);
  const float c = __fmul_rn(cosf(th), r.m_scale), sn = __fmul_rn(sinf(th), r.m_scale);
  const float x1 = sh[d1], x2 = sh[d2];
  o1 = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, sn));
  o2 = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, sn));
}

__device__ __forceinline__ uint32_t lds_u32(uint32_t saddr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(saddr));
  return v;
}

__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

}  // namespace aspida

#define ASPIDA_CHECK_LAUNCH() \
  do { cudaError_t _e = cudaGetLastError(); if (_e != cudaSuccess) return aspida::record_status((int)_e); } while (0)
