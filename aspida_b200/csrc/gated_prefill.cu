// gated_prefill.cu — the Qwen gated full-attention prefill behind the exact
// argument list of the shim's swap point aspida_ggml_fattn_prefill
// (gpu/fattn_ggml.cuh:109-112): f32 prepped queries [P][nq*hd], the fp16
// resident cache [pos][nkv*hd], the f32 sigmoid gate [P][nq*hd], f32 output,
// scale 1/sqrt(hd), causal over keys 0..pos_start+t. Like the shim, a failure
// zeroes `out` (fattn_ggml.cuh:117-122) so no stale attention is consumed.
//
// The queries are rounded to fp16 for the tensor cores by a small conversion
// kernel into scratch kept per (device, stream) and grown on demand. When a
// short chunk after a long prefix would leave SMs idle (hd 256), the same
// scratch holds split-KV partials (prefill_split_plan).
#include <map>
#include <mutex>
#include <utility>
#include <cmath>

#include "common.cuh"

namespace aspida {

int prefill_batch(int nseq, const void* const* q, const void* const* K, const void* const* V,
                  const float* const* gate, void* const* out, const int* P, const int* pos_start,
                  int out_f32, int nq, int nkv, int hd, float scale, int window, float softcap,
                  cudaStream_t st, const int* block_table, int num_blocks, int block_size,
                  int nsplit, float* part);
int prefill_split_plan(int P, int pos_start, int nq, int hd, int window);
size_t prefill_split_bytes(int nsplit, int P, int nq, int hd);

namespace {

__global__ void f32_to_f16(const float4* __restrict__ in, uint2* __restrict__ out, long n4) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n4; i += (long)gridDim.x * blockDim.x) {
    const float4 v = in[i];
    out[i] = make_uint2(pack_half2(v.x, v.y), pack_half2(v.z, v.w));
  }
}

// Q8_0 -> fp16: out = fp16(float(int8) * float(scale)), one scale per 32
// values along a row (the dequantisation of gpu/fattn_kvhalf.cu:88-92, rounded
// to fp16 for the tensor cores). Eight values per thread.
__global__ void q8_to_f16(const int8_t* __restrict__ q, const __half* __restrict__ sc,
                          uint4* __restrict__ out, long n8) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n8;
       i += (long)gridDim.x * blockDim.x) {
    const uint2 w = reinterpret_cast<const uint2*>(q)[i];
    const float s = __half2float(sc[i >> 2]);          // 8 values of a 32-value block
    const int8_t* b = reinterpret_cast<const int8_t*>(&w);
    uint32_t h[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) h[k] = pack_half2((float)b[2 * k] * s, (float)b[2 * k + 1] * s);
    out[i] = make_uint4(h[0], h[1], h[2], h[3]);
  }
}

std::mutex g_mu;
std::map<std::pair<int, cudaStream_t>, std::pair<void*, size_t>> g_scratch;

// Scratch of at least `need` bytes on (current device, st); null if none.
void* scratch(size_t need, cudaStream_t st) {
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(g_mu);
  auto& s = g_scratch[{dev, st}];
  if (s.second < need) {
    if (s.first) { cudaStreamSynchronize(st); cudaFree(s.first); s = {nullptr, 0}; }
    if (cudaMalloc(&s.first, need) != cudaSuccess) { cudaGetLastError(); return nullptr; }
    s.second = need;
  }
  return s.first;
}

}  // namespace
}  // namespace aspida

using namespace aspida;

extern "C" int aspida_attn_prefill_gated(const float* q_all, const void* K, const void* V,
                                         const float* gate, float* out, int nq, int nkv, int hd,
                                         int P, int pos_start, void* stream) {
  cudaStream_t st = (cudaStream_t)stream;
  if (P <= 0) return 0;
  int rc = 0;
  const long n = (long)P * nq * hd;
  if (!q_all || !K || !V || !out || nq <= 0 || nkv <= 0 || hd <= 0 || (n & 3) ||
      ((uintptr_t)q_all & 15)) {
    rc = record_status(ASPIDA_ERR_ARG);
  } else {
    float* part = nullptr;
    const int nsplit = prefill_split_plan(P, pos_start, nq, hd, 0);
    const size_t qbytes = ((size_t)n * 2 + 255) / 256 * 256;
    void* qh = scratch(qbytes + prefill_split_bytes(nsplit, P, nq, hd), st);
    if (!qh) rc = record_status(ASPIDA_ERR_NOMEM);
    else if (nsplit > 1) part = reinterpret_cast<float*>(static_cast<char*>(qh) + qbytes);
    if (!rc) {
      const long n4 = n / 4;
      const int blocks = (int)std::min<long>((n4 + 255) / 256, (long)num_sms() * 8);
      f32_to_f16<<<blocks, 256, 0, st>>>(reinterpret_cast<const float4*>(q_all),
                                          reinterpret_cast<uint2*>(qh), n4);
      if (cudaError_t e = cudaGetLastError(); e != cudaSuccess) rc = record_status((int)e);
    }
    if (!rc) {
      const void* qv = qh;
      void* ov = out;
      rc = prefill_batch(1, &qv, &K, &V, gate ? &gate : nullptr, &ov, &P, &pos_start, 1, nq,
                         nkv, hd, 1.0f / sqrtf((float)hd), 0, 0.0f, st, nullptr, 0, 0,
                         nsplit, part);
    }
  }
  if (rc) cudaMemsetAsync(out, 0, (size_t)n * sizeof(float), st);  // never leave `out` stale
  return rc;
}

extern "C" int aspida_attn_prefill_q8_gated(const float* q_all, const float* gate, const void* K8,
                                            const void* V8, const void* K_scales,
                                            const void* V_scales, float* out, int nq, int nkv,
                                            int hd, int P, int pos_start, void* stream) {
  cudaStream_t st = (cudaStream_t)stream;
  if (P <= 0) return 0;
  int rc = 0;
  const long n = (long)P * nq * hd;
  const long len = (long)pos_start + P, kv_vals = len * nkv * hd;
  if (!q_all || !K8 || !V8 || !K_scales || !V_scales || !out || nq <= 0 || nkv <= 0 || hd <= 0 ||
      pos_start < 0 || (n & 3) || ((uintptr_t)q_all & 15) || ((uintptr_t)K8 & 7) ||
      ((uintptr_t)V8 & 7) || ((nkv * hd) % 32)) {
    rc = record_status(ASPIDA_ERR_ARG);
  } else if (hd != 64 && hd != 128 && hd != 256) {
    rc = record_status(ASPIDA_ERR_UNSUPPORTED);
  } else {
    // scratch: fp16 queries | fp16 K | fp16 V | split partials
    auto al = [](size_t x) { return (x + 255) / 256 * 256; };
    const int nsplit = prefill_split_plan(P, pos_start, nq, hd, 0);
    const size_t qb = al((size_t)n * 2), kb = al((size_t)kv_vals * 2);
    char* base = static_cast<char*>(
        scratch(qb + 2 * kb + prefill_split_bytes(nsplit, P, nq, hd), st));
    if (!base) {
      rc = record_status(ASPIDA_ERR_NOMEM);
    } else {
      void* qh = base;
      void* Kh = base + qb;
      void* Vh = base + qb + kb;
      float* part = nsplit > 1 ? reinterpret_cast<float*>(base + qb + 2 * kb) : nullptr;
      const int cap = num_sms() * 8;
      f32_to_f16<<<(int)std::min<long>((n / 4 + 255) / 256, cap), 256, 0, st>>>(
          reinterpret_cast<const float4*>(q_all), reinterpret_cast<uint2*>(qh), n / 4);
      const long n8 = kv_vals / 8;
      q8_to_f16<<<(int)std::min<long>((n8 + 255) / 256, cap), 256, 0, st>>>(
          static_cast<const int8_t*>(K8), static_cast<const __half*>(K_scales),
          static_cast<uint4*>(Kh), n8);
      q8_to_f16<<<(int)std::min<long>((n8 + 255) / 256, cap), 256, 0, st>>>(
          static_cast<const int8_t*>(V8), static_cast<const __half*>(V_scales),
          static_cast<uint4*>(Vh), n8);
      if (cudaError_t e = cudaGetLastError(); e != cudaSuccess) rc = record_status((int)e);
      if (!rc) {
        const void* qv = qh;
        const void* Kv = Kh;
        const void* Vv = Vh;
        void* ov = out;
        rc = prefill_batch(1, &qv, &Kv, &Vv, gate ? &gate : nullptr, &ov, &P, &pos_start, 1, nq,
                           nkv, hd, 1.0f / sqrtf((float)hd), 0, 0.0f, st, nullptr, 0, 0, nsplit,
                           part);
      }
    }
  }
  if (rc) cudaMemsetAsync(out, 0, (size_t)n * sizeof(float), st);  // never leave `out` stale
  return rc;
}
