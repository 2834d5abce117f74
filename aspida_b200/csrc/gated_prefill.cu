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

std::mutex g_mu;
std::map<std::pair<int, cudaStream_t>, std::pair<void*, size_t>> g_scratch;

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
    void* qh = nullptr;
    float* part = nullptr;
    const int nsplit = prefill_split_plan(P, pos_start, nq, hd, 0);
    const size_t qbytes = ((size_t)n * 2 + 255) / 256 * 256;
    {
      int dev = 0;
      cudaGetDevice(&dev);
      std::lock_guard<std::mutex> lk(g_mu);
      auto& s = g_scratch[{dev, st}];
      const size_t need = qbytes + prefill_split_bytes(nsplit, P, nq, hd);
      if (s.second < need) {
        if (s.first) { cudaStreamSynchronize(st); cudaFree(s.first); s = {nullptr, 0}; }
        if (cudaMalloc(&s.first, need) != cudaSuccess) rc = record_status(ASPIDA_ERR_NOMEM);
        else s.second = need;
      }
      qh = s.first;
      if (nsplit > 1 && qh) part = reinterpret_cast<float*>(static_cast<char*>(qh) + qbytes);
    }
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
