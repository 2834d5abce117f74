// step_host.cu — host-buffer decode step over resident KV states: the
// attention half of the shim's aspida_gpu_fattn_step / chain_forward_batch
// (gpu/gpu_matvec.cu:1613-1666, 2783-2894) without the projections.
//
// Per call: one H2D of the lane descriptors (positions, bounds, K/V table),
// H2D of q/k/v, the batched prep (RoPE + fp16 K/V append at pos[b]), the
// split-KV decode, and a stream synchronise. Buffers in pinned host memory
// that the device can address (cudaMallocHost / cudaHostRegister) are used in
// place over PCIe: the prep kernel reads pinned q/k/v directly (no H2D copy
// calls, every row's loads in flight at once), and the decode writes a pinned
// `out` directly while other CTAs are still streaming the cache (no D2H copy
// after it). Pageable buffers go through device staging with one copy each.
// Device staging is cached per (device, stream) and grown on demand, so calls
// on different streams do not share scratch.
#include <map>
#include <mutex>
#include <vector>
#include <utility>
#include <cstring>

#include "common.cuh"

namespace aspida {

bool kv_lookup(int handle, __half** K, __half** V, int* max_len, int* kvd);
int launch_prep_lanes(const float* q, const float* k, const float* v, int B, int nq, int nkv,
                      int hd, void* q_out, __half* const* Ktab, __half* const* Vtab,
                      const int* pos, const int* max_len, int rd, float base, int interleaved,
                      cudaStream_t st);
int decode(const float* q, const float* gate, const void* const* K, const void* const* V,
           const int* pos, const int* max_len, float* out, int B, int nq, int nkv, int hd,
           float scale, int window, float softcap, int max_kv_len, int chunk, void* ws,
           size_t ws_bytes, cudaStream_t st, bool after_prep);
size_t decode_workspace_size(int B, int nq, int nkv, int hd, int max_kv_len, int chunk);


namespace {

struct Staging {
  void* dev = nullptr;       // one device block, carved below
  size_t dev_bytes = 0;
  void* pinned = nullptr;    // lane descriptors, host side
  size_t pinned_bytes = 0;
  bool pending = false;      // copies from `pinned` may still be in flight
};

std::mutex g_stage_mu;
std::map<std::pair<int, cudaStream_t>, Staging> g_stage;

size_t al256(size_t x) { return (x + 255) / 256 * 256; }

}  // namespace
}  // namespace aspida

using namespace aspida;

extern "C" int aspida_attn_step_host(const int* handles, int B, const float* q, const float* k,
                                     const float* v, const int* pos, float* out, int nq, int nkv,
                                     int hd, float scale, int window, float softcap, int rd,
                                     float base, int interleaved, void* stream) {
  if (B <= 0) return 0;
  if (!handles || !q || !k || !v || !pos || !out || nq <= 0 || nkv <= 0 || nq % nkv)
    return record_status(ASPIDA_ERR_ARG);
  cudaStream_t st = (cudaStream_t)stream;
  const int kvd = nkv * hd;

  // Resolve the lanes on the host.
  std::vector<__half*> Kp(B), Vp(B);
  std::vector<int> ml(B);
  int max_kv = 1;
  for (int b = 0; b < B; ++b) {
    int skvd = 0;
    if (!kv_lookup(handles[b], &Kp[b], &Vp[b], &ml[b], &skvd)) return record_status(ASPIDA_ERR_HANDLE);
    if (skvd != kvd) return record_status(ASPIDA_ERR_ARG);
    if (pos[b] < 0 || pos[b] >= ml[b]) return record_status(ASPIDA_ERR_ARG);
    max_kv = std::max(max_kv, pos[b] + 1);
  }

  const size_t desc_bytes = al256((size_t)B * (2 * sizeof(int) + 2 * sizeof(void*)));
  const size_t qb = al256((size_t)B * nq * hd * sizeof(float));
  const size_t kb = al256((size_t)B * kvd * sizeof(float));
  const size_t ws = al256(decode_workspace_size(B, nq, nkv, hd, max_kv, 0));
  const size_t need = desc_bytes + 3 * qb + 2 * kb + ws;  // q, q_roped, out, k, v, ws

  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(g_stage_mu);
  Staging& s = g_stage[{dev, st}];
  if (s.dev_bytes < need) {
    if (s.dev) { cudaStreamSynchronize(st); cudaFree(s.dev); s.dev = nullptr; s.dev_bytes = 0; }
    if (cudaMalloc(&s.dev, need) != cudaSuccess) return record_status(ASPIDA_ERR_NOMEM);
    s.dev_bytes = need;
  }
  if (s.pinned_bytes < desc_bytes) {
    if (s.pinned) { cudaStreamSynchronize(st); cudaFreeHost(s.pinned); s.pinned = nullptr; s.pinned_bytes = 0; }
    if (cudaMallocHost(&s.pinned, desc_bytes) != cudaSuccess) return record_status(ASPIDA_ERR_NOMEM);
    s.pinned_bytes = desc_bytes;
  }
  // The pinned descriptor block is reused by the next call on this stream:
  // a call that returned early may have left its H2D in flight (a complete
  // call ends with a synchronisation, so there is nothing to wait for).
  if (s.pending) {
    cudaStreamSynchronize(st);
    s.pending = false;
  }

  unsigned char* hp = static_cast<unsigned char*>(s.pinned);
  __half** hK = reinterpret_cast<__half**>(hp);
  __half** hV = hK + B;
  int* hpos = reinterpret_cast<int*>(hV + B);
  int* hml = hpos + B;
  for (int b = 0; b < B; ++b) { hK[b] = Kp[b]; hV[b] = Vp[b]; hpos[b] = pos[b]; hml[b] = ml[b]; }

  unsigned char* d = static_cast<unsigned char*>(s.dev);
  __half** dK = reinterpret_cast<__half**>(d);
  __half** dV = dK + B;
  int* dpos = reinterpret_cast<int*>(dV + B);
  int* dml = dpos + B;
  float* dq = reinterpret_cast<float*>(d + desc_bytes);
  float* dqr = reinterpret_cast<float*>(d + desc_bytes + qb);
  float* dout = reinterpret_cast<float*>(d + desc_bytes + 2 * qb);
  float* dk = reinterpret_cast<float*>(d + desc_bytes + 3 * qb);
  float* dv = reinterpret_cast<float*>(d + desc_bytes + 3 * qb + kb);
  void* dws = d + desc_bytes + 3 * qb + 2 * kb;

  const size_t qbytes = (size_t)B * nq * hd * sizeof(float), kbytes = (size_t)B * kvd * sizeof(float);
  // device address of a pinned host buffer, or null (pageable / unknown memory)
  auto mapped = [](const void* h) -> void* {
    cudaPointerAttributes pa;
    if (cudaPointerGetAttributes(&pa, h) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    return pa.type == cudaMemoryTypeHost ? pa.devicePointer : nullptr;
  };
  float* out_direct = static_cast<float*>(mapped(out));
#ifndef ASPIDA_STEP_NO_ZC_IN
  const float* qd = static_cast<const float*>(mapped(q));
  const float* kd = static_cast<const float*>(mapped(k));
  const float* vd = static_cast<const float*>(mapped(v));
  if (!qd || !kd || !vd) qd = kd = vd = nullptr;
#endif
  int rc = 0;
  s.pending = true;
  if ((rc = cuda_status(cudaMemcpyAsync(d, hp, desc_bytes, cudaMemcpyHostToDevice, st)))) return rc;
#ifndef ASPIDA_STEP_NO_ZC_IN
  if (qd) {
    dq = const_cast<float*>(qd);
    dk = const_cast<float*>(kd);
    dv = const_cast<float*>(vd);
  } else
#endif
  {
    if ((rc = cuda_status(cudaMemcpyAsync(dq, q, qbytes, cudaMemcpyHostToDevice, st)))) return rc;
    if ((rc = cuda_status(cudaMemcpyAsync(dk, k, kbytes, cudaMemcpyHostToDevice, st)))) return rc;
    if ((rc = cuda_status(cudaMemcpyAsync(dv, v, kbytes, cudaMemcpyHostToDevice, st)))) return rc;
  }
  // prep, then decode: measured faster on B200 than the single-launch
  // aspida_attn_decode_fused (config 2: 0.137 vs ~0.107 ms)
  if ((rc = launch_prep_lanes(dq, dk, dv, B, nq, nkv, hd, dqr, dK, dV, dpos, dml, rd, base,
                              interleaved, st)))
    return rc;
  if ((rc = decode(dqr, nullptr, reinterpret_cast<const void* const*>(dK),
                   reinterpret_cast<const void* const*>(dV), dpos, dml,
                   out_direct ? out_direct : dout, B, nq, nkv, hd, scale, window, softcap, max_kv,
                   0, dws, ws, st, true)))
    return rc;
  if (!out_direct &&
      (rc = cuda_status(cudaMemcpyAsync(out, dout, qbytes, cudaMemcpyDeviceToHost, st))))
    return rc;
  rc = cuda_status(cudaStreamSynchronize(st));
  if (rc == 0) s.pending = false;
  return rc;
}
