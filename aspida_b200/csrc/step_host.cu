// step_host.cu — host-buffer decode step over resident KV states: the
// attention half of the shim's aspida_gpu_fattn_step / chain_forward_batch
// (gpu/gpu_matvec.cu:1613-1666, 2783-2894) without the projections.
//
// Per call: one H2D of the lane descriptors (positions, bounds, K/V table),
// then, per chunk of the batch, H2D of its q/k/v, the batched prep (RoPE +
// fp16 K/V append at pos[b]), the split-KV decode and the D2H of its output;
// finally a stream synchronise. A batch of 16 or more sequences runs as two
// chunks on two streams (the caller's and a library-owned one), so the second
// chunk's host-to-device copies run under the first chunk's decode and the
// first chunk's output copy under the second's: the PCIe transfers, which at
// config 2 are a third of the step, mostly leave the critical path.
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
           size_t ws_bytes, cudaStream_t st);
size_t decode_workspace_size(int B, int nq, int nkv, int hd, int max_kv_len, int chunk);


namespace {

struct Staging {
  void* dev = nullptr;       // one device block, carved below
  size_t dev_bytes = 0;
  void* pinned = nullptr;    // lane descriptors, host side
  size_t pinned_bytes = 0;
  bool pending = false;      // copies from `pinned` may still be in flight
  cudaStream_t aux = nullptr;          // second stream for the second chunk
  cudaEvent_t ev_desc = nullptr, ev_done = nullptr;
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

  const int nch = B >= 16 ? 2 : 1;                       // batch chunks
  const int Bc[2] = {nch == 2 ? B / 2 : B, nch == 2 ? B - B / 2 : 0};
  int mkv[2] = {1, 1};
  for (int b = 0; b < B; ++b) {
    const int c = b < Bc[0] ? 0 : 1;
    mkv[c] = std::max(mkv[c], pos[b] + 1);
  }
  (void)max_kv;
  const size_t desc_bytes = al256((size_t)B * (2 * sizeof(int) + 2 * sizeof(void*)));
  const size_t qb = al256((size_t)B * nq * hd * sizeof(float));
  const size_t kb = al256((size_t)B * kvd * sizeof(float));
  size_t wsz[2] = {0, 0};
  for (int c = 0; c < nch; ++c) wsz[c] = al256(decode_workspace_size(Bc[c], nq, nkv, hd, mkv[c], 0));
  const size_t need = desc_bytes + 3 * qb + 2 * kb + wsz[0] + wsz[1];  // q, q_roped, out, k, v, ws

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
  if (nch == 2 && !s.aux) {
    if (cudaStreamCreateWithFlags(&s.aux, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&s.ev_desc, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&s.ev_done, cudaEventDisableTiming) != cudaSuccess) {
      cudaGetLastError();
      return record_status(ASPIDA_ERR_NOMEM);
    }
  }
  // The pinned descriptor block is reused by the next call on this stream:
  // a call that returned early may have left its H2D in flight (a complete
  // call ends with a synchronisation, so there is nothing to wait for).
  if (s.pending) {
    cudaStreamSynchronize(st);
    if (s.aux) cudaStreamSynchronize(s.aux);
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
  unsigned char* dws = d + desc_bytes + 3 * qb + 2 * kb;

  const long qrow = (long)nq * hd;
  int rc = 0;
  s.pending = true;
  if ((rc = cuda_status(cudaMemcpyAsync(d, hp, desc_bytes, cudaMemcpyHostToDevice, st)))) return rc;
  if (nch == 2) {
    if ((rc = cuda_status(cudaEventRecord(s.ev_desc, st)))) return rc;
    if ((rc = cuda_status(cudaStreamWaitEvent(s.aux, s.ev_desc, 0)))) return rc;
  }
  for (int c = 0, b0 = 0; c < nch; b0 += Bc[c], ++c) {
    cudaStream_t cs = c == 0 ? st : s.aux;
    const int n = Bc[c];
    const size_t qbytes = (size_t)n * qrow * sizeof(float), kbytes = (size_t)n * kvd * sizeof(float);
    float* cq = dq + b0 * qrow;
    float* cqr = dqr + b0 * qrow;
    float* cout = dout + b0 * qrow;
    float* ck = dk + (long)b0 * kvd;
    float* cv = dv + (long)b0 * kvd;
    if ((rc = cuda_status(cudaMemcpyAsync(cq, q + b0 * qrow, qbytes, cudaMemcpyHostToDevice, cs))))
      return rc;
    if ((rc = cuda_status(cudaMemcpyAsync(ck, k + (long)b0 * kvd, kbytes, cudaMemcpyHostToDevice, cs))))
      return rc;
    if ((rc = cuda_status(cudaMemcpyAsync(cv, v + (long)b0 * kvd, kbytes, cudaMemcpyHostToDevice, cs))))
      return rc;
    // prep, then decode: measured faster on B200 than the single-launch
    // aspida_attn_decode_fused (config 2: 0.137 vs ~0.107 ms)
    if ((rc = launch_prep_lanes(cq, ck, cv, n, nq, nkv, hd, cqr, dK + b0, dV + b0, dpos + b0,
                                dml + b0, rd, base, interleaved, cs)))
      return rc;
    if ((rc = decode(cqr, nullptr, reinterpret_cast<const void* const*>(dK + b0),
                     reinterpret_cast<const void* const*>(dV + b0), dpos + b0, dml + b0, cout, n,
                     nq, nkv, hd, scale, window, softcap, mkv[c], 0, dws + (c ? wsz[0] : 0),
                     wsz[c], cs)))
      return rc;
    if ((rc = cuda_status(cudaMemcpyAsync(out + b0 * qrow, cout, qbytes, cudaMemcpyDeviceToHost, cs))))
      return rc;
  }
  if (nch == 2) {
    if ((rc = cuda_status(cudaEventRecord(s.ev_done, s.aux)))) return rc;
    if ((rc = cuda_status(cudaStreamWaitEvent(st, s.ev_done, 0)))) return rc;
  }
  rc = cuda_status(cudaStreamSynchronize(st));
  if (rc == 0) s.pending = false;
  return rc;
}
