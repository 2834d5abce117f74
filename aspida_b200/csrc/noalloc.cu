// noalloc.cu — decode attention for callers that cannot allocate device
// memory: code running where cudaMalloc is not allowed or not wanted (inside
// an allocator or memory-pool callback, under a fixed memory budget that was
// reserved up front, or in a host thread that must never block on the
// device-wide synchronisation cudaMalloc/cudaFree can imply).
//
// The decode kernel needs scratch for the partial results of sequences that
// are split between CTAs. Here that scratch is a fixed array compiled into
// the library, g_noalloc_ws below, of kNoAllocBytes; every GPU that loads the
// library holds it until the process exits. The status word that the
// kernel's bounded waits write to when they run out is also compiled in; it
// is separate from the one aspida_attn_device_status() reads, so this path
// does not report such a timeout there (the output is then left incomplete).
//
// On the host, the names of these arrays are only host-side stand-ins, not
// device addresses, so the first call on each device looks up their device
// addresses with cudaGetSymbolAddress (with that device current) and caches
// them. Make that first call before any stream capture begins.
//
// The entry point calls no cudaMalloc, cudaFree or other allocating routine.
// Every call shares the one array, which keeps the previous call's contents;
// nothing in it has to start at zero (each call writes every partial it later
// reads). Calls that overlap on the GPU race on the array, so serialise them
// (one stream, or events).
#include <mutex>

#include "common.cuh"

namespace aspida {
int decode_with_status(const float* q, const float* gate, const void* const* K,
                       const void* const* V, const int* pos, const int* max_len, float* out,
                       int B, int nq, int nkv, int hd, float scale, int window, float softcap,
                       int max_kv_len, int chunk, void* ws, size_t ws_bytes,
                       DeviceStatus* status, cudaStream_t st);
size_t decode_workspace_size(int B, int nq, int nkv, int hd, int max_kv_len, int chunk);
}  // namespace aspida

namespace {

constexpr size_t kNoAllocBytes = 16u << 20;   // 16 MiB of decode scratch per GPU

static __device__ __align__(256) unsigned char g_noalloc_ws[kNoAllocBytes];

struct Addrs { void* ws = nullptr; aspida::DeviceStatus* status = nullptr; };
std::mutex g_mu;
Addrs g_addrs[64];

// Device addresses of the scratch array and the status word on the current
// device (looked up once).
int lookup(Addrs& out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return aspida::record_status((int)e);
  if (dev < 0 || dev >= 64) return aspida::record_status(ASPIDA_ERR_UNSUPPORTED);
  std::lock_guard<std::mutex> lk(g_mu);
  Addrs& a = g_addrs[dev];
  if (!a.ws) {
    void* ws = nullptr;
    e = cudaGetSymbolAddress(&ws, g_noalloc_ws);
    if (e != cudaSuccess) return aspida::record_status((int)e);
    aspida::DeviceStatus* st = aspida::device_status_ptr();   // compiled in, no allocation
    if (!st) return aspida::record_status(ASPIDA_ERR_UNSUPPORTED);
    a.ws = ws;
    a.status = st;
  }
  out = a;
  return 0;
}

}  // namespace

extern "C" int aspida_attn_decode_noalloc(const float* q, const float* gate, const void* const* K,
                                          const void* const* V, const int* pos,
                                          const int* max_len, float* out, int B, int nq, int nkv,
                                          int hd, float scale, int window, float softcap,
                                          int max_kv_len, int chunk, void* stream) {
  const size_t need = aspida::decode_workspace_size(B, nq, nkv, hd, max_kv_len, chunk);
  if (need > kNoAllocBytes) {
    // the batch needs more scratch than the compiled-in array holds
    return aspida::record_status(ASPIDA_ERR_WORKSPACE);
  }
  Addrs a;
  if (int rc = lookup(a)) return rc;
  return aspida::decode_with_status(q, gate, K, V, pos, max_len, out, B, nq, nkv, hd, scale,
                                    window, softcap, max_kv_len, chunk, a.ws, kNoAllocBytes,
                                    a.status, (cudaStream_t)stream);
}
