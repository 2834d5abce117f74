// peer.cu — the cross-GPU exchange of sequence-parallel decode over NVLink
// peer memory, fused with the log-sum-exp merge.
//
// The reference has no multi-GPU inference (its only distributed code is a
// TCP gradient exchange for training, gpu/dp_node.cu); the merge is the
// split-K combine of gpu/fattn_sk.cu:84-97.
//
// Every rank owns one receive buffer (cudaMalloc, zero-filled), shared with
// the other ranks of the node once through a CUDA IPC handle. Layout: two
// banks (step parity), each `world` 16-byte-aligned slots of one packed
// partial [m | l | o] (rows * (hd + 2) floats), then the banks' arrival
// flags (8 uint64 each). A step (tag = its 1-based step number, the same on
// every rank):
//   1. block p stores this rank's partial into slot `rank` of rank p's
//      buffer (plain stores through the peer mapping), then raises rank p's
//      flag[rank] = tag with a system-scope release;
//   2. every block waits (bounded) until all of its own buffer's flags of
//      this bank read `tag` (system-scope acquire), then merges its share of
//      the outputs (one per thread) from the `world` slots.
// Two banks are enough: a rank writes bank (t mod 2) of step t + 2 only
// after it has received every rank's step t + 1 partial, and each rank
// sends that only after its own step-t merge has finished reading bank
// (t mod 2). A wait that runs out (a rank that never arrives) sets the
// device status word and leaves; nothing spins without a bound.
#include <algorithm>
#include <cstring>

#include "common.cuh"

namespace aspida {
namespace {

constexpr int kMaxWorld = 8;
constexpr long long kDefaultWaitLimit = 1LL << 22;   // flag polls: seconds with the backoff

struct PeerArgs {
  float* recv[kMaxWorld];       // every rank's receive buffer (this rank's mapping)
  const float* part;            // this rank's packed partial
  const float* gate;
  float* out;
  DeviceStatus* status;
  int* fail_word;               // optional caller word (e.g. host-mapped), set on timeout
  long long wait_limit;         // polls per flag before giving up
  long per;                     // floats per partial: rows * (hd + 2)
  long stride;                  // floats per slot: per rounded up to 4 (16-byte slots)
  long bank_floats;             // floats of one bank's slots
  long flags_off;               // float offset of the flags (bank 0)
  int world, rank, rows, hd;
  unsigned long long tag;
};

__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(256) exchange_merge_kernel(const PeerArgs a) {
  const int bank = (int)(a.tag & 1);
  const int p = blockIdx.x;                     // blocks 0..world-1 also send to rank p
  // 1. send: this rank's partial -> slot `rank` of rank p's bank
  if (p < a.world) {
    float* dst = a.recv[p] + bank * a.bank_floats + (long)a.rank * a.stride;
    const float4* s4 = reinterpret_cast<const float4*>(a.part);
    float4* d4 = reinterpret_cast<float4*>(dst);
    const long n4 = a.per / 4;
    for (long i = threadIdx.x; i < n4; i += blockDim.x) d4[i] = s4[i];
    for (long i = n4 * 4 + threadIdx.x; i < a.per; i += blockDim.x) dst[i] = a.part[i];
    // the barrier makes the block's stores observed by thread 0, whose
    // system-scope fence + release store then publishes them (cumulativity)
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned long long* fl = reinterpret_cast<unsigned long long*>(a.recv[p] + a.flags_off) +
                               bank * kMaxWorld + a.rank;
      __threadfence_system();
      st_release_sys(fl, a.tag);
    }
  }
  // 2. wait for every rank's partial in this rank's own buffer
  const unsigned long long* myfl =
      reinterpret_cast<const unsigned long long*>(a.recv[a.rank] + a.flags_off) + bank * kMaxWorld;
  __shared__ int ok;
  if (threadIdx.x == 0) {
    ok = 1;
    for (int s = 0; s < a.world && ok; ++s) {
      uint32_t ns = 32;
      long it = 0;
      while (ld_acquire_sys(myfl + s) != a.tag) {
        if (++it > a.wait_limit) {                  // default limit: ~seconds with the backoff
          ok = 0;
          if (a.status) { atomicExch(&a.status->code, kDevTimeoutMbar); a.status->where = 60; }
          if (a.fail_word) {
            *(volatile int*)a.fail_word = kDevTimeoutMbar;
            __threadfence_system();
          }
          break;
        }
        if (it > 1024) {
          __nanosleep(ns);
          if (ns < 1024) ns <<= 1;
        }
      }
    }
  }
  // thread 0's acquire synchronises with every sender's release; the barrier
  // orders the other threads' reads after it
  __syncthreads();
  if (!ok) return;
  // 3. merge: one output element per thread; the loads of the `world` slots
  // are independent, so each thread waits about one L2 round trip
  const float* base = a.recv[a.rank] + bank * a.bank_floats;
  const long rows = a.rows, n = rows * a.hd;
  for (long e = (long)blockIdx.x * blockDim.x + threadIdx.x; e < n;
       e += (long)gridDim.x * blockDim.x) {
    const long r = e / a.hd;
    float ms[kMaxWorld], ls[kMaxWorld], os[kMaxWorld];
#pragma unroll
    for (int s = 0; s < kMaxWorld; ++s) {
      if (s < a.world) {
        const float* sl = base + s * a.stride;      // written by rank s over NVLink: via L2
        ms[s] = __ldcg(sl + r);
        ls[s] = __ldcg(sl + rows + r);
        os[s] = __ldcg(sl + 2 * rows + e);
      }
    }
    float M = -3.402823466e38f;
#pragma unroll
    for (int s = 0; s < kMaxWorld; ++s)
      if (s < a.world) M = fmaxf(M, ms[s]);
    float acc = 0.f, L = 0.f;
#pragma unroll
    for (int s = 0; s < kMaxWorld; ++s) {
      if (s < a.world && ms[s] >= -3.0e38f) {       // skip empty slices
        const float w = expf(ms[s] - M);
        L += w * ls[s];
        acc += w * os[s];
      }
    }
    float v = L > 0.f ? acc / L : 0.f;
    if (a.gate) v *= 1.f / (1.f + expf(-a.gate[e]));
    a.out[e] = v;
  }
}

size_t layout(int world, int rows, int hd, long* per, long* stride, long* bank_floats,
              long* flags_off) {
  *per = (long)rows * (hd + 2);
  *stride = (*per + 3) / 4 * 4;
  *bank_floats = (long)world * *stride;
  *flags_off = (2 * *bank_floats + 63) / 64 * 64;           // 256-byte aligned flags
  return (size_t)(*flags_off) * sizeof(float) + 2 * kMaxWorld * sizeof(unsigned long long);
}

}  // namespace
}  // namespace aspida

using namespace aspida;

extern "C" size_t aspida_attn_peer_buffer_size(int world, int rows, int hd) {
  if (world <= 0 || world > kMaxWorld || rows <= 0 || hd <= 0) return 0;
  long a, b, c, d;
  return layout(world, rows, hd, &a, &b, &c, &d);
}

extern "C" int aspida_attn_peer_alloc(size_t bytes, void** ptr, void* ipc_handle) {
  if (!ptr || !ipc_handle || bytes == 0) return record_status(ASPIDA_ERR_ARG);
  *ptr = nullptr;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return record_status(ASPIDA_ERR_NOMEM);
  cudaError_t e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) {
    cudaIpcMemHandle_t h;
    e = cudaIpcGetMemHandle(&h, p);
    if (e == cudaSuccess) memcpy(ipc_handle, &h, sizeof(h));
  }
  if (e != cudaSuccess) {
    cudaFree(p);
    return record_status((int)e);
  }
  *ptr = p;
  return 0;
}

extern "C" int aspida_attn_peer_open(const void* ipc_handle, void** peer_ptr) {
  if (!ipc_handle || !peer_ptr) return record_status(ASPIDA_ERR_ARG);
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  return cuda_status(cudaIpcOpenMemHandle(peer_ptr, h, cudaIpcMemLazyEnablePeerAccess));
}

extern "C" int aspida_attn_peer_close(void* peer_ptr) {
  if (!peer_ptr) return 0;
  return cuda_status(cudaIpcCloseMemHandle(peer_ptr));
}

extern "C" int aspida_attn_peer_free(void* ptr) {
  if (!ptr) return 0;
  return cuda_status(cudaFree(ptr));
}

extern "C" int aspida_attn_exchange_merge_ex(const float* part, void* const* recv, int world,
                                             int rank, unsigned long long step,
                                             const float* gate, float* out, int rows, int hd,
                                             int* fail_word, long long wait_limit,
                                             void* stream) {
  if (rows <= 0) return 0;
  if (!part || !recv || !out || world <= 0 || world > kMaxWorld || rank < 0 || rank >= world ||
      hd <= 0 || step == 0 || ((uintptr_t)part & 15) || wait_limit < 0)
    return record_status(ASPIDA_ERR_ARG);
  PeerArgs a{};
  for (int s = 0; s < world; ++s) {
    if (!recv[s] || ((uintptr_t)recv[s] & 255)) return record_status(ASPIDA_ERR_ARG);
    a.recv[s] = static_cast<float*>(recv[s]);
  }
  layout(world, rows, hd, &a.per, &a.stride, &a.bank_floats, &a.flags_off);
  a.part = part;
  a.gate = gate;
  a.out = out;
  a.status = device_status_ptr();
  a.fail_word = fail_word;
  a.wait_limit = wait_limit > 0 ? wait_limit : kDefaultWaitLimit;
  a.world = world;
  a.rank = rank;
  a.rows = rows;
  a.hd = hd;
  a.tag = step;
  // blocks: at least one per destination rank, enough for one thread per output
  const long outs = (long)rows * hd;
  const int blocks = (int)std::max<long>(world, std::min<long>((outs + 255) / 256, 1024));
  exchange_merge_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(a);
  ASPIDA_CHECK_LAUNCH();
  return 0;
}

extern "C" int aspida_attn_exchange_merge(const float* part, void* const* recv, int world,
                                          int rank, unsigned long long step, const float* gate,
                                          float* out, int rows, int hd, void* stream) {
  return aspida_attn_exchange_merge_ex(part, recv, world, rank, step, gate, out, rows, hd,
                                       nullptr, 0, stream);
}
