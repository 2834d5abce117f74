// kv_state.cu — resident fp16 KV caches behind integer handles, prefix
// snapshots, and the library's status latch.
//
// Semantics follow the shim's handle table (gpu/gpu_matvec.cu:1312-1425):
// handles index a table whose freed slots are reused; a snapshot copies the
// leading `rows` rows of K and V (the prefix of a positional cache is its
// leading block); restore copies them back. Unlike the shim there is no
// per-head score scratch: the decode kernels keep scores on chip.
#include <mutex>
#include <vector>
#include <atomic>
#include <cstdio>

#include "common.cuh"

namespace aspida {

namespace {

struct KvState {
  __half* K = nullptr;
  __half* V = nullptr;
  int max_len = 0, kvd = 0;
  bool live = false;
};
struct KvSnap {
  __half* K = nullptr;
  __half* V = nullptr;
  int rows = 0, kvd = 0;
  bool live = false;
};

std::mutex g_mu;                 // guards both tables
std::vector<KvState> g_states;
std::vector<int> g_state_free;
std::vector<KvSnap> g_snaps;
std::vector<int> g_snap_free;

std::atomic<int> g_last_status{0};
std::atomic<int> g_fail_allocs{0};

cudaError_t dev_alloc(void** p, size_t bytes) {
  int n = g_fail_allocs.load();
  while (n > 0) {
    if (g_fail_allocs.compare_exchange_weak(n, n - 1)) {
      *p = nullptr;
      return cudaErrorMemoryAllocation;
    }
  }
  return cudaMalloc(p, bytes);
}

}  // namespace

int record_status(int status) {
  if (status != 0) {
    int zero = 0;
    g_last_status.compare_exchange_strong(zero, status);
  }
  return status;
}

int num_sms() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (cached[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

// The status word is a file-scope device variable: every device that loads
// the library holds its own zero-initialised copy, so looking it up needs no
// allocation and no synchronisation (safe on a capturing stream). Host code
// only knows a stand-in for the symbol; the device address is resolved per
// device, with that device current, and cached.
static __device__ __align__(16) DeviceStatus g_dev_status;

DeviceStatus* device_status_ptr() {
  static std::mutex mu;
  static DeviceStatus* per_dev[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  if (dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(mu);
  if (!per_dev[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_dev_status) != cudaSuccess) return nullptr;
    per_dev[dev] = static_cast<DeviceStatus*>(p);
  }
  return per_dev[dev];
}

// Accessors used by the other translation units.
bool kv_lookup(int handle, __half** K, __half** V, int* max_len, int* kvd) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (handle < 0 || handle >= (int)g_states.size() || !g_states[handle].live) return false;
  const KvState& s = g_states[handle];
  if (K) *K = s.K;
  if (V) *V = s.V;
  if (max_len) *max_len = s.max_len;
  if (kvd) *kvd = s.kvd;
  return true;
}

}  // namespace aspida

using namespace aspida;

extern "C" int aspida_gpu_fattn_new(int max_len, int kvd, int nq) {
  if (max_len <= 0 || kvd <= 0 || nq <= 0) {
    record_status(ASPIDA_ERR_ARG);
    return -1;
  }
  size_t bytes = (size_t)max_len * kvd * sizeof(__half);
  KvState st;
  st.max_len = max_len;
  st.kvd = kvd;
  if (dev_alloc((void**)&st.K, bytes) != cudaSuccess) {
    record_status(ASPIDA_ERR_NOMEM);
    return -1;
  }
  if (dev_alloc((void**)&st.V, bytes) != cudaSuccess) {
    cudaFree(st.K);
    record_status(ASPIDA_ERR_NOMEM);
    return -1;
  }
  st.live = true;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_state_free.empty()) {
    int h = g_state_free.back();
    g_state_free.pop_back();
    g_states[h] = st;
    return h;
  }
  g_states.push_back(st);
  return (int)g_states.size() - 1;
}

extern "C" void aspida_gpu_fattn_free(int handle) {
  cudaDeviceSynchronize();  // in-flight work may still read the cache
  std::lock_guard<std::mutex> lk(g_mu);
  if (handle < 0 || handle >= (int)g_states.size() || !g_states[handle].live) return;
  KvState& st = g_states[handle];
  cudaFree(st.K);
  cudaFree(st.V);
  st = KvState();
  g_state_free.push_back(handle);
}

extern "C" int aspida_gpu_fattn_snapshot(int handle, int rows, int slot) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (handle < 0 || handle >= (int)g_states.size() || !g_states[handle].live) {
    record_status(ASPIDA_ERR_HANDLE);
    return -1;
  }
  const KvState& st = g_states[handle];
  if (rows <= 0 || rows > st.max_len) {
    record_status(ASPIDA_ERR_ARG);
    return -1;
  }
  size_t bytes = (size_t)rows * st.kvd * sizeof(__half);
  KvSnap sn;
  bool reuse = slot >= 0 && slot < (int)g_snaps.size() && g_snaps[slot].live &&
               g_snaps[slot].rows == rows && g_snaps[slot].kvd == st.kvd;
  if (reuse) {
    sn = g_snaps[slot];
  } else {
    if (dev_alloc((void**)&sn.K, bytes) != cudaSuccess) {
      record_status(ASPIDA_ERR_NOMEM);
      return -1;
    }
    if (dev_alloc((void**)&sn.V, bytes) != cudaSuccess) {
      cudaFree(sn.K);
      record_status(ASPIDA_ERR_NOMEM);
      return -1;
    }
    sn.rows = rows;
    sn.kvd = st.kvd;
    sn.live = true;
  }
  if (cuda_status(cudaMemcpy(sn.K, st.K, bytes, cudaMemcpyDeviceToDevice)) ||
      cuda_status(cudaMemcpy(sn.V, st.V, bytes, cudaMemcpyDeviceToDevice))) {
    if (!reuse) { cudaFree(sn.K); cudaFree(sn.V); }
    return -1;
  }
  if (slot >= 0 && slot < (int)g_snaps.size()) {
    if (!reuse && g_snaps[slot].live) {  // different geometry: replace
      cudaFree(g_snaps[slot].K);
      cudaFree(g_snaps[slot].V);
    }
    g_snaps[slot] = sn;
    return slot;
  }
  if (!g_snap_free.empty()) {
    int s = g_snap_free.back();
    g_snap_free.pop_back();
    g_snaps[s] = sn;
    return s;
  }
  g_snaps.push_back(sn);
  return (int)g_snaps.size() - 1;
}

extern "C" int aspida_gpu_fattn_restore(int handle, int slot) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (handle < 0 || handle >= (int)g_states.size() || !g_states[handle].live ||
      slot < 0 || slot >= (int)g_snaps.size() || !g_snaps[slot].live) {
    record_status(ASPIDA_ERR_HANDLE);
    return -1;
  }
  KvState& st = g_states[handle];
  const KvSnap& sn = g_snaps[slot];
  if (sn.kvd != st.kvd || sn.rows > st.max_len) {
    record_status(ASPIDA_ERR_ARG);
    return -1;
  }
  size_t bytes = (size_t)sn.rows * st.kvd * sizeof(__half);
  if (cuda_status(cudaMemcpy(st.K, sn.K, bytes, cudaMemcpyDeviceToDevice)) ||
      cuda_status(cudaMemcpy(st.V, sn.V, bytes, cudaMemcpyDeviceToDevice)))
    return -1;
  return 0;
}

extern "C" void aspida_gpu_prefix_reset(void) {
  cudaDeviceSynchronize();
  std::lock_guard<std::mutex> lk(g_mu);
  for (auto& sn : g_snaps) {
    if (sn.live) {
      cudaFree(sn.K);
      cudaFree(sn.V);
    }
  }
  g_snaps.clear();
  g_snap_free.clear();
}

extern "C" int aspida_gpu_last_error(void) {
  int s = g_last_status.exchange(0);
  if (s != 0) return s;
  return (int)cudaGetLastError();
}

extern "C" int aspida_gpu_fattn_kv(int handle, void** K, void** V, int* max_len, int* kvd) {
  __half *k = nullptr, *v = nullptr;
  if (!kv_lookup(handle, &k, &v, max_len, kvd)) return record_status(ASPIDA_ERR_HANDLE);
  if (K) *K = k;
  if (V) *V = v;
  return 0;
}

extern "C" int aspida_attn_device_status(void) {
  DeviceStatus* d = device_status_ptr();
  if (!d) return record_status(ASPIDA_ERR_UNSUPPORTED);
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return record_status((int)e);
  DeviceStatus h{0, 0};
  e = cudaMemcpy(&h, d, sizeof(h), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return record_status((int)e);
  if (h.code != 0) {
    const DeviceStatus zero{0, 0};
    cudaMemcpy(d, &zero, sizeof(zero), cudaMemcpyHostToDevice);
    return record_status(ASPIDA_ERR_DEVICE);
  }
  return 0;
}

extern "C" int aspida_attn_device_status_where(void) {
  DeviceStatus* d = device_status_ptr();
  if (!d) return record_status(ASPIDA_ERR_UNSUPPORTED);
  DeviceStatus h{0, 0};
  cudaError_t e = cudaMemcpy(&h, d, sizeof(h), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return record_status((int)e);
  return h.code ? h.where : 0;
}

extern "C" void aspida_attn_debug_fail_allocs(int n) { g_fail_allocs.store(n > 0 ? n : 0); }
