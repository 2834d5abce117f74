// decode.cu — GQA decode attention over the resident fp16 KV cache.
//
// Replaces the shim's k_fattn_attend / k_fattn_attend_b (gpu/gpu_matvec.cu:
// 1507-1609), which run one 256-thread block per query head and so read every
// KV byte nq/nkv times through a two-pass fp32 score scratch. Here:
//
//  * Work item = (sequence b, kv head, chunk of `chunk` keys). All G = nq/nkv
//    query heads of the kv group are handled by the same warp, so each KV byte
//    crosses HBM once. Items are ordered (b, chunk, kv head) and dealt to
//    persistent warps round-robin; the per-sequence item offsets are a prefix
//    sum every CTA computes in shared memory from pos[] (no host round trip,
//    so the launch is graph-capturable).
//  * Each warp owns a ring of STAGES stages of 16 K rows + 16 V rows, filled
//    by the bulk-copy (TMA) engine: one cp.async.bulk of hd*2 bytes per row,
//    completion counted on the stage's mbarrier. Rows are padded by 16 bytes
//    so ldmatrix reads are bank-conflict free.
//  * Scores are computed transposed, S^T = K Q^T, with mma.sync m16n8k16:
//    M = 16 keys, N = 8 query heads (the GQA group; padded when G < 8),
//    K = 16 dims. movmatrix turns the S^T accumulator into the P^T operand of
//    O^T = V^T P^T (M = 16 dims, N = 8 heads, K = 16 keys), so softmax state
//    and O live in registers with no shared-memory round trip.
//  * Online softmax in the log2 domain (scale folded with log2 e), fp32.
//  * A sequence whose range fits one chunk writes its output directly; longer
//    ones write per-chunk (m, l, o) partials to the workspace and a combine
//    kernel merges them (the log-sum-exp merge of gpu/fattn_sk.cu:84-97).
#include <algorithm>
#include <cmath>

#include "common.cuh"

namespace aspida {
namespace {

constexpr int kWarps = 4;     // warps per CTA (each an independent pipeline)
constexpr int kKeys = 16;     // keys per stage
constexpr int kMaxB = 1024;   // sequences per launch (prefix sums in smem)
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kNegBig = -3.402823466e38f;

struct DecodeParams {
  const float* q;
  const float* gate;
  const __half* const* K;
  const __half* const* V;
  const int* pos;       // mode 0
  const int* max_len;   // mode 0, optional
  const int* kv_lo;     // mode 1
  const int* kv_hi;     // mode 1
  float* out;           // mode 0: [B][nq*hd]
  float* part_m;        // mode 1: [B][nq]
  float* part_l;
  float* part_o;        // mode 1: [B][nq][hd]
  int* ws_pref;         // [B+1]
  float* ws_ml;         // [max_items][8][2]
  float* ws_o;          // [max_items][8][hd]
  DeviceStatus* status;
  long max_items;
  int B, nq, nkv, G, window, chunk, mode;
  float scale_log2, softcap;
};

// Key range [lo, hi) of sequence b.
__device__ __forceinline__ void seq_range(const DecodeParams& p, int b, int& lo, int& hi) {
  if (p.mode == 0) {
    int ps = p.pos[b];
    hi = ps + 1;
    if (p.max_len) hi = min(hi, p.max_len[b]);
    lo = p.window > 0 ? max(0, ps - p.window + 1) : 0;
    if (hi < lo) hi = lo;
    if (lo < 0) lo = 0;
  } else {
    lo = max(0, p.kv_lo[b]);
    hi = max(lo, p.kv_hi[b]);
  }
}

// Prefix sum of item counts per sequence into pref[0..B] (smem), by warp 0.
__device__ void build_prefix(const DecodeParams& p, int* pref) {
  const int lane = threadIdx.x & 31;
  if (threadIdx.x >= 32) return;
  const int per = (p.B + 31) / 32;
  const int b0 = lane * per, b1 = min(p.B, b0 + per);
  int local = 0;
  for (int b = b0; b < b1; ++b) {
    int lo, hi;
    seq_range(p, b, lo, hi);
    local += ((hi - lo + p.chunk - 1) / p.chunk) * p.nkv;
  }
  int incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  int run = incl - local;
  for (int b = b0; b < b1; ++b) {
    pref[b] = run;
    int lo, hi;
    seq_range(p, b, lo, hi);
    run += ((hi - lo + p.chunk - 1) / p.chunk) * p.nkv;
  }
  if (lane == 31) pref[p.B] = incl;
}

// Iterator over this warp's (item, stage) sequence.
struct ItemIter {
  long item;       // flat item index
  int b, kvh;      // sequence, kv head
  int k0, khi;     // next key, end of the item's range
  int kstart;      // first key of the item
  bool whole;      // the item covers the sequence's whole range
  bool valid;
};

__device__ __forceinline__ void iter_load(const DecodeParams& p, const int* pref, long total,
                                          ItemIter& it) {
  it.valid = it.item < total;
  if (!it.valid) return;
  // upper_bound over pref[0..B] for the owning sequence
  int lo = 0, hi = p.B;  // pref[lo] <= item < pref[hi]
  while (hi - lo > 1) {
    int mid = (lo + hi) >> 1;
    if (pref[mid] <= it.item) lo = mid; else hi = mid;
  }
  const int b = lo;
  const int r = (int)(it.item - pref[b]);
  const int c = r / p.nkv;
  it.b = b;
  it.kvh = r - c * p.nkv;
  int slo, shi;
  seq_range(p, b, slo, shi);
  it.kstart = slo + c * p.chunk;
  it.k0 = it.kstart;
  it.khi = min(shi, it.kstart + p.chunk);
  it.whole = (slo == it.kstart) && (it.khi == shi);
}

// Issue one stage (16 K rows + 16 V rows) for iterator position `it`.
template <int HD>
__device__ __forceinline__ void issue_stage(const DecodeParams& p, const ItemIter& it,
                                            unsigned char* stage, uint64_t* bar, int lane) {
  constexpr int ROWB = HD * 2 + 16;
  if (lane == 0) mbar_arrive_expect_tx(bar, 2 * kKeys * HD * 2);
  __syncwarp();
  const int which = lane >> 4;        // 0: K row, 1: V row
  const int r = lane & 15;
  const int key = min(it.k0 + r, it.khi - 1);   // clamp: rows past the end repeat a valid row
  const __half* base = which ? p.V[it.b] : p.K[it.b];
  const __half* src = base + (long)key * p.nkv * HD + (long)it.kvh * HD;
  bulk_g2s(stage + (which * kKeys + r) * ROWB, src, HD * 2, bar);
}

template <int HD, int STAGES>
__global__ void __launch_bounds__(kWarps * 32)
decode_kernel(const DecodeParams p) {
  constexpr int ROWB = HD * 2 + 16;
  constexpr int STAGE_BYTES = 2 * kKeys * ROWB;
  constexpr int KT = HD / 16;   // 16-dim steps
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ __align__(8) uint64_t bars[kWarps][STAGES];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  unsigned char* ring = smem + warp * STAGES * STAGE_BYTES;
  int* pref = reinterpret_cast<int*>(smem + kWarps * STAGES * STAGE_BYTES);

  build_prefix(p, pref);
  if (lane == 0)
    for (int s = 0; s < STAGES; ++s) mbar_init(&bars[warp][s], 1);
  fence_mbar_init();
  __syncthreads();
  const long total = pref[p.B];
  if (blockIdx.x == 0)
    for (int i = threadIdx.x; i <= p.B; i += blockDim.x) p.ws_pref[i] = pref[i];

  const long stride = (long)gridDim.x * kWarps;
  ItemIter prod, cons;
  prod.item = (long)blockIdx.x * kWarps + warp;
  iter_load(p, pref, total, prod);
  cons = prod;

  // prologue: fill the ring
  int issued = 0;
#pragma unroll 1
  for (int s = 0; s < STAGES && prod.valid; ++s) {
    issue_stage<HD>(p, prod, ring + s * STAGE_BYTES, &bars[warp][s], lane);
    ++issued;
    prod.k0 += kKeys;
    if (prod.k0 >= prod.khi) { prod.item += stride; iter_load(p, pref, total, prod); }
  }

  const int g = lane >> 2;            // query column this lane feeds in B fragments
  const int qc = 2 * (lane & 3);      // first of the two query columns this lane accumulates
  uint32_t qf[KT][2];
  float oacc[KT][4];
  float m_run[2], l_run[2];
  int cur_item_loaded = -1;
  long consumed = 0;

#pragma unroll 1
  while (cons.valid) {
    if (cons.k0 == cons.kstart) {
      // new item: load the G query rows of this kv group as the B operand
      const float* qb = p.q + ((long)cons.b * p.nq + (long)cons.kvh * p.G) * HD;
#pragma unroll
      for (int kt = 0; kt < KT; ++kt) {
        const int d = kt * 16 + qc;
        float2 lo2 = make_float2(0.f, 0.f), hi2 = make_float2(0.f, 0.f);
        if (g < p.G) {
          lo2 = *reinterpret_cast<const float2*>(qb + g * HD + d);
          hi2 = *reinterpret_cast<const float2*>(qb + g * HD + d + 8);
        }
        qf[kt][0] = pack_half2(lo2.x, lo2.y);
        qf[kt][1] = pack_half2(hi2.x, hi2.y);
#pragma unroll
        for (int j = 0; j < 4; ++j) oacc[kt][j] = 0.f;
      }
      m_run[0] = m_run[1] = -INFINITY;
      l_run[0] = l_run[1] = 0.f;
      cur_item_loaded = 1;
    }
    const int slot = (int)(consumed % STAGES);
    const uint32_t parity = (uint32_t)((consumed / STAGES) & 1);
    if (!mbar_wait_bounded(&bars[warp][slot], parity)) {
      if (lane == 0 && p.status) { atomicExch(&p.status->code, kDevTimeoutMbar); p.status->where = 1; }
      // drain the copies this warp still has in flight (bounded), then leave
      for (long c = consumed + 1; c < (long)issued; ++c)
        mbar_wait_bounded(&bars[warp][c % STAGES], (uint32_t)((c / STAGES) & 1));
      return;
    }
    unsigned char* st = ring + slot * STAGE_BYTES;
    const uint32_t kbase = smem_u32(st), vbase = smem_u32(st + kKeys * ROWB);

    // S^T = K Q^T for 16 keys x 8 query columns
    float s4[4] = {0.f, 0.f, 0.f, 0.f};
    {
      const int krow = (lane & 7) + ((lane >> 3) & 1) * 8;
      const int kcol = (lane >> 4) * 8;
#pragma unroll
      for (int kt = 0; kt < KT; ++kt) {
        uint32_t a[4];
        ldmatrix_x4(a[0], a[1], a[2], a[3], kbase + krow * ROWB + (kt * 16 + kcol) * 2);
        mma_16816(s4, a, qf[kt][0], qf[kt][1]);
      }
    }
    // scale (+ softcap), mask keys past the item's end
    const int key_a = cons.k0 + g, key_b = cons.k0 + g + 8;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float x = s4[j];
      if (p.softcap > 0.f) x = p.softcap * tanhf(x * (p.scale_log2 / kLog2e) / p.softcap) * kLog2e;
      else x *= p.scale_log2;
      const int key = (j < 2) ? key_a : key_b;
      s4[j] = key < cons.khi ? x : -INFINITY;
    }
    // online softmax per query column (q0 = qc, q1 = qc + 1)
    float mx0 = fmaxf(s4[0], s4[2]), mx1 = fmaxf(s4[1], s4[3]);
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
    }
    const float mn0 = fmaxf(m_run[0], mx0), mn1 = fmaxf(m_run[1], mx1);
    const float c0 = fast_exp2(m_run[0] - mn0), c1 = fast_exp2(m_run[1] - mn1);
    m_run[0] = mn0;
    m_run[1] = mn1;
    const float p0 = fast_exp2(s4[0] - mn0), p1 = fast_exp2(s4[1] - mn1);
    const float p2 = fast_exp2(s4[2] - mn0), p3 = fast_exp2(s4[3] - mn1);
    l_run[0] = l_run[0] * c0 + (p0 + p2);
    l_run[1] = l_run[1] * c1 + (p1 + p3);
#pragma unroll
    for (int kt = 0; kt < KT; ++kt) {
      oacc[kt][0] *= c0; oacc[kt][1] *= c1;
      oacc[kt][2] *= c0; oacc[kt][3] *= c1;
    }
    // P^T operand via in-register transpose, then O^T += V^T P^T
    const uint32_t b0 = movmatrix_trans(pack_half2(p0, p1));
    const uint32_t b1 = movmatrix_trans(pack_half2(p2, p3));
    {
      const int vrow = (lane & 7) + (lane >> 4) * 8;
      const int vcol = ((lane >> 3) & 1) * 8;
#pragma unroll
      for (int mt = 0; mt < KT; ++mt) {
        uint32_t a[4];
        ldmatrix_x4_trans(a[0], a[1], a[2], a[3], vbase + vrow * ROWB + (mt * 16 + vcol) * 2);
        mma_16816(oacc[mt], a, b0, b1);
      }
    }
    __syncwarp();
    ++consumed;

    // refill the freed slot
    if (prod.valid) {
      fence_proxy_async_smem();
      issue_stage<HD>(p, prod, st, &bars[warp][slot], lane);
      ++issued;
      prod.k0 += kKeys;
      if (prod.k0 >= prod.khi) { prod.item += stride; iter_load(p, pref, total, prod); }
    }

    cons.k0 += kKeys;
    if (cons.k0 >= cons.khi) {
      // item done: reduce l across the lanes that share a query column
      float l0 = l_run[0], l1 = l_run[1];
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {
        l0 += __shfl_xor_sync(0xffffffffu, l0, o);
        l1 += __shfl_xor_sync(0xffffffffu, l1, o);
      }
      const int h0 = cons.kvh * p.G + qc;  // head of column qc
      if (cons.whole && p.mode == 0) {
        const float inv0 = 1.f / l0, inv1 = 1.f / l1;
        float* ob = p.out + (long)cons.b * p.nq * HD;
        const float* gb = p.gate ? p.gate + (long)cons.b * p.nq * HD : nullptr;
#pragma unroll
        for (int mt = 0; mt < KT; ++mt) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int qq = qc + (j & 1);
            if (qq >= p.G) continue;
            const int dim = mt * 16 + g + (j >> 1) * 8;
            const long idx = (long)(h0 + (j & 1)) * HD + dim;
            float v = oacc[mt][j] * ((j & 1) ? inv1 : inv0);
            if (gb) v *= 1.f / (1.f + expf(-gb[idx]));
            ob[idx] = v;
          }
        }
      } else if (cons.item < p.max_items) {
        float* wo = p.ws_o + cons.item * 8 * HD;
        float* wml = p.ws_ml + cons.item * 16;
#pragma unroll
        for (int mt = 0; mt < KT; ++mt) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int qq = qc + (j & 1);
            const int dim = mt * 16 + g + (j >> 1) * 8;
            wo[qq * HD + dim] = oacc[mt][j];
          }
        }
        if (g == 0) {
          wml[qc * 2 + 0] = m_run[0];
          wml[qc * 2 + 1] = l0;
          wml[(qc + 1) * 2 + 0] = m_run[1];
          wml[(qc + 1) * 2 + 1] = l1;
        }
      } else if (lane == 0 && p.status) {
        atomicExch(&p.status->code, 2);  // workspace too small for the real lengths
        p.status->where = 2;
      }
      cons.item += stride;
      iter_load(p, pref, total, cons);
    }
  }
  (void)cur_item_loaded;
}

// Merge the per-chunk partials of each (sequence, kv head): one CTA per
// (b, kvh), one thread per dim, looping the G heads of the group.
template <int HD>
__global__ void combine_kernel(const DecodeParams p) {
  const int b = blockIdx.x, kvh = blockIdx.y, d = threadIdx.x;
  const int base = p.ws_pref[b];
  const int nch = (p.ws_pref[b + 1] - base) / p.nkv;
  if (p.mode == 0 && nch == 1) return;  // written directly by the decode kernel
  for (int gq = 0; gq < p.G; ++gq) {
    const int h = kvh * p.G + gq;
    float M = -INFINITY;
    for (int c = 0; c < nch; ++c) {
      const long it = base + (long)c * p.nkv + kvh;
      if (it < p.max_items) M = fmaxf(M, p.ws_ml[it * 16 + gq * 2]);
    }
    float acc = 0.f, L = 0.f;
    for (int c = 0; c < nch; ++c) {
      const long it = base + (long)c * p.nkv + kvh;
      if (it >= p.max_items) continue;
      const float w = fast_exp2(p.ws_ml[it * 16 + gq * 2] - M);
      L += w * p.ws_ml[it * 16 + gq * 2 + 1];
      acc += w * p.ws_o[it * 8 * HD + gq * HD + d];
    }
    const long oi = ((long)b * p.nq + h) * HD + d;
    if (p.mode == 0) {
      float v = L > 0.f ? acc / L : 0.f;
      if (p.gate) v *= 1.f / (1.f + expf(-p.gate[oi]));
      p.out[oi] = v;
    } else {
      p.part_o[oi] = nch > 0 ? acc : 0.f;
      if (d == 0) {
        p.part_m[(long)b * p.nq + h] = nch > 0 ? M * kLn2 : kNegBig;
        p.part_l[(long)b * p.nq + h] = nch > 0 ? L : 0.f;
      }
    }
  }
}

template <int HD> constexpr int stages_for() { return HD == 64 ? 6 : 3; }

template <int HD>
size_t ring_bytes() { return (size_t)kWarps * stages_for<HD>() * 2 * kKeys * (HD * 2 + 16); }

int auto_chunk(int B, int nkv, int max_kv_len) {
  // Aim for about 4 items per resident warp, 256..4096 keys per item.
  const long warps = (long)num_sms() * 2 * kWarps;
  long keys = (long)B * nkv * std::max(1, max_kv_len);
  long c = keys / (4 * warps);
  c = std::max(256L, std::min(4096L, c));
  return (int)((c + 63) / 64 * 64);
}

struct WsLayout { size_t pref, ml, o, total; long max_items; };

WsLayout ws_layout(int B, int nkv, int hd, int max_kv_len, int chunk) {
  WsLayout w;
  long nch = (std::max(1, max_kv_len) + chunk - 1) / chunk;
  w.max_items = (long)B * nkv * nch;
  auto al = [](size_t x) { return (x + 255) / 256 * 256; };
  w.pref = 0;
  w.ml = al((size_t)(B + 1) * sizeof(int));
  w.o = w.ml + al((size_t)w.max_items * 16 * sizeof(float));
  w.total = w.o + al((size_t)w.max_items * 8 * hd * sizeof(float));
  return w;
}

template <int HD>
int launch_decode_hd(DecodeParams& p, cudaStream_t st) {
  constexpr int S = stages_for<HD>();
  const size_t smem = ring_bytes<HD>() + (size_t)(p.B + 1) * sizeof(int);
  auto kern = decode_kernel<HD, S>;
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)(ring_bytes<HD>() + (kMaxB + 1) * sizeof(int)));
    if (e != cudaSuccess) return record_status((int)e);
    configured[dev] = 1;
  }
  int occ = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kWarps * 32, smem);
  if (occ < 1) occ = 1;
  int grid = num_sms() * occ;
  kern<<<grid, kWarps * 32, smem, st>>>(p);
  ASPIDA_CHECK_LAUNCH();
  combine_kernel<HD><<<dim3(p.B, p.nkv), HD, 0, st>>>(p);
  ASPIDA_CHECK_LAUNCH();
  return 0;
}

int run_decode(DecodeParams& p, int hd, int max_kv_len, int chunk, void* ws, size_t ws_bytes,
               cudaStream_t st) {
  if (p.B <= 0) return 0;
  if (p.B > kMaxB || p.nq <= 0 || p.nkv <= 0 || p.nq % p.nkv != 0 || !p.q || !p.K || !p.V)
    return record_status(ASPIDA_ERR_ARG);
  if (p.G > 8 || (hd != 64 && hd != 128 && hd != 256)) return record_status(ASPIDA_ERR_UNSUPPORTED);
  if (chunk <= 0) chunk = auto_chunk(p.B, p.nkv, max_kv_len);
  if (chunk % 64 != 0) return record_status(ASPIDA_ERR_ARG);
  WsLayout w = ws_layout(p.B, p.nkv, hd, max_kv_len, chunk);
  if (!ws || ws_bytes < w.total) return record_status(ASPIDA_ERR_WORKSPACE);
  if (((uintptr_t)ws & 255) != 0) return record_status(ASPIDA_ERR_ARG);
  unsigned char* wb = static_cast<unsigned char*>(ws);
  p.ws_pref = reinterpret_cast<int*>(wb + w.pref);
  p.ws_ml = reinterpret_cast<float*>(wb + w.ml);
  p.ws_o = reinterpret_cast<float*>(wb + w.o);
  p.max_items = w.max_items;
  p.chunk = chunk;
  p.status = device_status_ptr();
  switch (hd) {
    case 64: return launch_decode_hd<64>(p, st);
    case 128: return launch_decode_hd<128>(p, st);
    default: return launch_decode_hd<256>(p, st);
  }
}

}  // namespace

size_t decode_workspace_size(int B, int nq, int nkv, int hd, int max_kv_len, int chunk) {
  (void)nq;
  if (B <= 0 || nkv <= 0) return 0;
  if (chunk <= 0) chunk = auto_chunk(B, nkv, max_kv_len);
  return ws_layout(B, nkv, hd, max_kv_len, chunk).total;
}

int decode(const float* q, const float* gate, const void* const* K, const void* const* V,
           const int* pos, const int* max_len, float* out, int B, int nq, int nkv, int hd,
           float scale, int window, float softcap, int max_kv_len, int chunk, void* ws,
           size_t ws_bytes, cudaStream_t st) {
  DecodeParams p{};
  p.q = q; p.gate = gate;
  p.K = reinterpret_cast<const __half* const*>(K);
  p.V = reinterpret_cast<const __half* const*>(V);
  p.pos = pos; p.max_len = max_len; p.out = out;
  p.B = B; p.nq = nq; p.nkv = nkv; p.G = nkv > 0 ? nq / nkv : 0;
  p.window = window; p.mode = 0;
  p.scale_log2 = scale * kLog2e; p.softcap = softcap;
  if (!pos || !out) return record_status(ASPIDA_ERR_ARG);
  return run_decode(p, hd, max_kv_len, chunk, ws, ws_bytes, st);
}

int decode_partial(const float* q, const void* const* K, const void* const* V, const int* kv_lo,
                   const int* kv_hi, float* m, float* l, float* o, int B, int nq, int nkv, int hd,
                   float scale, float softcap, int max_kv_len, int chunk, void* ws,
                   size_t ws_bytes, cudaStream_t st) {
  DecodeParams p{};
  p.q = q;
  p.K = reinterpret_cast<const __half* const*>(K);
  p.V = reinterpret_cast<const __half* const*>(V);
  p.kv_lo = kv_lo; p.kv_hi = kv_hi;
  p.part_m = m; p.part_l = l; p.part_o = o;
  p.B = B; p.nq = nq; p.nkv = nkv; p.G = nkv > 0 ? nq / nkv : 0;
  p.window = 0; p.mode = 1;
  p.scale_log2 = scale * kLog2e; p.softcap = softcap;
  if (!kv_lo || !kv_hi || !m || !l || !o) return record_status(ASPIDA_ERR_ARG);
  return run_decode(p, hd, max_kv_len, chunk, ws, ws_bytes, st);
}

}  // namespace aspida

extern "C" size_t aspida_attn_decode_workspace_size(int B, int nq, int nkv, int hd,
                                                    int max_kv_len, int chunk) {
  return aspida::decode_workspace_size(B, nq, nkv, hd, max_kv_len, chunk);
}

extern "C" int aspida_attn_decode(const float* q, const float* gate, const void* const* K,
                                  const void* const* V, const int* pos, const int* max_len,
                                  float* out, int B, int nq, int nkv, int hd, float scale,
                                  int window, float softcap, int max_kv_len, int chunk,
                                  void* workspace, size_t workspace_bytes, void* stream) {
  return aspida::decode(q, gate, K, V, pos, max_len, out, B, nq, nkv, hd, scale, window, softcap,
                        max_kv_len, chunk, workspace, workspace_bytes, (cudaStream_t)stream);
}

extern "C" int aspida_attn_decode_partial(const float* q, const void* const* K,
                                          const void* const* V, const int* kv_lo,
                                          const int* kv_hi, float* m, float* l, float* o, int B,
                                          int nq, int nkv, int hd, float scale, float softcap,
                                          int max_kv_len, int chunk, void* workspace,
                                          size_t workspace_bytes, void* stream) {
  return aspida::decode_partial(q, K, V, kv_lo, kv_hi, m, l, o, B, nq, nkv, hd, scale, softcap,
                                max_kv_len, chunk, workspace, workspace_bytes,
                                (cudaStream_t)stream);
}
