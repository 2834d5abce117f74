// prefill.cu — causal (optionally sliding-window, softcapped, gated) GQA
// prefill attention on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// Replaces the shim's prefill attention, aspida_ggml_fattn_prefill
// (gpu/fattn_ggml.cuh:109-141, ggml fattn-mma) and its unused own variants
// k_fattn_attend_tile / k_fattn_tile_gqa / k_fattn_wmma[3]
// (gpu/gpu_matvec.cu:3309-3682). Semantics: P queries at positions
// pos_start..pos_start+P-1 attend keys max(0, pos-window+1)..pos of the fp16
// cache; out = softmax(scale * q k^T [softcapped]) v [x sigmoid(gate)].
//
// One CTA computes one 128-row query tile of one query head:
//   warp 0      TMA producer: the Q tile once, then K and V tiles of BN keys
//               (2D tensor maps, 128-byte swizzle, double-buffered stages).
//   warp 1      owns TMEM (alloc/dealloc); one elected lane issues the MMAs:
//               S_j = Q K_j^T (A, B from shared memory, K-major) into one of
//               two S buffers, then O += P_{j-1} V_{j-1} with P read from TMEM
//               (the A operand) and V from shared memory (MN-major).
//   warps 4-7   softmax: thread r owns query row r (TMEM lane r). It loads
//               S_j, masks (causal / window / length), computes the online
//               softmax in the log2 domain, writes P_j as fp16 back into the
//               S_j columns, and rescales O by exp2(m_old - m_new) once
//               PV_{j-1} has landed (skipped when no row of the warp grew).
//               The epilogue reads O, divides by l and stores the row.
// TMEM columns: S0 [0, BN), S1 [BN, 2BN), O [256, 256 + HD); 512 allocated.
//
// Every mbarrier wait is bounded; a wait that runs out sets the device
// status word and the CTA unwinds (TMEM is freed on every path).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <mutex>

#include "common.cuh"
#include "tcgen05.cuh"

namespace aspida {
namespace {

constexpr int BM = 128;
constexpr int kMaxSeq = 8;            // sequences per launch
constexpr int kThreads = 256;
constexpr float kLog2e = 1.4426950408889634f;

#ifdef ASPIDA_TRACE
// Opt-in timeline (debug builds only): per CTA (first 4), event x tile, clock64.
__device__ long long g_trace[4][16][64];
#define TRACE(ev, j) do { if (blockIdx.x + blockIdx.y * gridDim.x + blockIdx.z == 0 || \
    (blockIdx.y == 0 && blockIdx.z == 0 && blockIdx.x < 4)) \
    if ((j) < 64) g_trace[blockIdx.x & 3][ev][j] = clock64(); } while (0)
#else
#define TRACE(ev, j) do {} while (0)
#endif

struct PrefillParams {
  CUtensorMap qmap[kMaxSeq];
  CUtensorMap kmap[kMaxSeq];
  CUtensorMap vmap[kMaxSeq];
  CUtensorMap omap[kMaxSeq];        // fp16 output (TMA-store epilogue); unused for f32 out
  void* out[kMaxSeq];
  const float* gate[kMaxSeq];
  int P[kMaxSeq];
  int pos_start[kMaxSeq];
  DeviceStatus* status;
  int nq, nkv, G, window, out_f32, ntq;
  float scale_log2, softcap;
};

template <int HD>
struct PGeo {
  static constexpr int BN = HD <= 128 ? 128 : 64;     // keys per KV tile
  static constexpr int CH = HD / 64;                  // 64-column (128-byte) chunks
  static constexpr int Q_BYTES = BM * HD * 2;
  static constexpr int KV_BYTES = BN * HD * 2;        // one K (or V) tile
  static constexpr int NS = 2;                        // K/V stages
  static constexpr int SMEM_USED = Q_BYTES + 2 * NS * KV_BYTES;
  // at least ~116 KB so only one CTA (and one 512-column TMEM allocation) fits per SM
  static constexpr int SMEM = (SMEM_USED > 118 * 1024 ? SMEM_USED : 118 * 1024) + 1024;
  static constexpr uint32_t O_COL = 256;
  static constexpr uint32_t TMEM_COLS = 512;
};

struct Sync {
  uint64_t q_full;
  uint64_t k_full[2], v_full[2], k_empty[2], v_empty[2];
  uint64_t s_full[2], p_ready[2];
  uint64_t o_done, o_final;
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, Sync& sy,
                                              const PrefillParams& p, int where) {
  if (sy.abort) return false;
  if (mbar_wait_bounded(bar, parity)) return true;
  sy.abort = 1;
  if (p.status) {
    atomicExch(&p.status->code, kDevTimeoutMbar);
    p.status->where = where;
  }
  return false;
}

// Scores in the log2 domain: s*scale*log2e, or softcap*tanh(s*scale/softcap)
// *log2e. The branch is taken once per 32-column chunk, outside the element
// loop, so the uncapped path carries no tanh.
__device__ __forceinline__ void scores_log2(float* x, bool capped, float cap, float scale_log2) {
  if (capped) {
    const float sc = scale_log2 / kLog2e / cap;
#pragma unroll
    for (int i = 0; i < 32; ++i) x[i] = cap * tanhf(x[i] * sc) * kLog2e;
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) x[i] *= scale_log2;
  }
}

// Packed f32x2 arithmetic (sm_100): two lanes of fp32 per instruction.
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1,%2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float2 f2_unpack(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0,%1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// 2^x for a pair on the FMA/ALU pipes, to offload the MUFU unit (two softmax
// warps per SM sub-partition would otherwise saturate it). x = n + f with n
// = round(x) taken from the bits of x + 1.5*2^23, f in [-0.5, 0.5]; 2^f by a
// cubic fitted here by least squares on the relative error (max 7.7e-5,
// below fp16's half-ulp, so the fp16 P is unchanged); 2^n is added to the
// exponent bits. x is clamped at -125 (the result then rounds to 0 in fp16).
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
  constexpr float kMagic = 12582912.f;                 // 1.5 * 2^23
  const uint64_t a = f2_pack(fmaxf(x.x, -125.f), fmaxf(x.y, -125.f));
  const uint64_t t = f2_add(a, f2_pack(kMagic, kMagic));          // n in the low bits
  const uint64_t f = f2_add(a, f2_add(t, f2_pack(-kMagic, -kMagic)) ^ 0x8000000080000000ull);
  uint64_t q = f2_fma(f2_pack(0.05508872f, 0.05508872f), f, f2_pack(0.24260436f, 0.24260436f));
  q = f2_fma(q, f, f2_pack(0.69327629f, 0.69327629f));
  q = f2_fma(q, f, f2_pack(0.99992895f, 0.99992895f));
  const float2 r = f2_unpack(q), tn = f2_unpack(t);
  return make_float2(__int_as_float(__float_as_int(r.x) + (__float_as_int(tn.x) << 23)),
                     __int_as_float(__float_as_int(r.y) + (__float_as_int(tn.y) << 23)));
}

// max(a, b, c) in one instruction (sm_100 three-input max).
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Max of 128 values as a shallow tree of three-input maxes (independent
// partial maxima instead of one 128-long dependent chain).
__device__ __forceinline__ float rowmax128(const float* s) {
  float m[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) m[k] = max3(s[k], s[8 + k], s[16 + k]);
#pragma unroll
  for (int i = 24; i + 16 <= 128; i += 16) {
#pragma unroll
    for (int k = 0; k < 8; ++k) m[k] = max3(m[k], s[i + k], s[i + 8 + k]);
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) m[k] = fmaxf(m[k], s[120 + k]);
  return fmaxf(max3(m[0], m[1], m[2]), max3(max3(m[3], m[4], m[5]), m[6], m[7]));
}

// -inf outside keys max(0, qpos-window+1)..qpos and beyond the length.
__device__ __forceinline__ void mask_chunk(float* x, int key0, int qpos, int win_lo, int len) {
  const int hi = min(qpos, len - 1);
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const int key = key0 + i;
    x[i] = (key <= hi && key >= win_lo) ? x[i] : -INFINITY;
  }
}

template <int HD>
__global__ void __launch_bounds__(kThreads, 1)
prefill_kernel(const __grid_constant__ PrefillParams p) {
  using Geo = PGeo<HD>;
  constexpr int BN = Geo::BN, CH = Geo::CH, NS = Geo::NS;
  extern __shared__ unsigned char smem_raw[];
  __shared__ Sync sy;

  const int seq = blockIdx.z, h = blockIdx.y;
  const int qt = p.ntq - 1 - (int)blockIdx.x;      // heaviest (latest) tiles first
  const int P = p.P[seq], ps = p.pos_start[seq];
  if (qt * BM >= P) return;
  const int kvh = h / p.G;
  const int len = ps + P;
  const int q_first = ps + qt * BM;
  const int q_last = min(ps + P, q_first + BM) - 1;
  const int kv_lo = p.window > 0 ? max(0, q_first - p.window + 1) : 0;
  const int t0 = kv_lo / BN;
  const int n = q_last / BN - t0 + 1;                 // KV tiles

  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* Qs = smem;
  unsigned char* Ks = smem + Geo::Q_BYTES;
  unsigned char* Vs = Ks + NS * Geo::KV_BYTES;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(&sy.q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sy.k_full[s], 1);
      mbar_init(&sy.v_full[s], 1);
      mbar_init(&sy.k_empty[s], 1);
      mbar_init(&sy.v_empty[s], 1);
      mbar_init(&sy.s_full[s], 1);
      mbar_init(&sy.p_ready[s], 128);
    }
    mbar_init(&sy.o_done, 1);
    mbar_init(&sy.o_final, 1);
    sy.abort = 0;
  }
  if (warp == 1) {
    tc::tmem_alloc(&sy.tmem_base, Geo::TMEM_COLS);
    tc::tmem_relinquish();
  }
  fence_mbar_init();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = sy.tmem_base;

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (tc::elect_one()) {
      mbar_arrive_expect_tx(&sy.q_full, Geo::Q_BYTES);
      for (int c = 0; c < CH; ++c)
        tc::tma_load_2d(Qs + c * BM * 128, &p.qmap[seq], h * HD + c * 64, qt * BM, &sy.q_full);
      for (int j = 0; j < n; ++j) {
        const int s = j % NS;
        const int row = (t0 + j) * BN;
        if (j >= NS && !wait_or_abort(&sy.k_empty[s], ((j / NS) - 1) & 1, sy, p, 20)) break;
        TRACE(0, j);
        mbar_arrive_expect_tx(&sy.k_full[s], Geo::KV_BYTES);
        for (int c = 0; c < CH; ++c)
          tc::tma_load_2d(Ks + s * Geo::KV_BYTES + c * BN * 128, &p.kmap[seq], kvh * HD + c * 64,
                          row, &sy.k_full[s]);
        if (j >= NS && !wait_or_abort(&sy.v_empty[s], ((j / NS) - 1) & 1, sy, p, 21)) break;
        mbar_arrive_expect_tx(&sy.v_full[s], Geo::KV_BYTES);
        for (int c = 0; c < CH; ++c)
          tc::tma_load_2d(Vs + s * Geo::KV_BYTES + c * BN * 128, &p.vmap[seq], kvh * HD + c * 64,
                          row, &sy.v_full[s]);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------ MMA issuer --------------------------------
    if (tc::elect_one()) {
      constexpr uint32_t idS = tc::idesc_f16_f32(BM, BN, false, false);
      constexpr uint32_t idO = tc::idesc_f16_f32(BM, HD, false, true);
      const uint32_t qbase = smem_u32(Qs), kbase = smem_u32(Ks), vbase = smem_u32(Vs);
      bool ok = wait_or_abort(&sy.q_full, 0, sy, p, 30);
      tc::fence_after_sync();
      for (int j = 0; ok && j <= n; ++j) {
        if (j < n) {
          const int s = j % NS;
          if (!wait_or_abort(&sy.k_full[s], (j / NS) & 1, sy, p, 31)) break;
          TRACE(1, j);
          tc::fence_after_sync();
          const uint32_t sb = tmem + (uint32_t)((j & 1) * BN);
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk) {
            const int c = kk >> 2;
            const uint64_t a = tc::smem_desc_sw128(qbase + c * BM * 128 + (kk & 3) * 32, 16, 1024);
            const uint64_t b = tc::smem_desc_sw128(
                kbase + s * Geo::KV_BYTES + c * BN * 128 + (kk & 3) * 32, 16, 1024);
            tc::mma_ss(sb, a, b, idS, kk > 0);
          }
          tc::commit(&sy.s_full[j & 1]);
          tc::commit(&sy.k_empty[s]);
        }
        if (j >= 1) {
          const int jj = j - 1, s = jj % NS;
          if (!wait_or_abort(&sy.p_ready[jj & 1], (jj >> 1) & 1, sy, p, 32)) break;
          TRACE(2, jj);
          if (!wait_or_abort(&sy.v_full[s], (jj / NS) & 1, sy, p, 33)) break;
          TRACE(3, jj);
          tc::fence_after_sync();
          const uint32_t pb = tmem + (uint32_t)((jj & 1) * BN);
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk) {
            const uint64_t b = tc::smem_desc_sw128(vbase + s * Geo::KV_BYTES + kk * 16 * 128,
                                                   BN * 128, 1024);
            tc::mma_ts(tmem + Geo::O_COL, pb + kk * 8, b, idO, (jj > 0 || kk > 0) ? 1u : 0u);
          }
          tc::commit(&sy.v_empty[s]);
          tc::commit(&sy.o_done);
        }
      }
      tc::commit(&sy.o_final);   // fires once every MMA issued above has completed
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ------------------------------ softmax / epilogue ------------------------
    const int wq = warp & 3;
    const int r = wq * 32 + lane;                    // query row == TMEM lane
    const uint32_t lane_addr = (uint32_t)(wq * 32) << 16;
    const int qpos = q_first + r;
    const int win_lo = p.window > 0 ? qpos - p.window + 1 : 0;
    const bool capped = p.softcap > 0.f;
    float m_run = -INFINITY, l_run = 0.f;
    for (int j = 0; j < n; ++j) {
      if (!wait_or_abort(&sy.s_full[j & 1], (j >> 1) & 1, sy, p, 40)) break;
      if (r == 0) TRACE(4, j);
      tc::fence_after_sync();
      const uint32_t sb = tmem + lane_addr + (uint32_t)((j & 1) * BN);
      const int key0 = (t0 + j) * BN;
      // rows whose tile lies wholly inside their causal / window / length
      // range skip the per-element mask
      const bool masked = !(key0 + BN - 1 <= qpos && key0 >= win_lo && key0 + BN <= len);
      // pass 1: scaled (softcapped) scores, row max
      float mx = -INFINITY;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        float x[32];
        tc::tmem_ld32(sb + c * 32, x);
        tc::tmem_wait_ld();
        scores_log2(x, capped, p.softcap, p.scale_log2);
        if (masked) mask_chunk(x, key0 + c * 32, qpos, win_lo, len);
#pragma unroll
        for (int i = 0; i < 32; ++i) mx = fmaxf(mx, x[i]);
      }
      const float m_new = fmaxf(m_run, mx);
      const float m_use = m_new == -INFINITY ? 0.f : m_new;
      const float corr = fast_exp2(m_run - m_use);
      // pass 2: P = exp2(s - m) as fp16 pairs into the first BN/2 columns
      float sum = 0.f;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        float x[32];
        tc::tmem_ld32(sb + c * 32, x);
        tc::tmem_wait_ld();
        scores_log2(x, capped, p.softcap, p.scale_log2);
        if (masked) mask_chunk(x, key0 + c * 32, qpos, win_lo, len);
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float e0 = fast_exp2(x[2 * i] - m_use), e1 = fast_exp2(x[2 * i + 1] - m_use);
          sum += e0 + e1;
          pk[i] = pack_half2(e0, e1);
        }
        // P columns c*16.. overwrite S columns already read (<= c*32+31)
        tc::tmem_st16(sb + c * 16, pk);
      }
      l_run = l_run * corr + sum;
      m_run = m_new;
      if (r == 0) TRACE(5, j);
      if (j >= 1) {
        // O holds tiles < j at the previous max: rescale once PV_{j-1} landed
        if (!wait_or_abort(&sy.o_done, (j - 1) & 1, sy, p, 41)) break;
        if (r == 0) TRACE(6, j);
        tc::fence_after_sync();
        if (__any_sync(0xffffffffu, corr != 1.f)) {
          const uint32_t ob = tmem + lane_addr + Geo::O_COL;
#pragma unroll 1
          for (int c = 0; c < HD / 32; ++c) {
            float o[32];
            tc::tmem_ld32(ob + c * 32, o);
            tc::tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= corr;
            tc::tmem_st32(ob + c * 32, reinterpret_cast<const uint32_t*>(o));
          }
        }
      }
      tc::tmem_wait_st();
      tc::fence_before_sync();
      mbar_arrive(&sy.p_ready[j & 1]);
      if (r == 0) TRACE(7, j);
    }
    if (wait_or_abort(&sy.o_final, 0, sy, p, 42)) {
      tc::fence_after_sync();
      const int row = qt * BM + r;
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      const long obase = ((long)row * p.nq + h) * HD;
      const float* g = p.gate[seq];
      const uint32_t ob = tmem + lane_addr + Geo::O_COL;
#pragma unroll 1
      for (int c = 0; c < HD / 32; ++c) {
        float o[32];
        tc::tmem_ld32(ob + c * 32, o);
        tc::tmem_wait_ld();
        if (row < P) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            o[i] *= inv;
            if (g) o[i] *= 1.f / (1.f + expf(-g[obase + c * 32 + i]));
          }
          if (p.out_f32) {
            float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.out[seq]) + obase + c * 32);
#pragma unroll
            for (int i = 0; i < 8; ++i) dst[i] = make_float4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
          } else {
            uint4* dst = reinterpret_cast<uint4*>(static_cast<__half*>(p.out[seq]) + obase + c * 32);
#pragma unroll
            for (int i = 0; i < 4; ++i)
              dst[i] = make_uint4(pack_half2(o[8 * i], o[8 * i + 1]), pack_half2(o[8 * i + 2], o[8 * i + 3]),
                                  pack_half2(o[8 * i + 4], o[8 * i + 5]), pack_half2(o[8 * i + 6], o[8 * i + 7]));
          }
        }
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, Geo::TMEM_COLS);
  }
}


// ---------------------------------------------------------------------------
// Persistent two-query-tile kernel (hd <= 128). A work item is (sequence,
// head, 256-row tile); items are ordered heaviest first and dealt to one CTA
// per SM round-robin. Within an item, query tiles A = rows [256*qt, +128) and
// B = [256*qt + 128, +128) share every K/V tile; two softmax warpgroups
// (warps 2-5 for A, 6-9 for B) ping-pong against the MMA issuer, so one
// tile's softmax overlaps the other tile's PV and next S.
// TMEM: S_A [0,128), S_B [128,256), O_A [256,384), O_B [384,512).
// Across items: K/V keep streaming; each query tile's epilogue stages its fp16
// output in that tile's Q buffer (idle once O is final) and writes it with a
// TMA tensor store, then hands the buffer back (q_free) for the next item's
// Q; O_X is handed back through o_full / o_free.
// MMAs from one thread complete in issue order, so the commit that signals
// S_X(j) also certifies PV_X(j-1): the softmax may rescale O_X right after
// S_X(j) lands. O is only rescaled when some row's max grew by more than
// 2^8 (log2 domain 8): otherwise the stale max is kept, P <= 2^8 fits fp16,
// and the final 1/l uses the same max.
// ---------------------------------------------------------------------------
constexpr int kThreads2 = 576;   // producer, MMA, 2 x 8 softmax warps
constexpr float kRescaleThreshold = 8.f;

template <int HD>
struct PGeo2 {
  static constexpr int BN = 128;
  static constexpr int CH = HD / 64;
  static constexpr int QT_BYTES = BM * HD * 2;         // one 128-row Q tile
  static constexpr int KV_BYTES = BN * HD * 2;
  static constexpr int NS = 2;
  static constexpr int SMEM_USED = 2 * QT_BYTES + 2 * NS * KV_BYTES;
  static constexpr int SMEM = (SMEM_USED > 118 * 1024 ? SMEM_USED : 118 * 1024) + 1024;
};

struct Sync2 {
  uint64_t q_full, q_free[2];       // Q buffer of tile X released after its epilogue
  uint64_t k_full[2], v_full[2], k_empty[2], v_empty[2];
  uint64_t s_full[2], p_ready[2];   // per query tile
  uint64_t o_full[2], o_free[2];    // per query tile
  uint64_t drain;
  float xmax[2][2][2][128];         // [tile parity][query tile][column half][row]
  float xsum[2][2][128];            // [query tile][column half][row] for the epilogue
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ bool wait2(uint64_t* bar, uint32_t parity, Sync2& sy,
                                      const PrefillParams& p, int where) {
  if (sy.abort) return false;
  if (mbar_wait_bounded(bar, parity)) return true;
  sy.abort = 1;
  if (p.status) {
    atomicExch(&p.status->code, kDevTimeoutMbar);
    p.status->where = where;
  }
  return false;
}

// Geometry of one work item; identical in every role.
struct Item {
  int seq, h, qt, P, len, kvh;
  int qf[2], x0[2], x1[2];   // first position, active KV tiles [x0, x1) per query tile
  int t0, n;                 // union of KV tiles
  bool valid;
};

template <int BN>
__device__ __forceinline__ Item make_item(const PrefillParams& p, int nseq, int w) {
  Item it;
  const int per = nseq * p.nq;
  it.qt = p.ntq - 1 - w / per;
  const int rem = w % per;
  it.seq = rem / p.nq;
  it.h = rem % p.nq;
  int P = 0, ps = 0;
#pragma unroll
  for (int s = 0; s < kMaxSeq; ++s)      // compile-time indices: no local copy of the params
    if (s == it.seq) { P = p.P[s]; ps = p.pos_start[s]; }
  it.P = P;
  it.len = ps + it.P;
  it.kvh = it.h / p.G;
  it.valid = it.qt * 2 * BM < it.P;
  for (int X = 0; X < 2; ++X) {
    const int r0 = it.qt * 2 * BM + X * BM;
    it.qf[X] = ps + r0;
    if (r0 >= it.P) { it.x0[X] = it.x1[X] = 0; continue; }
    const int ql = min(ps + it.P, it.qf[X] + BM) - 1;
    const int lo = p.window > 0 ? max(0, it.qf[X] - p.window + 1) : 0;
    it.x0[X] = lo / BN;
    it.x1[X] = ql / BN + 1;
  }
  it.t0 = it.x0[0];
  it.n = max(it.x1[0], it.x1[1]) - it.t0;
  return it;
}

__device__ __forceinline__ bool item_act(const Item& it, int X, int j) {
  return it.t0 + j >= it.x0[X] && it.t0 + j < it.x1[X];
}

template <int HD>
__global__ void __launch_bounds__(kThreads2, 1)
prefill2_kernel(const __grid_constant__ PrefillParams p, int nseq, int nitems) {
  using Geo = PGeo2<HD>;
  constexpr int BN = Geo::BN, CH = Geo::CH, NS = Geo::NS;
  extern __shared__ unsigned char smem_raw[];
  __shared__ Sync2 sy;

  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* Qs = smem;                            // [2 tiles][CH][128][64]
  unsigned char* Ks = smem + 2 * Geo::QT_BYTES;
  unsigned char* Vs = Ks + NS * Geo::KV_BYTES;

  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    mbar_init(&sy.q_full, 1);
    mbar_init(&sy.drain, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sy.q_free[s], 1);
      mbar_init(&sy.k_full[s], 1);
      mbar_init(&sy.v_full[s], 1);
      mbar_init(&sy.k_empty[s], 1);
      mbar_init(&sy.v_empty[s], 1);
      mbar_init(&sy.s_full[s], 1);
      mbar_init(&sy.p_ready[s], 256);
      mbar_init(&sy.o_full[s], 1);
      mbar_init(&sy.o_free[s], 256);
    }
    sy.abort = 0;
  }
  if (warp == 1) {
    tc::tmem_alloc(&sy.tmem_base, 512);
    tc::tmem_relinquish();
  }
  fence_mbar_init();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = sy.tmem_base;
  // items are dealt boustrophedon-wise (round rr: CTA c takes the c-th item, or
  // the (C-1-c)-th on odd rounds) over the heaviest-first list, which evens out
  // the per-CTA load
  auto snake_item = [&](int rr) {
    const int c = (rr & 1) ? (int)gridDim.x - 1 - (int)blockIdx.x : (int)blockIdx.x;
    return rr * (int)gridDim.x + c;
  };

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (tc::elect_one()) {
      long g = 0;        // K/V tiles loaded so far (stage g % NS)
      int qrel[2] = {0, 0};      // q_free arrivals expected so far per query tile
      bool pend[2] = {false, false};
      int ic = 0;        // items started
      for (int rr = 0; rr * (int)gridDim.x < nitems && !sy.abort; ++rr) {
        const int w = snake_item(rr);
        if (w >= nitems) continue;
        const Item it = make_item<BN>(p, nseq, w);
        if (!it.valid) continue;
        // the previous item's epilogues must have released the Q buffer
        bool okq = true;
        for (int X = 0; X < 2 && okq; ++X)
          if (pend[X]) okq = wait2(&sy.q_free[X], (qrel[X] - 1) & 1, sy, p, 22);
        if (!okq) break;
        const int nqt = it.x1[1] > it.x0[1] ? 2 : 1;   // tile B may lie past P
        for (int X = 0; X < 2; ++X) {
          pend[X] = X < nqt;
          qrel[X] += X < nqt;
        }
        mbar_arrive_expect_tx(&sy.q_full, nqt * Geo::QT_BYTES);
        for (int X = 0; X < nqt; ++X)
          for (int c = 0; c < CH; ++c)
            tc::tma_load_2d(Qs + X * Geo::QT_BYTES + c * BM * 128, &p.qmap[it.seq],
                            it.h * HD + c * 64, it.qt * 2 * BM + X * BM, &sy.q_full);
        ++ic;
        for (int j = 0; j < it.n; ++j, ++g) {
          const int s = (int)(g % NS), row = (it.t0 + j) * BN;
          if (g >= NS && !wait2(&sy.k_empty[s], ((g / NS) - 1) & 1, sy, p, 20)) break;
          mbar_arrive_expect_tx(&sy.k_full[s], Geo::KV_BYTES);
          for (int c = 0; c < CH; ++c)
            tc::tma_load_2d(Ks + s * Geo::KV_BYTES + c * BN * 128, &p.kmap[it.seq],
                            it.kvh * HD + c * 64, row, &sy.k_full[s]);
          if (g >= NS && !wait2(&sy.v_empty[s], ((g / NS) - 1) & 1, sy, p, 21)) break;
          mbar_arrive_expect_tx(&sy.v_full[s], Geo::KV_BYTES);
          for (int c = 0; c < CH; ++c)
            tc::tma_load_2d(Vs + s * Geo::KV_BYTES + c * BN * 128, &p.vmap[it.seq],
                            it.kvh * HD + c * 64, row, &sy.v_full[s]);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------ MMA issuer --------------------------------
    if (tc::elect_one()) {
      constexpr uint32_t idS = tc::idesc_f16_f32(BM, BN, false, false);
      constexpr uint32_t idO = tc::idesc_f16_f32(BM, HD, false, true);
      const uint32_t qbase = smem_u32(Qs), kbase = smem_u32(Ks), vbase = smem_u32(Vs);
      long g = 0;                    // K/V tiles consumed (stage g % NS)
      int ic = 0;                    // items started
      int np[2] = {0, 0};            // P tiles consumed per query tile (all items)
      int no[2] = {0, 0};            // O accumulators handed to the epilogue
      auto issue_S = [&](int X, int s) {
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const int c = kk >> 2;
          const uint64_t a = tc::smem_desc_sw128(
              qbase + X * Geo::QT_BYTES + c * BM * 128 + (kk & 3) * 32, 16, 1024);
          const uint64_t b = tc::smem_desc_sw128(
              kbase + s * Geo::KV_BYTES + c * BN * 128 + (kk & 3) * 32, 16, 1024);
          tc::mma_ss(tmem + X * 128, a, b, idS, kk > 0);
        }
        tc::commit(&sy.s_full[X]);
      };
      auto issue_PV = [&](int X, int s, bool first) {
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint64_t b = tc::smem_desc_sw128(vbase + s * Geo::KV_BYTES + kk * 16 * 128,
                                                 BN * 128, 1024);
          tc::mma_ts(tmem + 256 + X * 128, tmem + X * 128 + kk * 8, b, idO,
                     (!first || kk > 0) ? 1u : 0u);
        }
      };
      bool ok = true;
      for (int rr = 0; ok && rr * (int)gridDim.x < nitems; ++rr) {
        const int w = snake_item(rr);
        if (w >= nitems) continue;
        const Item it = make_item<BN>(p, nseq, w);
        if (!it.valid) continue;
        if (!(ok = wait2(&sy.q_full, ic & 1, sy, p, 30))) break;
        ++ic;
        tc::fence_after_sync();
        // first S of the item
        {
          const int s = (int)(g % NS);
          if (!(ok = wait2(&sy.k_full[s], (g / NS) & 1, sy, p, 31))) break;
          tc::fence_after_sync();
          for (int X = 0; X < 2; ++X)
            if (item_act(it, X, 0)) issue_S(X, s);
          tc::commit(&sy.k_empty[s]);
        }
        for (int j = 0; ok && j < it.n; ++j) {
          const int s = (int)((g + j) % NS);
          if (!(ok = wait2(&sy.v_full[s], ((g + j) / NS) & 1, sy, p, 33))) break;
          const bool more = j + 1 < it.n;
          const int s1 = (int)((g + j + 1) % NS);
          if (more && !(ok = wait2(&sy.k_full[s1], ((g + j + 1) / NS) & 1, sy, p, 31))) break;
          tc::fence_after_sync();
          for (int X = 0; X < 2; ++X) {
            if (item_act(it, X, j)) {
              const bool first = it.t0 + j == it.x0[X];
              if (first && no[X] > 0 && !(ok = wait2(&sy.o_free[X], (no[X] - 1) & 1, sy, p, 34)))
                break;
              if (!(ok = wait2(&sy.p_ready[X], np[X] & 1, sy, p, 32))) break;
              TRACE(10 + X, np[X]);
              tc::fence_after_sync();
              issue_PV(X, s, first);
              ++np[X];
              if (it.t0 + j + 1 == it.x1[X]) {      // last PV of X in this item
                tc::commit(&sy.o_full[X]);
                ++no[X];
              }
            }
            if (more && item_act(it, X, j + 1)) issue_S(X, s1);
          }
          if (!ok) break;
          if (more) tc::commit(&sy.k_empty[s1]);
          tc::commit(&sy.v_empty[s]);
        }
        g += it.n;
      }
      // drain: every issued MMA completes before TMEM is released
      tc::commit(&sy.drain);
      mbar_wait_bounded(&sy.drain, 0);
    }
    __syncwarp();
  } else {
    // ------------------------------ softmax / epilogue ------------------------
    // Warps 2-9 serve query tile A, 10-17 tile B. Each row is split between
    // two threads (column halves) in warps with the same TMEM lane quarter;
    // they exchange partial row maxima through shared memory behind a
    // 64-thread named barrier, which also orders the P writes after both
    // halves have read their S columns.
    const int sw = warp - 2;
    const int X = sw >> 3;                            // query tile of this warp
    const int half = (sw >> 2) & 1;                   // column half of S / O
    const int lane = threadIdx.x & 31;
    const int wq = warp & 3;
    const int r = wq * 32 + lane;                     // row in tile == TMEM lane
    const int bar_id = 1 + X * 4 + wq;                // pairs the two halves
    constexpr int HB = BN / 2;                        // S columns per thread
    constexpr int HO = HD / 2;                        // O columns per thread
    const uint32_t lane_addr = (uint32_t)(wq * 32) << 16;
    const uint32_t sb = tmem + lane_addr + X * 128;
    const uint32_t ob = tmem + lane_addr + 256 + X * 128 + half * HO;
    const bool capped = p.softcap > 0.f;
    const float sc = capped ? 1.f : p.scale_log2;     // s -> log2 domain
    auto pair_sync = [&]() { asm volatile("bar.sync %0, 64;" ::"r"(bar_id) : "memory"); };
    int ks = 0;                                       // S tiles consumed (all items)
    int ne = 0;                                       // epilogues done
    for (int rr = 0; rr * (int)gridDim.x < nitems && !sy.abort; ++rr) {
        const int w = snake_item(rr);
        if (w >= nitems) continue;
      const Item it = make_item<BN>(p, nseq, w);
      if (!it.valid || it.x1[X] <= it.x0[X]) continue;
      const int qpos = it.qf[X] + r;
      const int win_lo = p.window > 0 ? qpos - p.window + 1 : 0;
      float m_run = -INFINITY, l_run = 0.f;
      bool ok = true;
      for (int t = it.x0[X]; t < it.x1[X]; ++t, ++ks) {
        if (!(ok = wait2(&sy.s_full[X], ks & 1, sy, p, 40))) break;
        tc::fence_after_sync();
        const int key0 = t * BN + half * HB;
        const bool masked = !(key0 + HB - 1 <= qpos && key0 >= win_lo && key0 + HB <= it.len);
        float s[HB];
        tc::tmem_ld32(sb + half * HB, s);
        tc::tmem_ld32(sb + half * HB + 32, s + 32);
        tc::tmem_wait_ld();
        if (capped) {
          scores_log2(s, true, p.softcap, p.scale_log2);
          scores_log2(s + 32, true, p.softcap, p.scale_log2);
        }
        if (masked) {
          mask_chunk(s, key0, qpos, win_lo, it.len);
          mask_chunk(s + 32, key0 + 32, qpos, win_lo, it.len);
        }
        // partial max (raw scores when uncapped: scale > 0 keeps the order)
        float m8[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) m8[k] = max3(s[k], s[8 + k], s[16 + k]);
#pragma unroll
        for (int k = 0; k < 8; ++k) m8[k] = max3(m8[k], s[24 + k], s[32 + k]);
#pragma unroll
        for (int k = 0; k < 8; ++k) m8[k] = max3(m8[k], s[40 + k], s[48 + k]);
#pragma unroll
        for (int k = 0; k < 8; ++k) m8[k] = fmaxf(m8[k], s[56 + k]);
        float mx = fmaxf(max3(m8[0], m8[1], m8[2]), max3(max3(m8[3], m8[4], m8[5]), m8[6], m8[7]));
        sy.xmax[ks & 1][X][half][r] = mx;
        pair_sync();                                  // both halves have read S
        mx = fmaxf(mx, sy.xmax[ks & 1][X][half ^ 1][r]) * sc;
        // keep the stale max unless some row of this warp grew by > 2^8
        const bool grow = __any_sync(0xffffffffu, mx > m_run + kRescaleThreshold);
        float corr = 1.f;
        if (grow) {
          const float m_new = fmaxf(m_run, mx);
          corr = m_new == -INFINITY ? 1.f : fast_exp2(m_run - m_new);
          m_run = m_new;
        }
        const float m_use = m_run == -INFINITY ? 0.f : m_run;
        const uint64_t sc2 = f2_pack(sc, sc), nm2 = f2_pack(-m_use, -m_use);
        uint64_t sum2[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) sum2[u] = f2_pack(0.f, 0.f);
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float2 a = f2_unpack(f2_fma(f2_pack(s[c * 32 + 2 * i], s[c * 32 + 2 * i + 1]), sc2, nm2));
            const float e0 = fast_exp2(a.x), e1 = fast_exp2(a.y);
            sum2[i & 3] = f2_add(sum2[i & 3], f2_pack(e0, e1));
            pk[i] = pack_half2(e0, e1);
          }
          tc::tmem_st16(sb + half * (HB / 2) + c * 16, pk);
        }
        const float2 sp = f2_unpack(f2_add(f2_add(sum2[0], sum2[1]), f2_add(sum2[2], sum2[3])));
        l_run = l_run * corr + (sp.x + sp.y);
        if (grow && t > it.x0[X]) {
          // S_X(t) landed, so PV_X(t-1) has too: rescale this half of O_X
#pragma unroll 1
          for (int c = 0; c < HO / 32; ++c) {
            float o[32];
            tc::tmem_ld32(ob + c * 32, o);
            tc::tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= corr;
            tc::tmem_st32(ob + c * 32, reinterpret_cast<const uint32_t*>(o));
          }
        }
        tc::tmem_wait_st();
        tc::fence_before_sync();
        mbar_arrive(&sy.p_ready[X]);
      }
      if (!ok || !wait2(&sy.o_full[X], ne & 1, sy, p, 42)) break;
      tc::fence_after_sync();
      sy.xsum[X][half][r] = l_run;
      pair_sync();
      const float l_tot = l_run + sy.xsum[X][half ^ 1][r];
      pair_sync();                                    // xsum reusable by the next item
      const int row0 = it.qt * 2 * BM + X * BM, row = row0 + r;
      const float inv = l_tot > 0.f ? 1.f / l_tot : 0.f;
      const float* gt = nullptr;
      void* outp = nullptr;
#pragma unroll
      for (int s = 0; s < kMaxSeq; ++s)
        if (s == it.seq) { gt = p.gate[s]; outp = p.out[s]; }
      const long obase = ((long)row * p.nq + it.h) * HD + half * HO;
      float o[HO];
#pragma unroll
      for (int c = 0; c < HO / 32; ++c) tc::tmem_ld32(ob + c * 32, o + c * 32);
      tc::tmem_wait_ld();
      tc::fence_before_sync();
      mbar_arrive(&sy.o_free[X]);                      // O_X may be overwritten
#pragma unroll
      for (int i = 0; i < HO; ++i) o[i] *= inv;
      if (gt && row < it.P) {
#pragma unroll
        for (int i = 0; i < HO; ++i) o[i] *= 1.f / (1.f + expf(-gt[obase + i]));
      }
      const bool leader = (sw & 7) == 0 && lane == 0;  // one thread per query tile
      if (!p.out_f32) {
        // stage the fp16 tile in this tile's (now idle) Q buffer, in the
        // 128-byte-swizzled layout of the TMA box, then store it with TMA
        // (rows past P are clipped by the tensor map)
        unsigned char* stg = Qs + X * Geo::QT_BYTES;
#pragma unroll
        for (int i8 = 0; i8 < HO / 8; ++i8) {
          const int col = half * HO + i8 * 8, chunk = col >> 6, cin = (col & 63) >> 3;
          const uint4 v = make_uint4(pack_half2(o[8 * i8], o[8 * i8 + 1]),
                                     pack_half2(o[8 * i8 + 2], o[8 * i8 + 3]),
                                     pack_half2(o[8 * i8 + 4], o[8 * i8 + 5]),
                                     pack_half2(o[8 * i8 + 6], o[8 * i8 + 7]));
          *reinterpret_cast<uint4*>(stg + chunk * BM * 128 + r * 128 + ((cin ^ (r & 7)) << 4)) = v;
        }
        fence_proxy_async_smem();
        asm volatile("bar.sync %0, 256;" ::"r"(9 + X) : "memory");
        if (leader) {
          for (int c = 0; c < CH; ++c)
            tc::tma_store_2d(&p.omap[it.seq], it.h * HD + c * 64, row0, stg + c * BM * 128);
          tc::bulk_commit_group();
          tc::bulk_wait_read();
          mbar_arrive(&sy.q_free[X]);                 // the producer may reload Q
        }
      } else {
        if (row < it.P) {
          float4* dst = reinterpret_cast<float4*>(static_cast<float*>(outp) + obase);
#pragma unroll
          for (int i = 0; i < HO / 4; ++i) dst[i] = make_float4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
        }
        if (leader) mbar_arrive(&sy.q_free[X]);       // Q is idle once O is final
      }
      ++ne;
    }
    if ((sw & 7) == 0 && (threadIdx.x & 31) == 0) tc::bulk_wait_all();  // stores landed
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, 512);
  }
}

// ---- host side ---------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

// 2D fp16 map over [rows][cols] (row stride cols*2 bytes), box 64 x box_rows,
// 128-byte swizzle, zero fill out of bounds.
bool make_map(CUtensorMap* m, const void* base, long cols, long rows, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <int HD>
int launch_prefill(PrefillParams& p, int nseq, cudaStream_t st) {
  using Geo = PGeo<HD>;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(prefill_kernel<HD>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, Geo::SMEM);
    if (e != cudaSuccess) return record_status((int)e);
    configured[dev] = true;
  }
  dim3 grid(p.ntq, p.nq, nseq);
  prefill_kernel<HD><<<grid, kThreads, Geo::SMEM, st>>>(p);
  ASPIDA_CHECK_LAUNCH();
  return 0;
}

template <int HD>
int launch_prefill2(PrefillParams& p, int nseq, cudaStream_t st) {
  using Geo = PGeo2<HD>;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(prefill2_kernel<HD>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, Geo::SMEM);
    if (e != cudaSuccess) return record_status((int)e);
    configured[dev] = true;
  }
  const int nitems = p.ntq * p.nq * nseq;
  const int grid = std::min(nitems, num_sms());
  prefill2_kernel<HD><<<grid, kThreads2, Geo::SMEM, st>>>(p, nseq, nitems);
  ASPIDA_CHECK_LAUNCH();
  return 0;
}

}  // namespace

int prefill_batch(int nseq, const void* const* q, const void* const* K, const void* const* V,
                  const float* const* gate, void* const* out, const int* P, const int* pos_start,
                  int out_f32, int nq, int nkv, int hd, float scale, int window, float softcap,
                  cudaStream_t st) {
  if (nseq <= 0) return 0;
  if (!q || !K || !V || !out || !P || !pos_start || nq <= 0 || nkv <= 0 || nq % nkv)
    return record_status(ASPIDA_ERR_ARG);
  if (hd != 64 && hd != 128 && hd != 256) return record_status(ASPIDA_ERR_UNSUPPORTED);
  for (int base = 0; base < nseq; base += kMaxSeq) {
    const int cnt = std::min(kMaxSeq, nseq - base);
    PrefillParams p;
    memset(&p, 0, sizeof(p));
    int maxP = 0;
    const int box_kv = hd <= 128 ? 128 : 64;
    for (int i = 0; i < cnt; ++i) {
      const int s = base + i;
      if (P[s] < 0 || pos_start[s] < 0 || !q[s] || !K[s] || !V[s] || !out[s])
        return record_status(ASPIDA_ERR_ARG);
      if (((uintptr_t)q[s] | (uintptr_t)K[s] | (uintptr_t)V[s] | (uintptr_t)out[s]) & 15)
        return record_status(ASPIDA_ERR_ARG);
      const int Pv = std::max(P[s], 1), len = pos_start[s] + Pv;
      if (!make_map(&p.qmap[i], q[s], (long)nq * hd, Pv, BM) ||
          !make_map(&p.kmap[i], K[s], (long)nkv * hd, len, box_kv) ||
          !make_map(&p.vmap[i], V[s], (long)nkv * hd, len, box_kv))
        return record_status(ASPIDA_ERR_ARG);
      if (!out_f32 && !make_map(&p.omap[i], out[s], (long)nq * hd, Pv, BM))
        return record_status(ASPIDA_ERR_ARG);
      p.out[i] = out[s];
      p.gate[i] = gate ? gate[s] : nullptr;
      p.P[i] = P[s];
      p.pos_start[i] = pos_start[s];
      maxP = std::max(maxP, P[s]);
    }
    if (maxP == 0) continue;
    p.status = device_status_ptr();
    p.nq = nq; p.nkv = nkv; p.G = nq / nkv;
    p.window = window; p.out_f32 = out_f32;
    p.scale_log2 = scale * kLog2e;
    p.softcap = softcap;
    int rc;
    if (hd <= 128) {
      p.ntq = (maxP + 2 * BM - 1) / (2 * BM);          // 256-row tiles
      rc = hd == 64 ? launch_prefill2<64>(p, cnt, st) : launch_prefill2<128>(p, cnt, st);
    } else {
      p.ntq = (maxP + BM - 1) / BM;
      rc = launch_prefill<256>(p, cnt, st);
    }
    if (rc) return rc;
  }
  return 0;
}

}  // namespace aspida

extern "C" int aspida_attn_prefill(const void* q, const void* K, const void* V, const float* gate,
                                   void* out, int out_f32, int nq, int nkv, int hd, int P,
                                   int pos_start, float scale, int window, float softcap,
                                   void* stream) {
  return aspida::prefill_batch(1, &q, &K, &V, gate ? &gate : nullptr, &out, &P, &pos_start,
                               out_f32, nq, nkv, hd, scale, window, softcap,
                               (cudaStream_t)stream);
}

extern "C" int aspida_attn_prefill_batch(int nseq, const void* const* q, const void* const* K,
                                         const void* const* V, const float* const* gate,
                                         void* const* out, const int* P, const int* pos_start,
                                         int out_f32, int nq, int nkv, int hd, float scale,
                                         int window, float softcap, void* stream) {
  return aspida::prefill_batch(nseq, q, K, V, gate, out, P, pos_start, out_f32, nq, nkv, hd, scale,
                               window, softcap, (cudaStream_t)stream);
}
