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
// Two persistent kernels (one CTA per SM walking a heaviest-first list of
// query tiles), both built from the same parts:
//   * a TMA producer warp: Q tiles and 2D-tensor-map K/V tiles (128-byte
//     swizzle) into double-buffered shared-memory stages;
//   * an MMA warp: one elected lane issues tcgen05.mma kind::f16,
//     S = Q K^T with A and B from shared memory (K-major descriptors) into
//     TMEM, and O += P V with P read from TMEM as the A operand (the TS form)
//     and V from shared memory (MN-major descriptor);
//   * softmax warps: thread r owns TMEM lane r (query row r), each row split
//     over two threads; online softmax in the log2 domain, P written as fp16
//     back into its S columns;
//   * an epilogue that stages O in the idle Q buffer and writes it with a TMA
//     tensor store.
// prefill2_kernel (hd 64/128) runs two 128-row query tiles per work item;
// prefill1_kernel (hd 256) runs one, with a double-buffered S.
//
// Every mbarrier wait is bounded; a wait that runs out sets the device
// status word and the CTA unwinds (TMEM is freed on every path).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <map>
#include <mutex>
#include <vector>
#include <queue>

#include "common.cuh"
#include "tcgen05.cuh"

namespace aspida {
namespace {

constexpr int BM = 128;
constexpr int kMaxSeq = 8;            // sequences per launch
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
  const int* btab[kMaxSeq];         // paged caches: block table per sequence, else null
  int block_size;                   // rows per block (a multiple of the key-tile height)
  // split-KV (one-tile kernel, one sequence): each query tile's key
  // range is cut into nsplit contiguous chunks, each an item writing an
  // unnormalised partial; split_merge_kernel combines them
  int nsplit;                       // 1 = no split
  // two-tile kernel: per-CTA item lists (CSR: offsets [grid + 1], then the
  // items), balanced on the host; null = items dealt boustrophedon-wise
  const int* sched;
  float* part_o;                    // [nsplit][P][nq][hd] unnormalised O
  float* part_ml;                   // [nsplit][P][nq][2]: row max (log2 units), row sum
  DeviceStatus* status;
  int nq, nkv, G, window, out_f32, ntq;
  float scale_log2, softcap;
};

// Row of the K/V tensor map holding key row `row` of sequence `seq`: the row
// itself for a contiguous cache; for a paged cache, its block's pool row
// (block_table[row / block_size] * block_size + row % block_size). A key
// tile never crosses a block because block_size is a multiple of its height.
__device__ __forceinline__ int kv_map_row(const PrefillParams& p, int seq, int row) {
  const int* bt = p.btab[seq];
  if (!bt) return row;
  return __ldg(bt + row / p.block_size) * p.block_size + row % p.block_size;
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

// 2^x for both lanes of an f32 pair on the FMA and integer pipes instead of
// the MUFU unit. Cody-Waite range reduction: n = round(x) with the 1.5 * 2^23
// shifter (n lands in the low mantissa bits), f = x - n in [-0.5, 0.5], 2^f
// from a polynomial (weighted least squares at Chebyshev nodes,
// exp2_poly_fit.py), and 2^n added to the exponent field. x is clamped to
// [-126, 64]: masked (-inf) scores give ~1e-38, which rounds to 0 in fp16.
//   DEG 3 (softmax P): max relative error 7.7e-5, below P's fp16 rounding.
//   DEG 4 (softcap tanh): 2.7e-6.
template <int DEG>
__device__ __forceinline__ uint64_t f2_exp2_poly(uint64_t x) {
  float2 v = f2_unpack(x);
  v.x = fminf(fmaxf(v.x, -126.f), 64.f);
  v.y = fminf(fmaxf(v.y, -126.f), 64.f);
  const uint64_t xc = f2_pack(v.x, v.y);
  const uint64_t t = f2_add(xc, f2_pack(12582912.f, 12582912.f));
  const uint64_t n = f2_add(t, f2_pack(-12582912.f, -12582912.f));
  const uint64_t f = f2_fma(n, f2_pack(-1.f, -1.f), xc);
  uint64_t p;
  if constexpr (DEG == 3) {
    p = f2_fma(f2_pack(0.055088684f, 0.055088684f), f, f2_pack(0.242604047f, 0.242604047f));
    p = f2_fma(p, f, f2_pack(0.693276227f, 0.693276227f));
    p = f2_fma(p, f, f2_pack(0.999928951f, 0.999928951f));
  } else {
    p = f2_fma(f2_pack(0.00956051052f, 0.00956051052f), f, f2_pack(0.0559170395f, 0.0559170395f));
    p = f2_fma(p, f, f2_pack(0.240249813f, 0.240249813f));
    p = f2_fma(p, f, f2_pack(0.69312197f, 0.69312197f));
    p = f2_fma(p, f, f2_pack(0.999999166f, 0.999999166f));
  }
  const float2 tv = f2_unpack(t), pv = f2_unpack(p);
  return f2_pack(__uint_as_float(__float_as_uint(pv.x) + (__float_as_uint(tv.x) << 23)),
                 __uint_as_float(__float_as_uint(pv.y) + (__float_as_uint(tv.y) << 23)));
}

// The two-tile kernel's softmax is MUFU-bound (two 128 x 128 score tiles need
// ~2048 MUFU cycles per key tile, as long as the tile's MMAs): one score pair
// in ASPIDA_EXP2_POLY_EVERY takes the polynomial path (config 3: +2%; the
// same split in the hd-256 kernel measured no gain).
#ifndef ASPIDA_EXP2_POLY_EVERY
#define ASPIDA_EXP2_POLY_EVERY 4
#endif

// Softcapped scores in log2 units: x <- cap * log2(e) * tanh(x * scale / cap),
// with tanh(y) = 1 - 2 / (1 + e^{2y}); e^{2y} from the degree-4 FMA-pipe
// exponential (taking one of the three MUFU operations per score off the
// MUFU unit) and the reciprocal from rcp.approx. Absolute tanh error ~2e-6
// (x50 cap: ~1e-4 in the score), no cancellation near 0 at that scale.
__device__ __forceinline__ void scores_log2(float* x, bool capped, float cap, float scale_log2) {
  if (capped) {
    const float sc2 = 2.f * scale_log2 / cap, cl = cap * kLog2e;   // 2y log2(e) = x * sc2
    const uint64_t s2 = f2_pack(sc2, sc2);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const uint64_t e2 = f2_exp2_poly<4>(f2_fma(f2_pack(x[2 * i], x[2 * i + 1]), s2,
                                                 f2_pack(0.f, 0.f)));
      const float2 e = f2_unpack(e2);
      float r0, r1;
      asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r0) : "f"(1.f + e.x));
      asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r1) : "f"(1.f + e.y));
      x[2 * i] = cl * fmaf(-2.f, r0, 1.f);
      x[2 * i + 1] = cl * fmaf(-2.f, r1, 1.f);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) x[i] *= scale_log2;
  }
}

// max(a, b, c) in one instruction (sm_100 three-input max).
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
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
  // or, with a host schedule, taken from this CTA's list; every role walks
  // the same sequence
  const int* sch = p.sched;
  const int s_begin = sch ? sch[blockIdx.x] : 0;
  const int rounds = sch ? sch[blockIdx.x + 1] - s_begin
                         : (nitems + (int)gridDim.x - 1) / (int)gridDim.x;
  auto snake_item = [&](int rr) {
    if (sch) return sch[gridDim.x + 1 + s_begin + rr];
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
      for (int rr = 0; rr < rounds && !sy.abort; ++rr) {
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
        // key-tile row in the K/V maps, looked up one tile ahead (paged caches)
        int nrow = it.n > 0 ? kv_map_row(p, it.seq, it.t0 * BN) : 0;
        for (int j = 0; j < it.n; ++j, ++g) {
          const int s = (int)(g % NS), row = nrow;
          if (j + 1 < it.n) nrow = kv_map_row(p, it.seq, (it.t0 + j + 1) * BN);
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
      for (int rr = 0; ok && rr < rounds; ++rr) {
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
    for (int rr = 0; rr < rounds && !sy.abort; ++rr) {
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
            const uint64_t a2 = f2_fma(f2_pack(s[c * 32 + 2 * i], s[c * 32 + 2 * i + 1]), sc2, nm2);
            float e0, e1;
            if (ASPIDA_EXP2_POLY_EVERY > 0 && i % ASPIDA_EXP2_POLY_EVERY == ASPIDA_EXP2_POLY_EVERY - 1) {
              const float2 e = f2_unpack(f2_exp2_poly<3>(a2));
              e0 = e.x;
              e1 = e.y;
            } else {
              const float2 a = f2_unpack(a2);
              e0 = fast_exp2(a.x);
              e1 = fast_exp2(a.y);
            }
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

// ---------------------------------------------------------------------------
// Persistent one-query-tile kernel for hd = 256 (two 128-row tiles do not fit
// TMEM next to a 256-column O). Work item: (sequence, head, 128-row tile),
// heaviest first, dealt boustrophedon-wise. K/V tiles of 64 keys; the S
// buffer is double-buffered, so the MMA issuer computes S(j+2) and PV(j)
// while the softmax works on S(j+1). TMEM: S0 [0,64), S1 [64,128),
// O [256,512). Softmax: 8 warps, each row split over two threads (32 keys
// each); O is rescaled only when a row's max grew by more than 2^8 (the
// rescale waits for the previous PV, o_done). Epilogue as in the two-tile
// kernel: O staged in the idle Q buffer, TMA tensor store, q_free.
// ---------------------------------------------------------------------------
constexpr int kThreads1 = 320;

template <int HD>
struct PGeo1 {
  static constexpr int BN = 64;
  static constexpr int CH = HD / 64;
  static constexpr int Q_BYTES = BM * HD * 2;
  static constexpr int KV_BYTES = BN * HD * 2;
  static constexpr int NS = 2;
  static constexpr int SMEM = Q_BYTES + 2 * NS * KV_BYTES + 1024;
};

struct Sync1 {
  uint64_t q_full, q_free;
  uint64_t k_full[2], v_full[2], k_empty[2], v_empty[2];
  uint64_t s_full[2], p_ready[2];
  uint64_t o_done, o_full, o_free, drain;
  float xmax[2][2][128];            // [tile parity][column half][row]
  float xsum[2][128];
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ bool wait1(uint64_t* bar, uint32_t parity, Sync1& sy,
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

struct Item1 {
  int seq, h, qt, P, len, kvh, qf, x0, x1, n, sp;
  bool valid;
};

// Key-tile chunk [a, b) of split sp of a query tile whose keys span tiles
// [x0, x1): equal contiguous chunks; empty when a >= b.
__host__ __device__ __forceinline__ void split_range(int x0, int x1, int nsplit, int sp, int& a,
                                                     int& b) {
  const int chunk = (x1 - x0 + nsplit - 1) / nsplit;
  a = x0 + sp * chunk;
  b = min(x1, a + chunk);
}

template <int BN>
__device__ __forceinline__ Item1 make_item1(const PrefillParams& p, int nseq, int w) {
  Item1 it;
  it.sp = w % p.nsplit;                    // the splits of one tile are dealt side by side
  w /= p.nsplit;
  const int per = nseq * p.nq;
  it.qt = p.ntq - 1 - w / per;
  const int rem = w % per;
  it.seq = rem / p.nq;
  it.h = rem % p.nq;
  int P = 0, ps = 0;
#pragma unroll
  for (int s = 0; s < kMaxSeq; ++s)
    if (s == it.seq) { P = p.P[s]; ps = p.pos_start[s]; }
  it.P = P;
  it.len = ps + P;
  it.kvh = it.h / p.G;
  it.valid = it.qt * BM < P;
  it.qf = ps + it.qt * BM;
  const int ql = min(ps + P, it.qf + BM) - 1;
  const int lo = p.window > 0 ? max(0, it.qf - p.window + 1) : 0;
  it.x0 = lo / BN;
  it.x1 = ql / BN + 1;
  if (p.nsplit > 1) {
    int a, b;
    split_range(it.x0, it.x1, p.nsplit, it.sp, a, b);
    it.x0 = a;
    it.x1 = max(a, b);
  }
  it.n = it.valid ? it.x1 - it.x0 : 0;
  it.valid = it.valid && it.n > 0;
  return it;
}

template <int HD>
__global__ void __launch_bounds__(kThreads1, 1)
prefill1_kernel(const __grid_constant__ PrefillParams p, int nseq, int nitems) {
  using Geo = PGeo1<HD>;
  constexpr int BN = Geo::BN, CH = Geo::CH, NS = Geo::NS;
  extern __shared__ unsigned char smem_raw[];
  __shared__ Sync1 sy;
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* Qs = smem;                                // [CH][128][64]
  unsigned char* Ks = smem + Geo::Q_BYTES;
  unsigned char* Vs = Ks + NS * Geo::KV_BYTES;
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    mbar_init(&sy.q_full, 1);
    mbar_init(&sy.q_free, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sy.k_full[s], 1);
      mbar_init(&sy.v_full[s], 1);
      mbar_init(&sy.k_empty[s], 1);
      mbar_init(&sy.v_empty[s], 1);
      mbar_init(&sy.s_full[s], 1);
      mbar_init(&sy.p_ready[s], 256);
    }
    mbar_init(&sy.o_done, 1);
    mbar_init(&sy.o_full, 1);
    mbar_init(&sy.o_free, 256);
    mbar_init(&sy.drain, 1);
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
  const int* sch = p.sched;                  // host schedule, or boustrophedon dealing
  const int s_begin = sch ? sch[blockIdx.x] : 0;
  const int rounds = sch ? sch[blockIdx.x + 1] - s_begin
                         : (nitems + (int)gridDim.x - 1) / (int)gridDim.x;
  auto snake_item = [&](int rr) {
    if (sch) return sch[gridDim.x + 1 + s_begin + rr];
    const int c = (rr & 1) ? (int)gridDim.x - 1 - (int)blockIdx.x : (int)blockIdx.x;
    return rr * (int)gridDim.x + c;
  };

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (tc::elect_one()) {
      long g = 0;
      int ic = 0;
      for (int rr = 0; rr < rounds && !sy.abort; ++rr) {
        const int w = snake_item(rr);
        if (w >= nitems) continue;
        const Item1 it = make_item1<BN>(p, nseq, w);
        if (!it.valid) continue;
        if (ic > 0 && !wait1(&sy.q_free, (ic - 1) & 1, sy, p, 22)) break;
        mbar_arrive_expect_tx(&sy.q_full, Geo::Q_BYTES);
        for (int c = 0; c < CH; ++c)
          tc::tma_load_2d(Qs + c * BM * 128, &p.qmap[it.seq], it.h * HD + c * 64, it.qt * BM,
                          &sy.q_full);
        ++ic;
        // key-tile row in the K/V maps, looked up one tile ahead (paged caches)
        int nrow = it.n > 0 ? kv_map_row(p, it.seq, it.x0 * BN) : 0;
        for (int j = 0; j < it.n; ++j, ++g) {
          const int s = (int)(g % NS), row = nrow;
          if (j + 1 < it.n) nrow = kv_map_row(p, it.seq, (it.x0 + j + 1) * BN);
          if (g >= NS && !wait1(&sy.k_empty[s], ((g / NS) - 1) & 1, sy, p, 20)) break;
          mbar_arrive_expect_tx(&sy.k_full[s], Geo::KV_BYTES);
          for (int c = 0; c < CH; ++c)
            tc::tma_load_2d(Ks + s * Geo::KV_BYTES + c * BN * 128, &p.kmap[it.seq],
                            it.kvh * HD + c * 64, row, &sy.k_full[s]);
          if (g >= NS && !wait1(&sy.v_empty[s], ((g / NS) - 1) & 1, sy, p, 21)) break;
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
      long g = 0;
      int ic = 0, kS = 0, kP = 0, nout = 0;
      bool ok = true;
      auto issue_S = [&](long gg) {
        const int s = (int)(gg % NS);
        if (!(ok = wait1(&sy.k_full[s], (gg / NS) & 1, sy, p, 31))) return;
        tc::fence_after_sync();
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const int c = kk >> 2;
          const uint64_t a = tc::smem_desc_sw128(qbase + c * BM * 128 + (kk & 3) * 32, 16, 1024);
          const uint64_t b = tc::smem_desc_sw128(
              kbase + s * Geo::KV_BYTES + c * BN * 128 + (kk & 3) * 32, 16, 1024);
          tc::mma_ss(tmem + (kS & 1) * 64, a, b, idS, kk > 0);
        }
        tc::commit(&sy.s_full[kS & 1]);
        tc::commit(&sy.k_empty[s]);
        ++kS;
      };
      for (int rr = 0; ok && rr < rounds; ++rr) {
        const int w = snake_item(rr);
        if (w >= nitems) continue;
        const Item1 it = make_item1<BN>(p, nseq, w);
        if (!it.valid) continue;
        if (!(ok = wait1(&sy.q_full, ic & 1, sy, p, 30))) break;
        ++ic;
        tc::fence_after_sync();
        for (int j = 0; ok && j < 2 && j < it.n; ++j) issue_S(g + j);
        for (int j = 0; ok && j < it.n; ++j) {
          const int s = (int)((g + j) % NS);
          if (!(ok = wait1(&sy.v_full[s], ((g + j) / NS) & 1, sy, p, 33))) break;
          if (j == 0 && nout > 0 && !(ok = wait1(&sy.o_free, (nout - 1) & 1, sy, p, 34))) break;
          if (!(ok = wait1(&sy.p_ready[kP & 1], (kP >> 1) & 1, sy, p, 32))) break;
          tc::fence_after_sync();
          const uint32_t pb = tmem + (kP & 1) * 64;
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk) {
            const uint64_t b = tc::smem_desc_sw128(vbase + s * Geo::KV_BYTES + kk * 16 * 128,
                                                   BN * 128, 1024);
            tc::mma_ts(tmem + 256, pb + kk * 8, b, idO, (j > 0 || kk > 0) ? 1u : 0u);
          }
          tc::commit(&sy.o_done);
          tc::commit(&sy.v_empty[s]);
          ++kP;
          if (j + 1 == it.n) {
            tc::commit(&sy.o_full);
            ++nout;
          }
          if (j + 2 < it.n) issue_S(g + j + 2);
        }
        g += it.n;
      }
      tc::commit(&sy.drain);
      mbar_wait_bounded(&sy.drain, 0);
    }
    __syncwarp();
  } else {
    // ------------------------------ softmax / epilogue ------------------------
    const int sw = warp - 2;                          // 0..7
    const int half = sw >> 2;                         // 32-key half of S; 128-col half of O
    const int lane = threadIdx.x & 31;
    const int wq = warp & 3;
    const int r = wq * 32 + lane;
    const int bar_id = 1 + wq;
    constexpr int HB = BN / 2, HO = HD / 2;
    const uint32_t lane_addr = (uint32_t)(wq * 32) << 16;
    const uint32_t ob = tmem + lane_addr + 256 + half * HO;
    const bool capped = p.softcap > 0.f;
    const float sc = capped ? 1.f : p.scale_log2;
    auto pair_sync = [&]() { asm volatile("bar.sync %0, 64;" ::"r"(bar_id) : "memory"); };
    int ks = 0, ne = 0;
    for (int rr = 0; rr < rounds && !sy.abort; ++rr) {
      const int w = snake_item(rr);
      if (w >= nitems) continue;
      const Item1 it = make_item1<BN>(p, nseq, w);
      if (!it.valid) continue;
      const int qpos = it.qf + r;
      const int win_lo = p.window > 0 ? qpos - p.window + 1 : 0;
      float m_run = -INFINITY, l_run = 0.f;
      bool ok = true;
      for (int t = it.x0; t < it.x1; ++t, ++ks) {
        const int kb = ks & 1;
        if (!(ok = wait1(&sy.s_full[kb], (ks >> 1) & 1, sy, p, 40))) break;
        tc::fence_after_sync();
        const uint32_t sb = tmem + lane_addr + kb * 64;
        const int key0 = t * BN + half * HB;
        const bool masked = !(key0 + HB - 1 <= qpos && key0 >= win_lo && key0 + HB <= it.len);
        float s[HB];
        tc::tmem_ld32(sb + half * HB, s);
        tc::tmem_wait_ld();
        if (capped) scores_log2(s, true, p.softcap, p.scale_log2);
        if (masked) mask_chunk(s, key0, qpos, win_lo, it.len);
        float m8[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) m8[k] = max3(s[k], s[8 + k], s[16 + k]);
#pragma unroll
        for (int k = 0; k < 8; ++k) m8[k] = fmaxf(m8[k], s[24 + k]);
        float mx = fmaxf(max3(m8[0], m8[1], m8[2]), max3(max3(m8[3], m8[4], m8[5]), m8[6], m8[7]));
        sy.xmax[kb][half][r] = mx;
        pair_sync();                                  // both halves have read S
        mx = fmaxf(mx, sy.xmax[kb][half ^ 1][r]) * sc;
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
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float2 a = f2_unpack(f2_fma(f2_pack(s[2 * i], s[2 * i + 1]), sc2, nm2));
          const float e0 = fast_exp2(a.x), e1 = fast_exp2(a.y);
          sum2[i & 3] = f2_add(sum2[i & 3], f2_pack(e0, e1));
          pk[i] = pack_half2(e0, e1);
        }
        tc::tmem_st16(sb + half * (HB / 2), pk);
        const float2 sp = f2_unpack(f2_add(f2_add(sum2[0], sum2[1]), f2_add(sum2[2], sum2[3])));
        l_run = l_run * corr + (sp.x + sp.y);
        if (grow && t > it.x0) {
          // rescale this half of O once PV(t-1) has landed
          if (!(ok = wait1(&sy.o_done, (ks - 1) & 1, sy, p, 41))) break;
          tc::fence_after_sync();
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
        mbar_arrive(&sy.p_ready[kb]);
      }
      if (!ok || !wait1(&sy.o_full, ne & 1, sy, p, 42)) break;
      tc::fence_after_sync();
      sy.xsum[half][r] = l_run;
      pair_sync();
      const float l_tot = l_run + sy.xsum[half ^ 1][r];
      pair_sync();
      const int row0 = it.qt * BM, row = row0 + r;
      const float inv = l_tot > 0.f ? 1.f / l_tot : 0.f;
      const float* gt = nullptr;
      void* outp = nullptr;
#pragma unroll
      for (int s = 0; s < kMaxSeq; ++s)
        if (s == it.seq) { gt = p.gate[s]; outp = p.out[s]; }
      const long obase = ((long)row * p.nq + it.h) * HD + half * HO;
      const bool leader = sw == 0 && lane == 0;
      if (p.nsplit > 1) {
        // split-KV partial: unnormalised O and (m, l) relative to m_run
        const long pr = ((long)it.sp * it.P + row) * p.nq + it.h;
#pragma unroll 1
        for (int c = 0; c < HO / 32; ++c) {
          float o[32];
          tc::tmem_ld32(ob + c * 32, o);
          tc::tmem_wait_ld();
          if (row < it.P) {
            float4* dst = reinterpret_cast<float4*>(p.part_o + pr * HD + half * HO + c * 32);
#pragma unroll
            for (int i = 0; i < 8; ++i) dst[i] = make_float4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
          }
        }
        if (row < it.P && half == 0) {
          p.part_ml[pr * 2] = m_run;
          p.part_ml[pr * 2 + 1] = l_tot;
        }
        tc::fence_before_sync();
        mbar_arrive(&sy.o_free);
        if (leader) mbar_arrive(&sy.q_free);
        ++ne;
        continue;
      }
#pragma unroll 1
      for (int c = 0; c < HO / 32; ++c) {
        float o[32];
        tc::tmem_ld32(ob + c * 32, o);
        tc::tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] *= inv;
        if (gt && row < it.P) {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= 1.f / (1.f + expf(-gt[obase + c * 32 + i]));
        }
        if (!p.out_f32) {
#pragma unroll
          for (int i8 = 0; i8 < 4; ++i8) {
            const int col = half * HO + c * 32 + i8 * 8, chunk = col >> 6, cin = (col & 63) >> 3;
            const uint4 v = make_uint4(pack_half2(o[8 * i8], o[8 * i8 + 1]),
                                       pack_half2(o[8 * i8 + 2], o[8 * i8 + 3]),
                                       pack_half2(o[8 * i8 + 4], o[8 * i8 + 5]),
                                       pack_half2(o[8 * i8 + 6], o[8 * i8 + 7]));
            *reinterpret_cast<uint4*>(Qs + chunk * BM * 128 + r * 128 + ((cin ^ (r & 7)) << 4)) = v;
          }
        } else if (row < it.P) {
          float4* dst = reinterpret_cast<float4*>(static_cast<float*>(outp) + obase + c * 32);
#pragma unroll
          for (int i = 0; i < 8; ++i) dst[i] = make_float4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
        }
      }
      tc::fence_before_sync();
      mbar_arrive(&sy.o_free);                         // O may be overwritten
      if (!p.out_f32) {
        fence_proxy_async_smem();
        asm volatile("bar.sync 9, 256;" ::: "memory");
        if (leader) {
          for (int c = 0; c < CH; ++c)
            tc::tma_store_2d(&p.omap[it.seq], it.h * HD + c * 64, row0, Qs + c * BM * 128);
          tc::bulk_commit_group();
          tc::bulk_wait_read();
          mbar_arrive(&sy.q_free);
        }
      } else if (leader) {
        mbar_arrive(&sy.q_free);
      }
      ++ne;
    }
    if (sw == 0 && (threadIdx.x & 31) == 0) tc::bulk_wait_all();
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, 512);
  }
}

// Combines the split-KV partials of one sequence: per (row, head), the
// log-sum-exp merge of gpu/fattn_sk.cu:84-97 over the splits that held keys
// of the row's query tile (recomputed as make_item1 cut them), then
// x sigmoid(gate). Block (row, head), one thread per dim.
__global__ void split_merge_kernel(const PrefillParams p, int hd, int bn) {
  const int row = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
  const int P = p.P[0], ps = p.pos_start[0];
  const int qt = row / BM, qf = ps + qt * BM;
  const int ql = min(ps + P, qf + BM) - 1;
  const int lo = p.window > 0 ? max(0, qf - p.window + 1) : 0;
  const int x0 = lo / bn, x1 = ql / bn + 1;
  float M = -INFINITY;
  for (int s = 0; s < p.nsplit; ++s) {
    int a, b;
    split_range(x0, x1, p.nsplit, s, a, b);
    if (a < b) M = fmaxf(M, p.part_ml[(((long)s * P + row) * p.nq + h) * 2]);
  }
  float L = 0.f, acc = 0.f;
  for (int s = 0; s < p.nsplit; ++s) {
    int a, b;
    split_range(x0, x1, p.nsplit, s, a, b);
    if (a >= b) continue;
    const long pr = ((long)s * P + row) * p.nq + h;
    const float m = p.part_ml[pr * 2];
    if (m == -INFINITY) continue;                 // no key of this split reached the row
    const float w = fast_exp2(m - M);
    L += w * p.part_ml[pr * 2 + 1];
    acc += w * p.part_o[pr * hd + d];
  }
  const long oi = ((long)row * p.nq + h) * hd + d;
  float v = L > 0.f ? acc / L : 0.f;
  if (p.gate[0]) v *= 1.f / (1.f + expf(-p.gate[0][oi]));
  if (p.out_f32) static_cast<float*>(p.out[0])[oi] = v;
  else static_cast<__half*>(p.out[0])[oi] = __float2half_rn(v);
}

const int* one_tile_schedule(const PrefillParams& p, int nseq, int nitems, int grid,
                             cudaStream_t st);

template <int HD>
int launch_prefill1(PrefillParams& p, int nseq, cudaStream_t st) {
  using Geo = PGeo1<HD>;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(prefill1_kernel<HD>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, Geo::SMEM);
    if (e != cudaSuccess) return record_status((int)e);
    configured[dev] = true;
  }
  const int nitems = p.ntq * p.nq * nseq * p.nsplit;
  const int grid = std::min(nitems, num_sms());
  p.sched = nitems > grid ? one_tile_schedule(p, nseq, nitems, grid, st) : nullptr;
  prefill1_kernel<HD><<<grid, kThreads1, Geo::SMEM, st>>>(p, nseq, nitems);
  ASPIDA_CHECK_LAUNCH();
  if (p.nsplit > 1) {
    split_merge_kernel<<<dim3(p.P[0], p.nq), HD, 0, st>>>(p, HD, Geo::BN);
    ASPIDA_CHECK_LAUNCH();
  }
  return 0;
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

// Longest-processing-time-first schedule of the two-tile kernel's items over
// `grid` CTAs: an item's cost is the key tiles of its two query tiles plus a
// fixed 2 for its Q load and epilogues (the same tile ranges make_item
// computes); items go, heaviest first, to the least-loaded CTA. Kept on the
// device per (device, shape); null when it cannot be had (then the kernel
// deals items boustrophedon-wise).
const int* two_tile_schedule(const PrefillParams& p, int nseq, int nitems, int grid,
                             cudaStream_t st) {
  constexpr int BN = 128;
  std::vector<int> key = {grid, nitems, nseq, p.nq, p.ntq, p.window};
  for (int s = 0; s < nseq; ++s) { key.push_back(p.P[s]); key.push_back(p.pos_start[s]); }
  int dev = 0;
  cudaGetDevice(&dev);
  key.push_back(dev);
  static std::mutex mu;
  static std::map<std::vector<int>, int*> cache;
  std::lock_guard<std::mutex> lk(mu);
  if (auto f = cache.find(key); f != cache.end()) return f->second;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) {
    cudaGetLastError();
    return nullptr;                       // no synchronous upload inside a capture
  }
  const int per = nseq * p.nq;
  std::vector<std::pair<long, int>> cost(nitems);
  for (int w = 0; w < nitems; ++w) {
    const int qt = p.ntq - 1 - w / per, seq = (w % per) / p.nq;
    const int P = p.P[seq], ps = p.pos_start[seq];
    long c = 2;
    for (int X = 0; X < 2; ++X) {
      const int r0 = qt * 2 * BM + X * BM;
      if (r0 >= P) continue;
      const int qf = ps + r0, ql = std::min(ps + P, qf + BM) - 1;
      const int lo = p.window > 0 ? std::max(0, qf - p.window + 1) : 0;
      c += ql / BN + 1 - lo / BN;
    }
    cost[w] = {qt * 2 * BM < P ? c : 0, w};
  }
  std::stable_sort(cost.begin(), cost.end(),
                   [](const auto& a, const auto& b) { return a.first > b.first; });
  std::vector<std::vector<int>> lists(grid);
  std::priority_queue<std::pair<long, int>, std::vector<std::pair<long, int>>,
                      std::greater<std::pair<long, int>>> load;
  for (int c = 0; c < grid; ++c) load.push({0, c});
  for (const auto& [c, w] : cost) {
    auto [l, cta] = load.top();
    load.pop();
    lists[cta].push_back(w);
    load.push({l + c, cta});
  }
  std::vector<int> csr(grid + 1 + nitems);
  csr[0] = 0;
  for (int c = 0; c < grid; ++c) {
    csr[c + 1] = csr[c] + (int)lists[c].size();
    std::copy(lists[c].begin(), lists[c].end(), csr.begin() + grid + 1 + csr[c]);
  }
  int* d = nullptr;
  if (cudaMalloc(&d, csr.size() * sizeof(int)) != cudaSuccess ||
      cudaMemcpy(d, csr.data(), csr.size() * sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess) {
    cudaGetLastError();
    if (d) cudaFree(d);
    return nullptr;
  }
  cache[key] = d;
  return d;
}

// The same schedule for the one-tile kernel: an item (query tile, head,
// split) costs its key tiles (64 keys) plus 2.
const int* one_tile_schedule(const PrefillParams& p, int nseq, int nitems, int grid,
                             cudaStream_t st) {
  constexpr int BN = 64;
  std::vector<int> key = {-1, grid, nitems, nseq, p.nq, p.ntq, p.window, p.nsplit};
  for (int s = 0; s < nseq; ++s) { key.push_back(p.P[s]); key.push_back(p.pos_start[s]); }
  int dev = 0;
  cudaGetDevice(&dev);
  key.push_back(dev);
  static std::mutex mu;
  static std::map<std::vector<int>, int*> cache;
  std::lock_guard<std::mutex> lk(mu);
  if (auto f = cache.find(key); f != cache.end()) return f->second;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) {
    cudaGetLastError();
    return nullptr;                       // no synchronous upload inside a capture
  }
  const int per = nseq * p.nq;
  std::vector<std::pair<long, int>> cost(nitems);
  for (int w0 = 0; w0 < nitems; ++w0) {
    const int sp = w0 % p.nsplit, w = w0 / p.nsplit;
    const int qt = p.ntq - 1 - w / per, seq = (w % per) / p.nq;
    const int P = p.P[seq], ps = p.pos_start[seq];
    long c = 0;
    if (qt * BM < P) {
      const int qf = ps + qt * BM, ql = std::min(ps + P, qf + BM) - 1;
      const int lo = p.window > 0 ? std::max(0, qf - p.window + 1) : 0;
      int x0 = lo / BN, x1 = ql / BN + 1;
      if (p.nsplit > 1) {
        int a, b;
        split_range(x0, x1, p.nsplit, sp, a, b);
        x0 = a;
        x1 = std::max(a, b);
      }
      if (x1 > x0) c = x1 - x0 + 2;
    }
    cost[w0] = {c, w0};
  }
  std::stable_sort(cost.begin(), cost.end(),
                   [](const auto& a, const auto& b) { return a.first > b.first; });
  std::vector<std::vector<int>> lists(grid);
  std::priority_queue<std::pair<long, int>, std::vector<std::pair<long, int>>,
                      std::greater<std::pair<long, int>>> load;
  for (int c = 0; c < grid; ++c) load.push({0, c});
  for (const auto& [c, w] : cost) {
    auto [l, cta] = load.top();
    load.pop();
    lists[cta].push_back(w);
    load.push({l + c, cta});
  }
  std::vector<int> csr(grid + 1 + nitems);
  csr[0] = 0;
  for (int c = 0; c < grid; ++c) {
    csr[c + 1] = csr[c] + (int)lists[c].size();
    std::copy(lists[c].begin(), lists[c].end(), csr.begin() + grid + 1 + csr[c]);
  }
  int* d = nullptr;
  if (cudaMalloc(&d, csr.size() * sizeof(int)) != cudaSuccess ||
      cudaMemcpy(d, csr.data(), csr.size() * sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess) {
    cudaGetLastError();
    if (d) cudaFree(d);
    return nullptr;
  }
  cache[key] = d;
  return d;
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
  p.sched = nitems > grid ? two_tile_schedule(p, nseq, nitems, grid, st) : nullptr;
  prefill2_kernel<HD><<<grid, kThreads2, Geo::SMEM, st>>>(p, nseq, nitems);
  ASPIDA_CHECK_LAUNCH();
  return 0;
}

}  // namespace

// Split-KV plan for a single-sequence prefill on the one-tile kernel (hd 256,
// or hd 128 for short chunks): when its (128-row query tile, head) items
// would leave SMs idle, cut each tile's key range into up to SMs / items
// chunks of at least 4 key tiles (so a long prefix fills the GPU); 1 = no
// split. prefill_split_bytes: the f32 partials' size.
int prefill_split_plan(int P, int pos_start, int nq, int hd, int window) {
  if ((hd != 256 && hd != 128) || P <= 0 || nq <= 0) return 1;
  const int items = ((P + BM - 1) / BM) * nq;
  const int sms = num_sms();
  if (items * 2 > sms) return 1;
  const int keys = window > 0 ? std::min(window + BM, pos_start + P) : pos_start + P;
  const int ns = std::min(sms / items, std::max(1, keys / 64 / 4));
  return std::max(1, std::min(ns, 16));
}
size_t prefill_split_bytes(int nsplit, int P, int nq, int hd) {
  return nsplit > 1 ? (size_t)nsplit * P * nq * (hd + 2) * sizeof(float) : 0;
}

// Paged form (block_table != null, one sequence): K/V are pools of num_blocks
// blocks of block_size rows.
int prefill_batch(int nseq, const void* const* q, const void* const* K, const void* const* V,
                  const float* const* gate, void* const* out, const int* P, const int* pos_start,
                  int out_f32, int nq, int nkv, int hd, float scale, int window, float softcap,
                  cudaStream_t st, const int* block_table = nullptr, int num_blocks = 0,
                  int block_size = 0, int nsplit = 1, float* part = nullptr) {
  if (nseq <= 0) return 0;
  if (!q || !K || !V || !out || !P || !pos_start || nq <= 0 || nkv <= 0 || nq % nkv)
    return record_status(ASPIDA_ERR_ARG);
  if (hd != 64 && hd != 128 && hd != 256) return record_status(ASPIDA_ERR_UNSUPPORTED);
  const int tile_rows = hd <= 128 ? 128 : 64;       // key-tile height of the kernel
  if (block_table) {
    if (nseq != 1 || num_blocks <= 0 || block_size <= 0) return record_status(ASPIDA_ERR_ARG);
    if (block_size % tile_rows) return record_status(ASPIDA_ERR_UNSUPPORTED);
    if ((long)num_blocks * block_size >= (1L << 31)) return record_status(ASPIDA_ERR_UNSUPPORTED);
  }
  for (int base = 0; base < nseq; base += kMaxSeq) {
    const int cnt = std::min(kMaxSeq, nseq - base);
    PrefillParams p;
    memset(&p, 0, sizeof(p));
    int maxP = 0;
    for (int i = 0; i < cnt; ++i) maxP = std::max(maxP, P[base + i]);
    // hd 128 normally runs two 128-row query tiles per item; a chunk too
    // short to fill the SMs with such items (or one being split) runs one
    // tile per item on the 64-key one-tile kernel instead
    const bool one_tile =
        hd == 256 || (hd == 128 && (nsplit > 1 || (long)((maxP + 2 * BM - 1) / (2 * BM)) * nq *
                                                          cnt * 2 <= num_sms()));
    const int box_kv = one_tile ? 64 : 128;           // the kernel's key-tile height
    maxP = 0;
    for (int i = 0; i < cnt; ++i) {
      const int s = base + i;
      if (P[s] < 0 || pos_start[s] < 0 || !q[s] || !K[s] || !V[s] || !out[s])
        return record_status(ASPIDA_ERR_ARG);
      if (((uintptr_t)q[s] | (uintptr_t)K[s] | (uintptr_t)V[s] | (uintptr_t)out[s]) & 15)
        return record_status(ASPIDA_ERR_ARG);
      const int Pv = std::max(P[s], 1), len = pos_start[s] + Pv;
      const int kv_rows = block_table ? num_blocks * block_size : len;
      if (!make_map(&p.qmap[i], q[s], (long)nq * hd, Pv, BM) ||
          !make_map(&p.kmap[i], K[s], (long)nkv * hd, kv_rows, box_kv) ||
          !make_map(&p.vmap[i], V[s], (long)nkv * hd, kv_rows, box_kv))
        return record_status(ASPIDA_ERR_ARG);
      p.btab[i] = block_table;
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
    p.block_size = block_size;
    p.nsplit = 1;
    if (nsplit > 1) {
      // split-KV partials (the one-tile kernel, one sequence)
      if (!one_tile || nseq != 1 || !part) return record_status(ASPIDA_ERR_ARG);
      p.nsplit = nsplit;
      p.part_o = part;
      p.part_ml = part + (size_t)nsplit * P[0] * nq * hd;
    }
    p.nq = nq; p.nkv = nkv; p.G = nq / nkv;
    p.window = window; p.out_f32 = out_f32;
    p.scale_log2 = scale * kLog2e;
    p.softcap = softcap;
    int rc;
    if (!one_tile) {
      p.ntq = (maxP + 2 * BM - 1) / (2 * BM);          // 256-row tiles
      rc = hd == 64 ? launch_prefill2<64>(p, cnt, st) : launch_prefill2<128>(p, cnt, st);
    } else {
      p.ntq = (maxP + BM - 1) / BM;
      rc = hd == 128 ? launch_prefill1<128>(p, cnt, st) : launch_prefill1<256>(p, cnt, st);
    }
    if (rc) return rc;
  }
  return 0;
}

}  // namespace aspida

namespace aspida {
namespace {
// Split-KV partial scratch of the single-sequence entry, per (device, stream).
std::mutex g_split_mu;
std::map<std::pair<int, cudaStream_t>, std::pair<void*, size_t>> g_split_scratch;
}  // namespace

// Scratch of at least `bytes` for split partials on (current device, st), or
// null when it cannot be had (the caller then runs without splitting).
float* split_scratch(size_t bytes, cudaStream_t st) {
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(g_split_mu);
  auto& s = g_split_scratch[{dev, st}];
  if (s.second < bytes) {
    if (s.first) { cudaStreamSynchronize(st); cudaFree(s.first); s = {nullptr, 0}; }
    if (cudaMalloc(&s.first, bytes) != cudaSuccess) { cudaGetLastError(); return nullptr; }
    s.second = bytes;
  }
  return static_cast<float*>(s.first);
}
}  // namespace aspida

extern "C" int aspida_attn_prefill(const void* q, const void* K, const void* V, const float* gate,
                                   void* out, int out_f32, int nq, int nkv, int hd, int P,
                                   int pos_start, float scale, int window, float softcap,
                                   void* stream) {
  cudaStream_t st = (cudaStream_t)stream;
  int nsplit = aspida::prefill_split_plan(P, pos_start, nq, hd, window);
  float* part = nullptr;
  if (nsplit > 1) {
    part = aspida::split_scratch(aspida::prefill_split_bytes(nsplit, P, nq, hd), st);
    if (!part) nsplit = 1;
  }
  return aspida::prefill_batch(1, &q, &K, &V, gate ? &gate : nullptr, &out, &P, &pos_start,
                               out_f32, nq, nkv, hd, scale, window, softcap, st, nullptr, 0, 0,
                               nsplit, part);
}

extern "C" int aspida_attn_prefill_paged(const void* q, const void* K_pool, const void* V_pool,
                                         const int* block_table, int num_blocks, int block_size,
                                         const float* gate, void* out, int out_f32, int nq,
                                         int nkv, int hd, int P, int pos_start, float scale,
                                         int window, float softcap, void* stream) {
  if (!block_table) return aspida::record_status(ASPIDA_ERR_ARG);
  return aspida::prefill_batch(1, &q, &K_pool, &V_pool, gate ? &gate : nullptr, &out, &P,
                               &pos_start, out_f32, nq, nkv, hd, scale, window, softcap,
                               (cudaStream_t)stream, block_table, num_blocks, block_size);
}

extern "C" int aspida_attn_prefill_batch(int nseq, const void* const* q, const void* const* K,
                                         const void* const* V, const float* const* gate,
                                         void* const* out, const int* P, const int* pos_start,
                                         int out_f32, int nq, int nkv, int hd, float scale,
                                         int window, float softcap, void* stream) {
  return aspida::prefill_batch(nseq, q, K, V, gate, out, P, pos_start, out_f32, nq, nkv, hd, scale,
                               window, softcap, (cudaStream_t)stream);
}
