// decode.cu — GQA decode attention over the resident fp16 KV cache.
//
// Replaces the shim's k_fattn_attend / k_fattn_attend_b (gpu/gpu_matvec.cu:
// 1507-1609), which run one 256-thread block per query head and so read every
// KV byte nq/nkv times through a two-pass fp32 score scratch. Here:
//
//  * A CTA owns a group of HPC adjacent kv heads. A cache row holds all kv
//    heads of one position ([pos][kv_head][dim]), so the group's slice of a
//    row is one contiguous HPC*hd*2-byte run (2 KB for 8 heads x hd 128, or
//    4 heads x hd 256). A producer warp streams 16 K rows + 16 V rows per
//    stage with the bulk-copy (TMA) engine, one cp.async.bulk per row,
//    completion counted on the stage's mbarrier; HPC consumer warps, one per
//    kv head, read their slice. Every KV byte crosses HBM once and DRAM sees
//    contiguous multi-KB runs.
//  * The work is the flattened list of 16-key units over all (sequence,
//    head group) segments, cut into equal contiguous ranges, one per CTA (a
//    stream-K style split): with ragged lengths every CTA streams the same
//    number of bytes, so none idles at the end. The per-sequence unit offsets
//    are a prefix sum every CTA computes in shared memory from pos[] (no host
//    round trip, so the launch is graph-capturable).
//  * Each consumer warp handles all G = nq/nkv query heads of its kv head.
//    Scores are computed transposed, S^T = K Q^T, with mma.sync m16n8k16:
//    M = 16 keys, N = 8 query heads (padded when G < 8), K = 16 dims. Q
//    enters as an fp16 hi + lo pair (two MMAs), so scores keep ~22 bits of
//    the f32 query. movmatrix turns the S^T accumulator into the P^T operand
//    of O^T = V^T P^T (M = 16 dims, N = 8 heads, K = 16 keys): softmax state
//    and O stay in registers.
//  * Online softmax in the log2 domain (scale folded with log2 e), fp32.
//  * A segment inside one CTA's range is finished by that CTA; a segment cut
//    between CTAs leaves one (m, l, o) partial per piece in the workspace
//    (slot = CTA + segment, unique because ranges are contiguous), and a
//    combine kernel merges them (the log-sum-exp merge of
//    gpu/fattn_sk.cu:84-97). The combine is launched as a programmatic
//    dependent, so its launch overlaps the decode grid and only its merge
//    work follows it.
#include <algorithm>
#include <type_traits>
#include <cmath>

#include <cuda_fp8.h>

#include "common.cuh"

namespace aspida {
namespace {

constexpr int kKeys = 16;       // keys per stage (one unit)
constexpr int kMaxB = 1024;     // sequences per launch (prefix sums in smem)
constexpr int kSmemBudget = 210 * 1024;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kNegBig = -3.402823466e38f;
// Q8_0 path: P x (V scale) is carried x 64 in fp16 so that small products
// stay normal; undone when a piece finishes. Safe for scales up to 1023
// (|v| up to ~130k before quantisation).
constexpr float kVScale = 64.f;

struct DecodeParams {
  const float* q;
  const float* gate;
  const __half* const* K;
  const __half* const* V;
  const int8_t* const* K8;    // Q8_0 form: int8 caches [rows][nkv*hd] ...
  const int8_t* const* V8;
  const __half* const* Ks;    // ... and fp16 scales [rows][nkv*hd/32]
  const __half* const* Vs;
  int f8;                     // the 8-bit caches hold fp8 e4m3 values, not int8
  int pdl;                    // launched as a programmatic dependent of the prep kernel
  const __half* Kpool;  // paged form: shared pools of blocks of block_size rows
  const __half* Vpool;
  const int* block_table;   // [B][max_blocks] block ids, or null (per-sequence caches)
  int block_size, max_blocks;
  const int* pos;       // mode 0
  const int* max_len;   // mode 0, optional
  const int* kv_lo;     // mode 1
  const int* kv_hi;     // mode 1
  float* out;           // mode 0: [B][nq*hd]
  float* part_m;        // mode 1: [B][nq]
  float* part_l;
  float* part_o;        // mode 1: [B][nq][hd]
  int* ws_pref;         // [B+1] unit offsets per sequence (for the combine)
  float* ws_ml;         // [slots][HPC][8][2]  (m in log2 units, l)
  float* ws_o;          // [slots][HPC][8][hd]
  DeviceStatus* status;
  // fused pre-attention step (aspida_attn_decode_fused): `q` holds raw
  // queries; the new raw K/V rows are appended at pos by the CTA that owns
  // each sequence's last unit; QK-RMSNorm weights (or null) and RoPE
  // parameters as for aspida_attn_prep
  const float* k_new;
  const float* v_new;
  const float* q_norm;
  const float* k_norm;
  const float* ff;
  float eps, rbase, freq_scale, m_scale, corr_lo, corr_hi;
  int fuse, rd, yarn_on, use_ff, interleaved, sec_total;
  long slots;
  int B, nq, nkv, G, window, mode;
  int hpc, ngroups;     // kv heads per CTA, head groups
  int nctas;            // CTAs that share the units
  float scale_log2, softcap;
};

// Key range [lo, hi) of sequence b.
__device__ __forceinline__ void seq_range(const DecodeParams& p, int b, int& lo, int& hi) {
  if (p.mode == 0) {
    const int ps = p.pos[b];
    hi = ps + 1;
    if (p.max_len) hi = min(hi, p.max_len[b]);
    lo = p.window > 0 ? max(0, ps - p.window + 1) : 0;
    if (lo < 0) lo = 0;
    if (hi < lo) hi = lo;
  } else {
    lo = max(0, p.kv_lo[b]);
    hi = max(lo, p.kv_hi[b]);
  }
}

__device__ __forceinline__ int units_of(const DecodeParams& p, int b) {
  int lo, hi;
  seq_range(p, b, lo, hi);
  return ((hi - lo + kKeys - 1) / kKeys) * p.ngroups;
}

// Prefix sum of unit counts per sequence into pref[0..B] (smem), by warp 0.
__device__ void build_prefix(const DecodeParams& p, int* pref) {
  const int lane = threadIdx.x & 31;
  if (threadIdx.x >= 32) return;
  const int per = (p.B + 31) / 32;
  const int b0 = lane * per, b1 = min(p.B, b0 + per);
  int local = 0;
  for (int b = b0; b < b1; ++b) local += units_of(p, b);
  int incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  int run = incl - local;
  for (int b = b0; b < b1; ++b) {
    pref[b] = run;
    run += units_of(p, b);
  }
  if (lane == 31) pref[p.B] = incl;
}

// First unit of CTA c's range: floor(c * U / C).
__device__ __forceinline__ long range_start(long c, long U, long C) { return c * U / C; }

// CTA whose range holds unit u: the largest c with range_start(c) <= u.
__device__ __forceinline__ long owner_of(long u, long U, long C) {
  long c = u * C / U;
  while (c + 1 < C && range_start(c + 1, U, C) <= u) ++c;
  return c;
}

// Cursor over a CTA's units; caches the current (sequence, head group) segment.
struct Cursor {
  long u, u_end;        // next unit, end of the CTA's range
  long seg_u0, seg_u1;  // unit range of the current segment
  int b, grp, lo, hi;   // sequence, head group, its key range
  bool valid;
};

__device__ __forceinline__ void cursor_seek(const DecodeParams& p, const int* pref, Cursor& c) {
  c.valid = c.u < c.u_end;
  if (!c.valid || (c.u >= c.seg_u0 && c.u < c.seg_u1)) return;
  int lo = 0, hi = p.B;  // largest b with pref[b] <= u
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (pref[mid] <= c.u) lo = mid; else hi = mid;
  }
  c.b = lo;
  seq_range(p, lo, c.lo, c.hi);
  const int nu = (c.hi - c.lo + kKeys - 1) / kKeys;  // units per head group
  c.grp = (int)(c.u - pref[lo]) / nu;
  c.seg_u0 = pref[lo] + (long)c.grp * nu;
  c.seg_u1 = c.seg_u0 + nu;
}

__device__ __forceinline__ int cursor_key0(const Cursor& c) {
  return c.lo + (int)(c.u - c.seg_u0) * kKeys;
}

template <int HD, int HPC, bool Q8>
struct Geometry {
  static constexpr int SLICE = HPC * HD * (Q8 ? 1 : 2);  // bytes of one row's group slice
  static constexpr int SSL = Q8 ? HPC * HD / 16 : 0;     // bytes of one row's group scales
  // A side's 16 stage rows sit in groups of RG consecutive rows padded by
  // PADG bytes. Q8_0: 4-row groups, one bulk copy each when the head group
  // is a whole cache row (the copy engine, not DRAM, bounds 1 KB row copies).
  // fp16: single rows (2 KB copies; 2-row copies measured no faster on the
  // batched shape and 4% slower on one long sequence).
  static constexpr int RG = Q8 ? 4 : 1, PADG = Q8 ? 32 : 16;
  static constexpr int GRPB = RG * SLICE + PADG;
  static constexpr int KVB = (kKeys / RG) * GRPB;        // bytes of one side's 16 rows
  static constexpr int STAGE_BYTES = 2 * KVB + 2 * kKeys * SSL;
  static constexpr int STAGES_RAW = (kSmemBudget - (kMaxB + 1) * 4) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_RAW > 8 ? 8 : (STAGES_RAW < 2 ? 2 : STAGES_RAW);
  static constexpr int THREADS = (HPC + 1) * 32;
  static constexpr int STAGE_TX = 2 * kKeys * (SLICE + SSL);  // bytes the copies bring per stage
};

// int8 -> fp16 helpers for the Q8_0 path. A byte b of a word pre-xored with
// 0x80808080 holds b + 128; placed in the low byte of an fp16 whose high byte
// is 0x64 it reads 1024 + b + 128, exact, so subtracting 1152 gives b exactly.
__device__ __forceinline__ uint32_t i8pair_to_h2(uint32_t biased, uint32_t sel) {
  const uint32_t x = __byte_perm(biased, 0x64646464u, sel);
  __half2 h = *reinterpret_cast<const __half2*>(&x);
  h = __hsub2(h, __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480)));
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Two 8-bit cache values -> fp16x2, exactly: bytes (0, 1) of w for sel
// 0x4140, bytes (2, 3) for 0x4342. int8 (F8 = false): w pre-xored with
// 0x80808080, i8pair_to_h2. fp8 e4m3 (F8 = true): every e4m3 value is an
// fp16 value, one cvt per pair.
template <bool F8>
__device__ __forceinline__ uint32_t kv8_to_h2(uint32_t w, uint32_t sel) {
  if constexpr (F8) {
    const __nv_fp8x2_storage_t pr = (__nv_fp8x2_storage_t)(sel == 0x4140u ? (w & 0xffffu) : (w >> 16));
    const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(pr, __NV_E4M3);
    return (uint32_t)h.x | ((uint32_t)h.y << 16);
  } else {
    return i8pair_to_h2(w, sel);
  }
}
// The bias that the int8 conversion expects; fp8 words are used as stored.
template <bool F8>
__device__ __forceinline__ uint32_t kv8_bias(uint32_t w) {
  return F8 ? w : (w ^ 0x80808080u);
}

// Byte offset of stage row k (0..15) within one side of a stage.
template <class Geo>
__device__ __forceinline__ int row_off(int k) {
  return (k / Geo::RG) * Geo::GRPB + (k % Geo::RG) * Geo::SLICE;
}
// Stage row held by MMA row m (the S^T row, and the k index of P^T / V^T).
// A slice is a multiple of 128 bytes, so rows of one group share banks and
// only the group padding separates them.
//  fp16 (1-row groups, 16-byte pad): identity; every 8-row ldmatrix phase
//    reads eight distinct 16-byte bank groups.
//  Q8_0 (4-row groups, 32-byte pad): MMA rows 0..7 fall two per group (K
//    reads at most 2-way conflicted); k indices 2t (and 2t+1, 2t+8, 2t+9),
//    t = 0..3, fall one per group (V reads conflict-free).
template <bool Q8>
__device__ __forceinline__ int stage_row(int m) {
  if constexpr (Q8) return 4 * ((m & 7) >> 1) + (m & 1) + 2 * (m >> 3);
  else return m;
}

// fp16 number i (0: low half) of a packed pair, as f32.
__device__ __forceinline__ float half_of(uint32_t w, int i) {
  return __half2float(__ushort_as_half((unsigned short)(i ? (w >> 16) : (w & 0xffffu))));
}

// Output dimension of accumulator element j of M tile mt. fp16 path: tile mt
// covers dims 16mt..16mt+15 in order. Q8 path: the two tiles of 32-dim block
// mt/2 interleave so that lane group g owns dims 4g..4g+3 of the block
// (rows g, g+8 of tile 2i -> dims 4g, 4g+1; of tile 2i+1 -> 4g+2, 4g+3).
template <bool Q8>
__device__ __forceinline__ int out_dim(int mt, int j, int g) {
  if constexpr (Q8) return (mt >> 1) * 32 + 4 * g + (mt & 1) * 2 + (j >> 1);
  else return mt * 16 + g + (j >> 1) * 8;
}

// Fused step, at a piece's start: RMSNorm (optional) and RoPE of this lane's
// raw query values (fp16 fragment layout: qv[kt][j] = dim kt*16 + qc + off,
// off = 0, 1, 8, 9). The 4 lanes of a column hold all its dims; a NeoX pair
// (d, d + rd/2) sits in one lane (kt and kt + rd/32) because rd is a multiple
// of 32, an interleaved pair (2i, 2i+1) in j = 0/1 or 2/3. Same formulas as
// prep_kernel (sum of squares reduced across the 4 lanes).
template <int HD>
__device__ __forceinline__ void fuse_q(const DecodeParams& p, float (&qv)[HD / 16][4], int pos,
                                       int qc, int lane) {
  constexpr int KT = HD / 16, NA = HD / 64;     // angles per lane: pairs lane + 32k, k < NA
  if (p.q_norm) {
    float ss = 0.f;
#pragma unroll
    for (int kt = 0; kt < KT; ++kt)
#pragma unroll
      for (int j = 0; j < 4; ++j) ss = fmaf(qv[kt][j], qv[kt][j], ss);
    ss += __shfl_xor_sync(0xffffffffu, ss, 1);
    ss += __shfl_xor_sync(0xffffffffu, ss, 2);
    const float rms = sqrtf(ss / (float)HD + p.eps);
#pragma unroll
    for (int kt = 0; kt < KT; ++kt)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int d = kt * 16 + qc + (j & 1) + (j >> 1) * 8;
        qv[kt][j] = __fmul_rn(qv[kt][j] / rms, p.q_norm[d]);
      }
  }
  // every angle once per warp: lane l evaluates pairs l + 32k (the same
  // formula as prep_kernel); a pair's lane fetches its cos / sin by shuffle
  const int npair = p.rd / 2;
  float ca[NA], sa[NA];
#pragma unroll
  for (int k = 0; k < NA; ++k) {
    const int i = lane + 32 * k;
    ca[k] = 1.f;
    sa[k] = 0.f;
    if (i < npair) {
      const int pos_eff = i < p.sec_total ? pos : 0;
      const float th = rope_angle(i, pos_eff, p.rd, p.rbase, p.freq_scale, p.yarn_on, p.corr_lo,
                                  p.corr_hi, p.ff, p.use_ff);
      ca[k] = __fmul_rn(cosf(th), p.m_scale);
      sa[k] = __fmul_rn(sinf(th), p.m_scale);
    }
  }
  const int half = p.rd / 2;
#pragma unroll
  for (int kt = 0; kt < KT; ++kt) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int d = kt * 16 + qc + (j & 1) + (j >> 1) * 8;
      // pair index of this dim (as the first of its pair), or -1
      int i = -1, kt2 = kt, j2 = j;
      if (p.interleaved) {
        if (d < p.rd && !(d & 1)) { i = d >> 1; j2 = j + 1; }
      } else if (d < half) {
        i = d;
        kt2 = kt + half / 16;
      }
      // all lanes take part in the shuffles; i's owner lane is i & 31
      const int src = i < 0 ? 0 : (i & 31), k = i < 0 ? 0 : (i >> 5);
      float c = 0.f, sn = 0.f;
#pragma unroll
      for (int kk = 0; kk < NA; ++kk) {
        const float cv = __shfl_sync(0xffffffffu, ca[kk], src);
        const float sv = __shfl_sync(0xffffffffu, sa[kk], src);
        if (kk == k) { c = cv; sn = sv; }
      }
      if (i < 0) continue;
      float x2 = 0.f;
#pragma unroll
      for (int kk = 0; kk < KT; ++kk)                 // kt2 is not a compile-time index
        if (kk == kt2) x2 = qv[kk][j2];
      const float x1 = qv[kt][j];
      const float o1 = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, sn));
      const float o2 = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, sn));
      qv[kt][j] = o1;
#pragma unroll
      for (int kk = 0; kk < KT; ++kk)
        if (kk == kt2) qv[kk][j2] = o2;
    }
  }
}

// One warp appends sequence b's new row for kv head kvh at position pos:
// V as given, K RMSNorm'ed (optional) and rotated, both to fp16 - through the
// same warp helpers as prep_kernel (warp_norm_row, rope_pair), so the cache
// rows are identical. sh: HD floats of scratch for the warp.
template <int HD>
__device__ void append_row(const DecodeParams& p, int b, int kvh, int pos, float* sh, int lane) {
  const long kvd = (long)p.nkv * HD;
  const float* kr = p.k_new + (long)b * kvd + (long)kvh * HD;
  const float* vr = p.v_new + (long)b * kvd + (long)kvh * HD;
  __half* Kc = const_cast<__half*>(p.K[b]) + (long)pos * kvd + (long)kvh * HD;
  __half* Vc = const_cast<__half*>(p.V[b]) + (long)pos * kvd + (long)kvh * HD;
  for (int d = lane; d < HD; d += 32) Vc[d] = __float2half_rn(vr[d]);
  warp_norm_row(kr, p.k_norm, p.eps, HD, sh, lane);
  RopeArgs r;
  r.ff = p.ff; r.base = p.rbase; r.freq_scale = p.freq_scale; r.m_scale = p.m_scale;
  r.corr_lo = p.corr_lo; r.corr_hi = p.corr_hi; r.rd = p.rd; r.yarn_on = p.yarn_on;
  r.use_ff = p.use_ff; r.interleaved = p.interleaved; r.sec_total = p.sec_total;
  for (int i = lane; i < p.rd / 2; i += 32) {
    int d1, d2;
    float o1, o2;
    rope_pair(sh, i, pos, r, d1, d2, o1, o2);
    Kc[d1] = __float2half_rn(o1);
    Kc[d2] = __float2half_rn(o2);
  }
  for (int d = p.rd + lane; d < HD; d += 32) Kc[d] = __float2half_rn(sh[d]);
  __syncwarp();
}

// Fused step: this CTA appends the new row of every (sequence, head group)
// segment whose last unit lies in its range [u0, u1) - the only unit that
// reads row pos - one consumer warp per kv head of the group.
template <int HD, int HPC>
__device__ void append_owned_rows(const DecodeParams& p, const int* pref, long u0, long u1,
                                  float* scratch, int warp, int lane) {
  long u = u0;
  while (u < u1) {
    int lo = 0, hi = p.B;                 // largest b with pref[b] <= u
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (pref[mid] <= u) lo = mid; else hi = mid;
    }
    const int b = lo;
    int klo, khi;
    seq_range(p, b, klo, khi);
    const int nu = (khi - klo + kKeys - 1) / kKeys;
    const int grp = (int)((u - pref[b]) / nu);
    const long s1 = pref[b] + (long)(grp + 1) * nu;
    const int pos = p.pos[b];
    if (s1 - 1 < u1 && pos >= 0 && khi == pos + 1 && warp < HPC)
      append_row<HD>(p, b, grp * HPC + warp, pos, scratch + warp * HD, lane);
    u = s1;
  }
}

template <int HD, int HPC, bool Q8, bool FUSE = false, bool F8 = false>
__global__ void __launch_bounds__(Geometry<HD, HPC, Q8>::THREADS, 1)
decode_kernel(const DecodeParams p) {
  using Geo = Geometry<HD, HPC, Q8>;
  constexpr int STAGE_BYTES = Geo::STAGE_BYTES, STAGES = Geo::STAGES;
  constexpr int KT = HD / 16;   // 16-dim steps
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ __align__(8) uint64_t full[STAGES], empty[STAGES];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int* pref = reinterpret_cast<int*>(smem + STAGES * STAGE_BYTES);

  build_prefix(p, pref);
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], HPC);
    }
  }
  fence_mbar_init();
  __syncthreads();
  const long U = pref[p.B];
  if (blockIdx.x == 0)
    for (int i = threadIdx.x; i <= p.B; i += blockDim.x) p.ws_pref[i] = pref[i];
  // let the combine grid get scheduled now; it waits for this grid to finish
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  // Every participating CTA owns at least one unit (piece counting relies on
  // it): with fewer units than CTAs, the surplus CTAs leave.
  const long C = min((long)p.nctas, max(U, 1L));
  const long cta = blockIdx.x;
  if (cta >= C) return;
  const long u_begin = range_start(cta, U, C), u_end = range_start(cta + 1, U, C);
  if constexpr (FUSE) {
    {
      // append the new rows this CTA will read, before its producer starts
      // (the stage buffers are idle scratch until then); the async-proxy
      // fence orders these generic stores before the bulk copies
      append_owned_rows<HD, HPC>(p, pref, u_begin, u_end, reinterpret_cast<float*>(smem), warp,
                                 lane);
      asm volatile("fence.proxy.async.global;" ::: "memory");
      __syncthreads();
    }
  }
  Cursor cur;
  cur.u = u_begin;
  cur.u_end = u_end;
  cur.seg_u0 = cur.seg_u1 = -1;
  cursor_seek(p, pref, cur);

  if (warp == HPC) {
    // ---------------- producer warp ----------------
    long fill = 0;
    // this lane's cache base pointers, reloaded only when the sequence
    // changes: a table read per stage would put a dependent global load on
    // the producer's critical path every 16 keys
    int cached_b = -1;
    const unsigned char *kb = nullptr, *vb = nullptr;
    [[maybe_unused]] const unsigned char *ksb = nullptr, *vsb = nullptr;
    // one head group per row: a stage's 16 rows are contiguous
    [[maybe_unused]] const bool whole_row = HPC == p.nkv;
    // As a programmatic dependent of the prep kernel, the cache rows it
    // appends (each segment's last rows) are loaded only after it completed;
    // the rows before them stream in the meantime.
    bool dep_done = p.pdl == 0;
#pragma unroll 1
    while (cur.valid) {
      const int slot = (int)(fill % STAGES);
      if (!dep_done && cursor_key0(cur) + kKeys >= cur.hi) {
        asm volatile("griddepcontrol.wait;" ::: "memory");
        dep_done = true;
      }
      if (fill >= STAGES) {
        const uint32_t par = (uint32_t)(((fill / STAGES) - 1) & 1);
        if (!mbar_wait_bounded(&empty[slot], par)) {
          if (lane == 0 && p.status) { atomicExch(&p.status->code, kDevTimeoutMbar); p.status->where = 10; }
          break;   // consumers drain what is in flight, then also stop
        }
      }
      if (lane == 0) mbar_arrive_expect_tx(&full[slot], Geo::STAGE_TX);
      __syncwarp();
      if (cur.b != cached_b) {
        cached_b = cur.b;
        if constexpr (Q8) {
          kb = reinterpret_cast<const unsigned char*>(p.K8[cur.b]);
          vb = reinterpret_cast<const unsigned char*>(p.V8[cur.b]);
          ksb = reinterpret_cast<const unsigned char*>(p.Ks[cur.b]);
          vsb = reinterpret_cast<const unsigned char*>(p.Vs[cur.b]);
        } else {
          kb = reinterpret_cast<const unsigned char*>(p.block_table ? p.Kpool : p.K[cur.b]);
          vb = reinterpret_cast<const unsigned char*>(p.block_table ? p.Vpool : p.V[cur.b]);
        }
      }
      unsigned char* dst = smem + slot * STAGE_BYTES;
      const int key0 = cursor_key0(cur);
      if constexpr (Q8) {
        const long rowb = (long)p.nkv * HD, srowb = rowb / 16;  // bytes per cache / scale row
        if (whole_row && key0 + kKeys <= cur.hi) {
          // 4 copies of 4 rows per side + one copy of the 16 rows' scales per side
          if (lane < 8) {
            const int which = lane >> 2, gq = lane & 3;
            bulk_g2s(dst + which * Geo::KVB + gq * Geo::GRPB,
                     (which ? vb : kb) + (long)(key0 + 4 * gq) * rowb, 4 * Geo::SLICE, &full[slot]);
          } else if (lane < 10) {
            const int which = lane - 8;
            bulk_g2s(dst + 2 * Geo::KVB + which * kKeys * Geo::SSL,
                     (which ? vsb : ksb) + (long)key0 * srowb, kKeys * Geo::SSL, &full[slot]);
          }
        } else {
          // row by row (segment end: rows past it repeat a valid row; or a
          // head group that is part of a row)
          const int which = lane >> 4, r = lane & 15;
          const int key = min(key0 + r, cur.hi - 1);
          bulk_g2s(dst + which * Geo::KVB + row_off<Geo>(r),
                   (which ? vb : kb) + (long)key * rowb + (long)cur.grp * Geo::SLICE, Geo::SLICE,
                   &full[slot]);
          bulk_g2s(dst + 2 * Geo::KVB + (which * kKeys + r) * Geo::SSL,
                   (which ? vsb : ksb) + (long)key * srowb + (long)cur.grp * Geo::SSL, Geo::SSL,
                   &full[slot]);
        }
      } else {
        const long rowb = 2L * p.nkv * HD;  // bytes per cache row
        const int which = lane >> 4;        // 0: K row, 1: V row
        const int r = lane & 15;
        const int key = min(key0 + r, cur.hi - 1);  // past the end: repeat a valid row
        long row = key;
        if (p.block_table) {            // paged: key -> (block id, row in block)
          const int blk = p.block_table[(long)cur.b * p.max_blocks + key / p.block_size];
          row = (long)blk * p.block_size + key % p.block_size;
        }
        bulk_g2s(dst + which * Geo::KVB + row_off<Geo>(r),
                 (which ? vb : kb) + row * rowb + (long)cur.grp * Geo::SLICE, Geo::SLICE,
                 &full[slot]);
      }
      ++fill;
      ++cur.u;
      cursor_seek(p, pref, cur);
    }
    return;
  }

  // ---------------- consumer warps: warp h = kv head grp*HPC + h ----------------
  const int h = warp;
  const int g = lane >> 2;            // query column this lane feeds in B fragments
  const int qc = 2 * (lane & 3);      // first of the two query columns it accumulates
  uint32_t qhi[KT][2], qlo[KT][2];
  float oacc[KT][4];
  float m_run[2], l_run[2];
  long consumed = 0;
  // fp16: ldmatrix row addresses of K (MMA row krow) and V^T (k index vrow)
  const int kcol = (lane >> 4) * 8, vcol = ((lane >> 3) & 1) * 8;
  [[maybe_unused]] const int krow_off =
      row_off<Geo>(stage_row<Q8>((lane & 7) + ((lane >> 3) & 1) * 8));
  [[maybe_unused]] const int vrow_off = row_off<Geo>(stage_row<Q8>((lane & 7) + (lane >> 4) * 8));
  // stage rows of MMA rows g and g+8 (masking, Q8_0 scales)
  const int q_r0 = stage_row<Q8>(g), q_r1 = stage_row<Q8>(g + 8);
  // Q8_0: K byte offsets of those rows, V byte offsets of k indices 2t,
  // 2t+1, 2t+8, 2t+9
  [[maybe_unused]] const int q_k0 = row_off<Geo>(q_r0), q_k1 = row_off<Geo>(q_r1);
  [[maybe_unused]] int q_v[4];
  {
    const int t = lane & 3;
    q_v[0] = row_off<Geo>(stage_row<Q8>(2 * t));
    q_v[1] = row_off<Geo>(stage_row<Q8>(2 * t + 1));
    q_v[2] = row_off<Geo>(stage_row<Q8>(2 * t + 8));
    q_v[3] = row_off<Geo>(stage_row<Q8>(2 * t + 9));
  }

  // the queries may come from the prep kernel this grid depends on
  if (p.pdl) asm volatile("griddepcontrol.wait;" ::: "memory");
#pragma unroll 1
  while (cur.valid) {
    const int kvh = cur.grp * HPC + h;
    if (cur.u == cur.seg_u0 || cur.u == u_begin) {
      // first unit of a piece: this kv head's G query rows as an fp16 hi/lo
      // pair in B-fragment layout; reset the softmax state
      const float* qb = p.q + ((long)cur.b * p.nq + (long)kvh * p.G) * HD;
      // this lane's query values of column g: qv[kt][j] = dims kt*16 + off(j),
      // fp16 path off = qc, qc+1, qc+8, qc+9; Q8 path 2qc .. 2qc+3
      float qv[KT][4];
#pragma unroll
      for (int kt = 0; kt < KT; ++kt) {
#pragma unroll
        for (int j = 0; j < 4; ++j) qv[kt][j] = 0.f;
        if (g < p.G) {
          if constexpr (Q8) {
            const float4 f = *reinterpret_cast<const float4*>(qb + g * HD + kt * 16 + 2 * qc);
            qv[kt][0] = f.x; qv[kt][1] = f.y; qv[kt][2] = f.z; qv[kt][3] = f.w;
          } else {
            const int d = kt * 16 + qc;
            const float2 a = *reinterpret_cast<const float2*>(qb + g * HD + d);
            const float2 c = *reinterpret_cast<const float2*>(qb + g * HD + d + 8);
            qv[kt][0] = a.x; qv[kt][1] = a.y; qv[kt][2] = c.x; qv[kt][3] = c.y;
          }
        }
      }
      if constexpr (FUSE) fuse_q<HD>(p, qv, p.pos[cur.b], qc, lane);
#pragma unroll
      for (int kt = 0; kt < KT; ++kt) {
        const float2 a = make_float2(qv[kt][0], qv[kt][1]), c = make_float2(qv[kt][2], qv[kt][3]);
        const __half2 ah = __floats2half2_rn(a.x, a.y), ch = __floats2half2_rn(c.x, c.y);
        const float2 ar = __half22float2(ah), cr = __half22float2(ch);
        qhi[kt][0] = *reinterpret_cast<const uint32_t*>(&ah);
        qhi[kt][1] = *reinterpret_cast<const uint32_t*>(&ch);
        qlo[kt][0] = pack_half2(a.x - ar.x, a.y - ar.y);
        qlo[kt][1] = pack_half2(c.x - cr.x, c.y - cr.y);
#pragma unroll
        for (int j = 0; j < 4; ++j) oacc[kt][j] = 0.f;
      }
      m_run[0] = m_run[1] = -INFINITY;
      l_run[0] = l_run[1] = 0.f;
    }
    // A pass handles NU consecutive units of a piece under one softmax
    // update. Passes take one unit: two per pass (one max over 32 keys,
    // interleaved MMA chains) measured slower on B200 for both cache types.
    const long piece_end = min(cur.seg_u1, u_end);
    constexpr int nu = 1;
    bool ok = true;
    auto pass = [&](auto nu_c) {
      constexpr int NU = decltype(nu_c)::value;
      int slot[NU];
#pragma unroll
      for (int i = 0; i < NU; ++i) {
        slot[i] = (int)((consumed + i) % STAGES);
        if (!mbar_wait_bounded(&full[slot[i]], (uint32_t)(((consumed + i) / STAGES) & 1))) {
          if (lane == 0 && p.status) { atomicExch(&p.status->code, kDevTimeoutMbar); p.status->where = 11; }
          ok = false;
          return;
        }
      }
      uint32_t kbase[NU], vbase[NU];
      // Q8_0: this head's block scales of key rows g and g+8 (K, then V), as
      // packed fp16 pairs, HD/64 words per row
      [[maybe_unused]] uint32_t kscw[NU][2][HD / 64], vscw[NU][2][HD / 64];
      float s4[NU][4];
#pragma unroll
      for (int i = 0; i < NU; ++i) {
        const unsigned char* st = smem + slot[i] * STAGE_BYTES + h * HD * (Q8 ? 1 : 2);
        kbase[i] = smem_u32(st);
        vbase[i] = smem_u32(st + Geo::KVB);
#pragma unroll
        for (int j = 0; j < 4; ++j) s4[i][j] = 0.f;
      }
      if constexpr (Q8) {
        const int t = lane & 3;
#pragma unroll
        for (int i = 0; i < NU; ++i) {
          const uint32_t sc = smem_u32(smem + slot[i] * STAGE_BYTES + 2 * Geo::KVB) + h * (HD / 16);
#pragma unroll
          for (int w = 0; w < HD / 64; ++w) {
            kscw[i][0][w] = lds_u32(sc + q_r0 * Geo::SSL + 4 * w);
            kscw[i][1][w] = lds_u32(sc + q_r1 * Geo::SSL + 4 * w);
            vscw[i][0][w] = lds_u32(sc + (kKeys + q_r0) * Geo::SSL + 4 * w);
            vscw[i][1][w] = lds_u32(sc + (kKeys + q_r1) * Geo::SSL + 4 * w);
          }
        }
        // per 32-dim block: integer K (exact in fp16) times Q, then the
        // block's per-key scale in f32
#pragma unroll
        for (int blk = 0; blk < HD / 32; ++blk) {
#pragma unroll
          for (int i = 0; i < NU; ++i) {
            float sb[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int kk = 0; kk < 2; ++kk) {
              const int kt = 2 * blk + kk;
              const uint32_t w0 = kv8_bias<F8>(lds_u32(kbase[i] + q_k0 + kt * 16 + 4 * t));
              const uint32_t w1 = kv8_bias<F8>(lds_u32(kbase[i] + q_k1 + kt * 16 + 4 * t));
              uint32_t a[4];
              a[0] = kv8_to_h2<F8>(w0, 0x4140);
              a[1] = kv8_to_h2<F8>(w1, 0x4140);
              a[2] = kv8_to_h2<F8>(w0, 0x4342);
              a[3] = kv8_to_h2<F8>(w1, 0x4342);
              mma_16816(sb, a, qlo[kt][0], qlo[kt][1]);
              mma_16816(sb, a, qhi[kt][0], qhi[kt][1]);
            }
            const float c0 = half_of(kscw[i][0][blk >> 1], blk & 1);
            const float c1 = half_of(kscw[i][1][blk >> 1], blk & 1);
            s4[i][0] = fmaf(c0, sb[0], s4[i][0]);
            s4[i][1] = fmaf(c0, sb[1], s4[i][1]);
            s4[i][2] = fmaf(c1, sb[2], s4[i][2]);
            s4[i][3] = fmaf(c1, sb[3], s4[i][3]);
          }
        }
      } else {
        // S^T = K (Q_hi + Q_lo)^T for 16 keys x 8 query columns
#pragma unroll
        for (int kt = 0; kt < KT; ++kt) {
#pragma unroll
          for (int i = 0; i < NU; ++i) {
            uint32_t a[4];
            ldmatrix_x4(a[0], a[1], a[2], a[3], kbase[i] + krow_off + (kt * 16 + kcol) * 2);
            mma_16816(s4[i], a, qlo[kt][0], qlo[kt][1]);
            mma_16816(s4[i], a, qhi[kt][0], qhi[kt][1]);
          }
        }
      }
      // scale (+ softcap), mask keys past the segment's end
      const int key0 = cursor_key0(cur);
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int i = 0; i < NU; ++i) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float x = s4[i][j];
          if (p.softcap > 0.f) x = p.softcap * tanhf(x * (p.scale_log2 / kLog2e) / p.softcap) * kLog2e;
          else x *= p.scale_log2;
          const int r = (j >> 1) ? q_r1 : q_r0;  // stage row
          s4[i][j] = key0 + i * kKeys + r < cur.hi ? x : -INFINITY;
        }
        mx0 = fmaxf(mx0, fmaxf(s4[i][0], s4[i][2]));
        mx1 = fmaxf(mx1, fmaxf(s4[i][1], s4[i][3]));
      }
      // online softmax per query column (qc, qc + 1)
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
      }
      const float mn0 = fmaxf(m_run[0], mx0), mn1 = fmaxf(m_run[1], mx1);
      const float c0 = fast_exp2(m_run[0] - mn0), c1 = fast_exp2(m_run[1] - mn1);
      m_run[0] = mn0;
      m_run[1] = mn1;
      float pr[NU][4];
      float ls0 = 0.f, ls1 = 0.f;
#pragma unroll
      for (int i = 0; i < NU; ++i) {
        pr[i][0] = fast_exp2(s4[i][0] - mn0);
        pr[i][1] = fast_exp2(s4[i][1] - mn1);
        pr[i][2] = fast_exp2(s4[i][2] - mn0);
        pr[i][3] = fast_exp2(s4[i][3] - mn1);
        ls0 += pr[i][0] + pr[i][2];
        ls1 += pr[i][1] + pr[i][3];
      }
      l_run[0] = l_run[0] * c0 + ls0;
      l_run[1] = l_run[1] * c1 + ls1;
#pragma unroll
      for (int kt = 0; kt < KT; ++kt) {
        oacc[kt][0] *= c0; oacc[kt][1] *= c1;
        oacc[kt][2] *= c0; oacc[kt][3] *= c1;
      }
      if constexpr (Q8) {
        // Per 32-dim block: P times the block's per-key V scale (and
        // kVScale), transposed into the B operand; V^T as exact integers
        // from four 4-byte reads (the stage rows of k indices 2t, 2t+1,
        // 2t+8, 2t+9, at dims 4g..4g+3).
#pragma unroll
        for (int blk = 0; blk < HD / 32; ++blk) {
#pragma unroll
          for (int i = 0; i < NU; ++i) {
            const float v0 = half_of(vscw[i][0][blk >> 1], blk & 1) * kVScale;
            const float v1 = half_of(vscw[i][1][blk >> 1], blk & 1) * kVScale;
            const uint32_t b0 = movmatrix_trans(pack_half2(pr[i][0] * v0, pr[i][1] * v0));
            const uint32_t b1 = movmatrix_trans(pack_half2(pr[i][2] * v1, pr[i][3] * v1));
            const uint32_t col = vbase[i] + blk * 32 + 4 * g;
            const uint32_t x0 = kv8_bias<F8>(lds_u32(col + q_v[0]));
            const uint32_t x1 = kv8_bias<F8>(lds_u32(col + q_v[1]));
            const uint32_t x2 = kv8_bias<F8>(lds_u32(col + q_v[2]));
            const uint32_t x3 = kv8_bias<F8>(lds_u32(col + q_v[3]));
            // byte-interleave rows: lo = dims 0,1 of both keys, hi = dims 2,3
            const uint32_t l01 = __byte_perm(x0, x1, 0x5140), h01 = __byte_perm(x0, x1, 0x7362);
            const uint32_t l23 = __byte_perm(x2, x3, 0x5140), h23 = __byte_perm(x2, x3, 0x7362);
            uint32_t a[4];
            a[0] = kv8_to_h2<F8>(l01, 0x4140);  // dim 4g   (tile 2blk row g),   keys 2t, 2t+1
            a[1] = kv8_to_h2<F8>(l01, 0x4342);  // dim 4g+1 (tile 2blk row g+8)
            a[2] = kv8_to_h2<F8>(l23, 0x4140);  // dim 4g,   keys 2t+8, 2t+9
            a[3] = kv8_to_h2<F8>(l23, 0x4342);
            mma_16816(oacc[2 * blk], a, b0, b1);
            a[0] = kv8_to_h2<F8>(h01, 0x4140);  // dims 4g+2, 4g+3 (tile 2blk+1)
            a[1] = kv8_to_h2<F8>(h01, 0x4342);
            a[2] = kv8_to_h2<F8>(h23, 0x4140);
            a[3] = kv8_to_h2<F8>(h23, 0x4342);
            mma_16816(oacc[2 * blk + 1], a, b0, b1);
          }
        }
      } else {
        // P^T operand via in-register transpose, then O^T += V^T P^T
#pragma unroll
        for (int i = 0; i < NU; ++i) {
          const uint32_t b0 = movmatrix_trans(pack_half2(pr[i][0], pr[i][1]));
          const uint32_t b1 = movmatrix_trans(pack_half2(pr[i][2], pr[i][3]));
#pragma unroll
          for (int mt = 0; mt < KT; ++mt) {
            uint32_t a[4];
            ldmatrix_x4_trans(a[0], a[1], a[2], a[3], vbase[i] + vrow_off + (mt * 16 + vcol) * 2);
            mma_16816(oacc[mt], a, b0, b1);
          }
        }
      }
      __syncwarp();
      if (lane == 0) {
#pragma unroll
        for (int i = 0; i < NU; ++i) mbar_arrive(&empty[slot[i]]);   // slots may be refilled
      }
    };
    pass(std::integral_constant<int, nu>{});
    if (!ok) return;
    consumed += nu;

    if (cur.u + nu == piece_end) {
      // piece done: reduce l across the lanes that share a query column
      float l0 = l_run[0], l1 = l_run[1];
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {
        l0 += __shfl_xor_sync(0xffffffffu, l0, o);
        l1 += __shfl_xor_sync(0xffffffffu, l1, o);
      }
      if constexpr (Q8) {
#pragma unroll
        for (int mt = 0; mt < KT; ++mt)
#pragma unroll
          for (int j = 0; j < 4; ++j) oacc[mt][j] *= 1.f / kVScale;
      }
      const bool whole = cur.seg_u0 >= u_begin && cur.seg_u1 <= u_end;
      const int h0 = kvh * p.G + qc;
      if (whole) {
        const float inv0 = 1.f / l0, inv1 = 1.f / l1;
        const long ob = (long)cur.b * p.nq * HD;
#pragma unroll
        for (int mt = 0; mt < KT; ++mt) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            if (qc + (j & 1) >= p.G) continue;
            const int dim = out_dim<Q8>(mt, j, g);
            const long idx = ob + (long)(h0 + (j & 1)) * HD + dim;
            if (p.mode == 0) {
              float v = oacc[mt][j] * ((j & 1) ? inv1 : inv0);
              if (p.gate) v *= 1.f / (1.f + expf(-p.gate[idx]));
              p.out[idx] = v;
            } else {
              p.part_o[idx] = oacc[mt][j];
            }
          }
        }
        if (p.mode == 1 && g == 0) {
          if (qc < p.G) {
            p.part_m[(long)cur.b * p.nq + h0] = m_run[0] * kLn2;
            p.part_l[(long)cur.b * p.nq + h0] = l0;
          }
          if (qc + 1 < p.G) {
            p.part_m[(long)cur.b * p.nq + h0 + 1] = m_run[1] * kLn2;
            p.part_l[(long)cur.b * p.nq + h0 + 1] = l1;
          }
        }
      } else {
        // a piece of a segment split between CTAs: leave its partial
        const long sid = (cta + (long)cur.b * p.ngroups + cur.grp) * HPC + h;
        float* wo = p.ws_o + sid * 8 * HD;
        float* wml = p.ws_ml + sid * 16;
#pragma unroll
        for (int mt = 0; mt < KT; ++mt) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int dim = out_dim<Q8>(mt, j, g);
            wo[(qc + (j & 1)) * HD + dim] = oacc[mt][j];
          }
        }
        if (g == 0) {
          wml[qc * 2 + 0] = m_run[0];
          wml[qc * 2 + 1] = l0;
          wml[(qc + 1) * 2 + 0] = m_run[1];
          wml[(qc + 1) * 2 + 1] = l1;
        }
      }
    }
    cur.u += nu;
    cursor_seek(p, pref, cur);
  }
}

// Merge the pieces of each split (sequence, kv head) segment, one block per
// query head: the log-sum-exp merge of gpu/fattn_sk.cu:84-97. The block's
// NW warps (4, or 32 when few segments are cut into many pieces) take every
// NW-th piece (lanes over dims), then reduce through shared memory. 4-warp
// blocks let a batch's blocks (config 2: 1024) be resident in one wave
// (8 warps: 1.2% slower step; 2 warps: 2.3% slower). Launched as a programmatic dependent of decode_kernel: the block
// is scheduled early and waits in griddepcontrol.wait until the decode grid
// has finished and its writes are visible. Sequences with an empty key range
// (no units) get zeros (mode 0) or an empty partial (mode 1) here.
template <int HD, int NW>
__global__ void __launch_bounds__(NW * 32) combine_kernel(const DecodeParams p) {
  constexpr int PER = HD / 32;
  __shared__ float red_o[NW][HD];
  __shared__ float red_m[NW], red_l[NW];
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int b = blockIdx.x, kvh = blockIdx.y, gq = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = kvh / p.hpc, h = kvh % p.hpc;
  const int hq = kvh * p.G + gq;
  const long U = p.ws_pref[p.B];
  const int nu = (p.ws_pref[b + 1] - p.ws_pref[b]) / p.ngroups;
  const long oi = ((long)b * p.nq + hq) * HD;
  if (nu == 0) {
    for (int d = threadIdx.x; d < HD; d += blockDim.x) {
      if (p.mode == 0) p.out[oi + d] = 0.f;
      else p.part_o[oi + d] = 0.f;
    }
    if (p.mode == 1 && threadIdx.x == 0) {
      p.part_m[(long)b * p.nq + hq] = kNegBig;
      p.part_l[(long)b * p.nq + hq] = 0.f;
    }
    return;
  }
  const long C = min((long)p.nctas, max(U, 1L));
  const long s0 = p.ws_pref[b] + (long)grp * nu;
  const long ca = owner_of(s0, U, C), cb = owner_of(s0 + nu - 1, U, C);
  if (ca == cb) return;  // whole segment: finished by its CTA
  const long seg = (long)b * p.ngroups + grp;

  float M = -INFINITY;
  for (long c = ca + threadIdx.x; c <= cb; c += blockDim.x)
    M = fmaxf(M, p.ws_ml[((c + seg) * p.hpc + h) * 16 + gq * 2]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
  if (lane == 0) red_m[warp] = M;
  __syncthreads();
  M = red_m[0];
#pragma unroll
  for (int w = 1; w < NW; ++w) M = fmaxf(M, red_m[w]);

  float L = 0.f, acc[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) acc[i] = 0.f;
#pragma unroll 8
  for (long c = ca + warp; c <= cb; c += NW) {
    const long s = (c + seg) * p.hpc + h;
    const float wt = fast_exp2(p.ws_ml[s * 16 + gq * 2] - M);
    L += wt * p.ws_ml[s * 16 + gq * 2 + 1];
    const float* o = p.ws_o + s * 8 * HD + gq * HD + lane * PER;
    if constexpr (PER == 2) {
      const float2 t = *reinterpret_cast<const float2*>(o);
      acc[0] += wt * t.x; acc[1] += wt * t.y;
    } else {
#pragma unroll
      for (int i = 0; i < PER; i += 4) {
        const float4 t = *reinterpret_cast<const float4*>(o + i);
        acc[i] += wt * t.x; acc[i + 1] += wt * t.y; acc[i + 2] += wt * t.z; acc[i + 3] += wt * t.w;
      }
    }
  }
#pragma unroll
  for (int i = 0; i < PER; ++i) red_o[warp][lane * PER + i] = acc[i];
  if (lane == 0) red_l[warp] = L;
  __syncthreads();
  L = 0.f;
#pragma unroll
  for (int w = 0; w < NW; ++w) L += red_l[w];
  for (int d = threadIdx.x; d < HD; d += blockDim.x) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) v += red_o[w][d];
    if (p.mode == 0) {
      float r = L > 0.f ? v / L : 0.f;
      if (p.gate) r *= 1.f / (1.f + expf(-p.gate[oi + d]));
      p.out[oi + d] = r;
    } else {
      p.part_o[oi + d] = v;
    }
  }
  if (p.mode == 1 && threadIdx.x == 0) {
    p.part_m[(long)b * p.nq + hq] = M * kLn2;
    p.part_l[(long)b * p.nq + hq] = L;
  }
}

// kv heads per CTA: the largest of 8/4/2/1 that divides nkv with a group
// slice of at most 1024 halves (2 KB per row). Q8_0 caches: the same head
// count bound, and a slice of at least 256 bytes so that a row's group scales
// are a whole number of 16-byte units for the bulk copy (0 = no such split).
int heads_per_cta(int nkv, int hd, bool q8 = false) {
  for (int h : {8, 4, 2, 1}) {
    if (nkv % h != 0) continue;
    if (!q8 && h * hd <= 1024) return h;
    if (q8 && h * hd <= 1024 && (h * hd) % 256 == 0) return h;
  }
  return q8 ? 0 : 1;
}

long max_ctas() { return (long)num_sms(); }

struct WsLayout { size_t pref, ml, o, total; long slots; };

WsLayout ws_layout(int B, int nkv, int hd, int hpc) {
  WsLayout w;
  w.slots = max_ctas() + (long)B * (nkv / hpc);
  auto al = [](size_t x) { return (x + 255) / 256 * 256; };
  w.pref = 0;
  w.ml = al((size_t)(B + 1) * sizeof(int));
  w.o = w.ml + al((size_t)w.slots * hpc * 16 * sizeof(float));
  w.total = w.o + al((size_t)w.slots * hpc * 8 * hd * sizeof(float));
  return w;
}

template <int HD, int HPC, bool Q8, bool FUSE = false, bool F8 = false>
int launch_decode_v(DecodeParams& p, long units_hint, int chunk, cudaStream_t st) {
  using Geo = Geometry<HD, HPC, Q8>;
  const size_t smem = (size_t)Geo::STAGES * Geo::STAGE_BYTES + (size_t)(p.B + 1) * sizeof(int);
  auto kern = decode_kernel<HD, HPC, Q8, FUSE, F8>;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(
        kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
        (int)((size_t)Geo::STAGES * Geo::STAGE_BYTES + (kMaxB + 1) * sizeof(int)));
    if (e != cudaSuccess) return record_status((int)e);
    configured[dev] = true;
  }
  long ctas = max_ctas();
  // chunk > 0: at least `chunk` keys per CTA range (fewer, longer ranges)
  if (chunk > 0) ctas = std::min(ctas, std::max(1L, units_hint * kKeys / chunk));
  ctas = std::min(ctas, std::max(1L, units_hint));
  p.nctas = (int)ctas;
  p.hpc = HPC;
  p.ngroups = p.nkv / HPC;
  if (p.pdl) {
    cudaLaunchConfig_t kc = {};
    kc.gridDim = dim3((unsigned)ctas);
    kc.blockDim = dim3(Geo::THREADS);
    kc.dynamicSmemBytes = smem;
    kc.stream = st;
    cudaLaunchAttribute ka[1];
    ka[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    ka[0].val.programmaticStreamSerializationAllowed = 1;
    kc.attrs = ka;
    kc.numAttrs = 1;
    if (cudaError_t e = cudaLaunchKernelEx(&kc, kern, p); e != cudaSuccess)
      return record_status((int)e);
  } else {
    kern<<<(int)ctas, Geo::THREADS, smem, st>>>(p);
    ASPIDA_CHECK_LAUNCH();
  }
  // the combine is a programmatic dependent: launched now, it runs its
  // merges as soon as the decode grid completes
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.B, p.nkv, p.G);
  // few segments for many CTAs (one long sequence): a segment has about
  // nctas / segments pieces; past 16, give each query head's merge 32 warps
  const bool wide = (long)p.B * p.ngroups * 16 < p.nctas;
  cfg.blockDim = dim3(wide ? 1024 : 128);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaError_t e = wide ? cudaLaunchKernelEx(&cfg, combine_kernel<HD, 32>, p)
                            : cudaLaunchKernelEx(&cfg, combine_kernel<HD, 4>, p);
      e != cudaSuccess)
    return record_status((int)e);
  return 0;
}

template <int HD>
int launch_decode_hd(DecodeParams& p, long units_hint, int chunk, cudaStream_t st) {
  if (p.K8 && p.f8) {
    switch (heads_per_cta(p.nkv, HD, true)) {
      case 8: return launch_decode_v<HD, (HD <= 128 ? 8 : 4), true, false, true>(p, units_hint, chunk, st);
      case 4: return launch_decode_v<HD, 4, true, false, true>(p, units_hint, chunk, st);
      case 2: return launch_decode_v<HD, (HD >= 128 ? 2 : 4), true, false, true>(p, units_hint, chunk, st);
      default: return launch_decode_v<HD, (HD == 256 ? 1 : 4), true, false, true>(p, units_hint, chunk, st);
    }
  }
  if (p.K8) {
    switch (heads_per_cta(p.nkv, HD, true)) {
      case 8: return launch_decode_v<HD, (HD <= 128 ? 8 : 4), true>(p, units_hint, chunk, st);
      case 4: return launch_decode_v<HD, 4, true>(p, units_hint, chunk, st);
      case 2: return launch_decode_v<HD, (HD >= 128 ? 2 : 4), true>(p, units_hint, chunk, st);
      default: return launch_decode_v<HD, (HD == 256 ? 1 : 4), true>(p, units_hint, chunk, st);
    }
  }
  if (p.fuse) {
    switch (heads_per_cta(p.nkv, HD)) {
      case 8: return launch_decode_v<HD, (HD <= 128 ? 8 : 4), false, true>(p, units_hint, chunk, st);
      case 4: return launch_decode_v<HD, 4, false, true>(p, units_hint, chunk, st);
      case 2: return launch_decode_v<HD, 2, false, true>(p, units_hint, chunk, st);
      default: return launch_decode_v<HD, 1, false, true>(p, units_hint, chunk, st);
    }
  }
  switch (heads_per_cta(p.nkv, HD)) {
    case 8: return launch_decode_v<HD, (HD <= 128 ? 8 : 4), false>(p, units_hint, chunk, st);
    case 4: return launch_decode_v<HD, 4, false>(p, units_hint, chunk, st);
    case 2: return launch_decode_v<HD, 2, false>(p, units_hint, chunk, st);
    default: return launch_decode_v<HD, 1, false>(p, units_hint, chunk, st);
  }
}

int run_decode(DecodeParams& p, int hd, int max_kv_len, int chunk, void* ws, size_t ws_bytes,
               cudaStream_t st) {
  if (p.B <= 0) return 0;
  if (p.B > kMaxB || p.nq <= 0 || p.nkv <= 0 || p.nq % p.nkv != 0 || !p.q ||
      (p.block_table ? (!p.Kpool || !p.Vpool || p.block_size <= 0 || p.max_blocks <= 0)
       : p.K8        ? (!p.V8 || !p.Ks || !p.Vs)
                     : (!p.K || !p.V)) ||
      max_kv_len < 0 || chunk < 0)
    return record_status(ASPIDA_ERR_ARG);
  if (p.G > 8 || (hd != 64 && hd != 128 && hd != 256)) return record_status(ASPIDA_ERR_UNSUPPORTED);
  if (p.K8 && heads_per_cta(p.nkv, hd, true) == 0) return record_status(ASPIDA_ERR_UNSUPPORTED);
  const int hpc = heads_per_cta(p.nkv, hd, p.K8 != nullptr);
  const long units_hint = (long)p.B * p.nkv * ((std::max(1, max_kv_len) + kKeys - 1) / kKeys);
  if (units_hint >= (1L << 31)) return record_status(ASPIDA_ERR_UNSUPPORTED);
  WsLayout w = ws_layout(p.B, p.nkv, hd, hpc);
  if (!ws || ws_bytes < w.total) return record_status(ASPIDA_ERR_WORKSPACE);
  if (((uintptr_t)ws & 255) != 0) return record_status(ASPIDA_ERR_ARG);
  unsigned char* wb = static_cast<unsigned char*>(ws);
  p.ws_pref = reinterpret_cast<int*>(wb + w.pref);
  p.ws_ml = reinterpret_cast<float*>(wb + w.ml);
  p.ws_o = reinterpret_cast<float*>(wb + w.o);
  p.slots = w.slots;
  if (!p.status) p.status = device_status_ptr();
  switch (hd) {
    case 64: return launch_decode_hd<64>(p, units_hint / hpc, chunk, st);
    case 128: return launch_decode_hd<128>(p, units_hint / hpc, chunk, st);
    default: return launch_decode_hd<256>(p, units_hint / hpc, chunk, st);
  }
}

}  // namespace

size_t decode_workspace_size(int B, int nq, int nkv, int hd, int max_kv_len, int chunk) {
  (void)nq; (void)max_kv_len; (void)chunk;
  if (B <= 0 || nkv <= 0) return 0;
  // one size serves the fp16 and the Q8_0 caches
  size_t n = ws_layout(B, nkv, hd, heads_per_cta(nkv, hd)).total;
  if (const int h8 = heads_per_cta(nkv, hd, true)) n = std::max(n, ws_layout(B, nkv, hd, h8).total);
  return n;
}

int decode(const float* q, const float* gate, const void* const* K, const void* const* V,
           const int* pos, const int* max_len, float* out, int B, int nq, int nkv, int hd,
           float scale, int window, float softcap, int max_kv_len, int chunk, void* ws,
           size_t ws_bytes, cudaStream_t st, bool after_prep = false) {
  DecodeParams p{};
  p.pdl = after_prep ? 1 : 0;
  p.q = q; p.gate = gate;
  p.K = reinterpret_cast<const __half* const*>(K);
  p.V = reinterpret_cast<const __half* const*>(V);
  p.pos = pos; p.max_len = max_len; p.out = out;
  p.B = B; p.nq = nq; p.nkv = nkv; p.G = nkv > 0 ? nq / nkv : 0;
  p.window = window; p.mode = 0;
  p.scale_log2 = scale * kLog2e; p.softcap = softcap;
  if (B > 0 && (!pos || !out)) return record_status(ASPIDA_ERR_ARG);
  return run_decode(p, hd, max_kv_len, chunk, ws, ws_bytes, st);
}

// As decode(), with the device status word supplied by the caller instead of
// the library's lazily allocated one.
int decode_with_status(const float* q, const float* gate, const void* const* K,
                       const void* const* V, const int* pos, const int* max_len, float* out,
                       int B, int nq, int nkv, int hd, float scale, int window, float softcap,
                       int max_kv_len, int chunk, void* ws, size_t ws_bytes,
                       DeviceStatus* status, cudaStream_t st) {
  DecodeParams p{};
  p.q = q; p.gate = gate;
  p.K = reinterpret_cast<const __half* const*>(K);
  p.V = reinterpret_cast<const __half* const*>(V);
  p.pos = pos; p.max_len = max_len; p.out = out;
  p.B = B; p.nq = nq; p.nkv = nkv; p.G = nkv > 0 ? nq / nkv : 0;
  p.window = window; p.mode = 0;
  p.scale_log2 = scale * kLog2e; p.softcap = softcap;
  p.status = status;
  if (B > 0 && (!pos || !out)) return record_status(ASPIDA_ERR_ARG);
  return run_decode(p, hd, max_kv_len, chunk, ws, ws_bytes, st);
}

int decode_paged(const float* q, const float* gate, const void* K_pool, const void* V_pool,
                 const int* block_table, int max_blocks, int block_size, const int* pos,
                 float* out, int B, int nq, int nkv, int hd, float scale, int window,
                 float softcap, int max_kv_len, int chunk, void* ws, size_t ws_bytes,
                 cudaStream_t st) {
  DecodeParams p{};
  p.q = q; p.gate = gate;
  p.Kpool = static_cast<const __half*>(K_pool);
  p.Vpool = static_cast<const __half*>(V_pool);
  p.block_table = block_table; p.block_size = block_size; p.max_blocks = max_blocks;
  p.pos = pos; p.out = out;
  p.B = B; p.nq = nq; p.nkv = nkv; p.G = nkv > 0 ? nq / nkv : 0;
  p.window = window; p.mode = 0;
  p.scale_log2 = scale * kLog2e; p.softcap = softcap;
  if (B > 0 && (!pos || !out || !block_table)) return record_status(ASPIDA_ERR_ARG);
  if (max_kv_len > (long)max_blocks * block_size) return record_status(ASPIDA_ERR_ARG);
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
  if (B > 0 && (!kv_lo || !kv_hi || !m || !l || !o)) return record_status(ASPIDA_ERR_ARG);
  return run_decode(p, hd, max_kv_len, chunk, ws, ws_bytes, st);
}

int decode_fused(const float* q_raw, const float* k_raw, const float* v_raw, const float* gate,
                 const void* const* K, const void* const* V, const int* pos, const int* max_len,
                 float* out, int B, int nq, int nkv, int hd, const float* q_norm,
                 const float* k_norm, float eps, int rd, float base, float freq_scale,
                 float m_scale, int yarn_on, float corr_lo, float corr_hi, const float* ff,
                 int use_ff, int interleaved, int sec_total, float scale, int window,
                 float softcap, int max_kv_len, int chunk, void* ws, size_t ws_bytes,
                 cudaStream_t st) {
  DecodeParams p{};
  p.q = q_raw; p.gate = gate;
  p.K = reinterpret_cast<const __half* const*>(K);
  p.V = reinterpret_cast<const __half* const*>(V);
  p.pos = pos; p.max_len = max_len; p.out = out;
  p.B = B; p.nq = nq; p.nkv = nkv; p.G = nkv > 0 ? nq / nkv : 0;
  p.window = window; p.mode = 0;
  p.scale_log2 = scale * kLog2e; p.softcap = softcap;
  p.fuse = 1;
  p.k_new = k_raw; p.v_new = v_raw; p.q_norm = q_norm; p.k_norm = k_norm; p.eps = eps;
  p.rd = rd; p.rbase = base; p.freq_scale = freq_scale; p.m_scale = m_scale;
  p.yarn_on = yarn_on; p.corr_lo = corr_lo; p.corr_hi = corr_hi; p.ff = ff; p.use_ff = use_ff;
  p.interleaved = interleaved; p.sec_total = sec_total;
  if (B > 0 && (!pos || !out || !k_raw || !v_raw || rd < 0 || rd > hd || (rd & 1) ||
                (use_ff && !ff)))
    return record_status(ASPIDA_ERR_ARG);
  // a NeoX pair (d, d + rd/2) must sit in one lane of the fragment layout
  if (!interleaved && (rd % 32) != 0) return record_status(ASPIDA_ERR_UNSUPPORTED);
  return run_decode(p, hd, max_kv_len, chunk, ws, ws_bytes, st);
}

int decode_q8(const float* q, const float* gate, const void* const* K8, const void* const* V8,
              const void* const* Ks, const void* const* Vs, const int* pos, const int* max_len,
              float* out, int B, int nq, int nkv, int hd, float scale, int window, float softcap,
              int max_kv_len, int chunk, void* ws, size_t ws_bytes, cudaStream_t st,
              bool f8 = false) {
  DecodeParams p{};
  p.f8 = f8 ? 1 : 0;
  p.q = q; p.gate = gate;
  p.K8 = reinterpret_cast<const int8_t* const*>(K8);
  p.V8 = reinterpret_cast<const int8_t* const*>(V8);
  p.Ks = reinterpret_cast<const __half* const*>(Ks);
  p.Vs = reinterpret_cast<const __half* const*>(Vs);
  p.pos = pos; p.max_len = max_len; p.out = out;
  p.B = B; p.nq = nq; p.nkv = nkv; p.G = nkv > 0 ? nq / nkv : 0;
  p.window = window; p.mode = 0;
  p.scale_log2 = scale * kLog2e; p.softcap = softcap;
  if (B > 0 && (!pos || !out || !K8)) return record_status(ASPIDA_ERR_ARG);
  return run_decode(p, hd, max_kv_len, chunk, ws, ws_bytes, st);
}

// Q8_0 quantiser: the algorithm of k_to_q8 (gpu/fattn_kvhalf.cu:143-152).
// Each 32-value block gets d = max|v| / 127 (stored as fp16) and values
// round-to-nearest(v * (1/d)) clamped to [-127, 127]; an all-zero block gets
// d = 0 and zeros. One thread per block; a warp covers 32 consecutive blocks.
__global__ void quantize_q8_kernel(const float* __restrict__ in, int8_t* __restrict__ q,
                                   __half* __restrict__ sc, long nblk) {
  const long b = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= nblk) return;
  const float4* v4 = reinterpret_cast<const float4*>(in + b * 32);
  float v[32];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float4 t = v4[i];
    v[4 * i] = t.x; v[4 * i + 1] = t.y; v[4 * i + 2] = t.z; v[4 * i + 3] = t.w;
  }
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
  const float d = __fdiv_rn(amax, 127.f);
  const float id = d > 0.f ? __fdiv_rn(1.f, d) : 0.f;
  sc[b] = __float2half_rn(d);
  uint32_t w[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    uint32_t x = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int qi = max(-127, min(127, __float2int_rn(__fmul_rn(v[4 * i + k], id))));
      x |= (uint32_t)(qi & 0xff) << (8 * k);
    }
    w[i] = x;
  }
  uint4* qo = reinterpret_cast<uint4*>(q + b * 32);
  qo[0] = make_uint4(w[0], w[1], w[2], w[3]);
  qo[1] = make_uint4(w[4], w[5], w[6], w[7]);
}

int quantize_q8(const float* in, void* q, void* scales, long nblk, cudaStream_t st) {
  if (nblk < 0 || (nblk > 0 && (!in || !q || !scales))) return record_status(ASPIDA_ERR_ARG);
  if (((uintptr_t)in & 15) || ((uintptr_t)q & 15) || ((uintptr_t)scales & 1))
    return record_status(ASPIDA_ERR_ARG);
  if (nblk == 0) return 0;
  const int threads = 128;
  quantize_q8_kernel<<<(unsigned)((nblk + threads - 1) / threads), threads, 0, st>>>(
      in, static_cast<int8_t*>(q), static_cast<__half*>(scales), nblk);
  ASPIDA_CHECK_LAUNCH();
  return 0;
}

// fp8 (e4m3) quantiser for the 8-bit cache layout of the Q8_0 path: each
// 32-value block gets s = fp16(max|v| / 448) and values e4m3(v / s) rounded
// to nearest even with saturation to +-448 (cvt.rn.satfinite); a block whose
// scale is 0 gets zeros. A value reads back as e4m3 x s. No counterpart in
// the reference (its 8-bit KV mode is Q8_0); same storage geometry.
__global__ void quantize_fp8_kernel(const float* __restrict__ in, uint8_t* __restrict__ q,
                                    __half* __restrict__ sc, long nblk) {
  const long b = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= nblk) return;
  const float4* v4 = reinterpret_cast<const float4*>(in + b * 32);
  float v[32];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float4 t = v4[i];
    v[4 * i] = t.x; v[4 * i + 1] = t.y; v[4 * i + 2] = t.z; v[4 * i + 3] = t.w;
  }
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
  const __half sh = __float2half_rn(__fdiv_rn(amax, 448.f));
  sc[b] = sh;
  const float s = __half2float(sh);
  uint32_t w[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    uint32_t x = 0;
#pragma unroll
    for (int k = 0; k < 4; k += 2) {
      float2 f = make_float2(0.f, 0.f);
      if (s > 0.f) f = make_float2(__fdiv_rn(v[4 * i + k], s), __fdiv_rn(v[4 * i + k + 1], s));
      const __nv_fp8x2_storage_t pr = __nv_cvt_float2_to_fp8x2(f, __NV_SATFINITE, __NV_E4M3);
      x |= (uint32_t)pr << (8 * k);
    }
    w[i] = x;
  }
  uint4* qo = reinterpret_cast<uint4*>(q + b * 32);
  qo[0] = make_uint4(w[0], w[1], w[2], w[3]);
  qo[1] = make_uint4(w[4], w[5], w[6], w[7]);
}

int quantize_fp8(const float* in, void* q, void* scales, long nblk, cudaStream_t st) {
  if (nblk < 0 || (nblk > 0 && (!in || !q || !scales))) return record_status(ASPIDA_ERR_ARG);
  if (((uintptr_t)in & 15) || ((uintptr_t)q & 15) || ((uintptr_t)scales & 1))
    return record_status(ASPIDA_ERR_ARG);
  if (nblk == 0) return 0;
  const int threads = 128;
  quantize_fp8_kernel<<<(unsigned)((nblk + threads - 1) / threads), threads, 0, st>>>(
      in, static_cast<uint8_t*>(q), static_cast<__half*>(scales), nblk);
  ASPIDA_CHECK_LAUNCH();
  return 0;
}

}  // namespace aspida

extern "C" int aspida_attn_decode_q8(const float* q, const float* gate, const void* const* K8,
                                     const void* const* V8, const void* const* K_scales,
                                     const void* const* V_scales, const int* pos,
                                     const int* max_len, float* out, int B, int nq, int nkv,
                                     int hd, float scale, int window, float softcap,
                                     int max_kv_len, int chunk, void* workspace,
                                     size_t workspace_bytes, void* stream) {
  return aspida::decode_q8(q, gate, K8, V8, K_scales, V_scales, pos, max_len, out, B, nq, nkv,
                           hd, scale, window, softcap, max_kv_len, chunk, workspace,
                           workspace_bytes, (cudaStream_t)stream);
}

extern "C" int aspida_attn_decode_fused(
    const float* q_raw, const float* k_raw, const float* v_raw, const float* gate,
    const void* const* K, const void* const* V, const int* pos, const int* max_len, float* out,
    int B, int nq, int nkv, int hd, const float* q_norm, const float* k_norm, float eps, int rd,
    float base, float freq_scale, float m_scale, int yarn_on, float corr_lo, float corr_hi,
    const float* ff, int use_ff, int interleaved, int sec_total, float scale, int window,
    float softcap, int max_kv_len, int chunk, void* workspace, size_t workspace_bytes,
    void* stream) {
  return aspida::decode_fused(q_raw, k_raw, v_raw, gate, K, V, pos, max_len, out, B, nq, nkv, hd,
                              q_norm, k_norm, eps, rd, base, freq_scale, m_scale, yarn_on,
                              corr_lo, corr_hi, ff, use_ff, interleaved, sec_total, scale, window,
                              softcap, max_kv_len, chunk, workspace, workspace_bytes,
                              (cudaStream_t)stream);
}

extern "C" int aspida_attn_quantize_q8(const float* in, void* q, void* scales, long long nblk,
                                       void* stream) {
  return aspida::quantize_q8(in, q, scales, (long)nblk, (cudaStream_t)stream);
}

extern "C" int aspida_attn_quantize_fp8(const float* in, void* q, void* scales, long long nblk,
                                        void* stream) {
  return aspida::quantize_fp8(in, q, scales, (long)nblk, (cudaStream_t)stream);
}

extern "C" int aspida_attn_decode_fp8(const float* q, const float* gate, const void* const* K8,
                                      const void* const* V8, const void* const* K_scales,
                                      const void* const* V_scales, const int* pos,
                                      const int* max_len, float* out, int B, int nq, int nkv,
                                      int hd, float scale, int window, float softcap,
                                      int max_kv_len, int chunk, void* workspace,
                                      size_t workspace_bytes, void* stream) {
  return aspida::decode_q8(q, gate, K8, V8, K_scales, V_scales, pos, max_len, out, B, nq, nkv,
                           hd, scale, window, softcap, max_kv_len, chunk, workspace,
                           workspace_bytes, (cudaStream_t)stream, true);
}

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

extern "C" int aspida_attn_decode_paged(const float* q, const float* gate, const void* K_pool,
                                        const void* V_pool, const int* block_table,
                                        int max_blocks, int block_size, const int* pos,
                                        float* out, int B, int nq, int nkv, int hd, float scale,
                                        int window, float softcap, int max_kv_len, int chunk,
                                        void* workspace, size_t workspace_bytes, void* stream) {
  return aspida::decode_paged(q, gate, K_pool, V_pool, block_table, max_blocks, block_size, pos,
                              out, B, nq, nkv, hd, scale, window, softcap, max_kv_len, chunk,
                              workspace, workspace_bytes, (cudaStream_t)stream);
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
