// prep.cu — the pre-attention step: per-head RMSNorm (optional), partial
// RoPE, and the fp16 K/V append for P consecutive tokens.
//
// Arithmetic follows LLM_RoPE.Apply_Sections (src/llm/llm_rope.adb:84-200) and
// the shim's k_fattn_prep_chunk (gpu/gpu_matvec.cu:3235-3292), which run one
// thread per element with a per-thread O(hd) norm sum; here one warp owns a
// head row (warp-reduced norm, one angle per rotated pair): theta =
// pos/base^(2i/rd) (x freq_scale, YaRN blend, / ff[i]), cos/sin x m_scale,
// NeoX split-half or interleaved pairs, pairs i >= sec_total at position 0.
// Precise powf/cosf/sinf (no fast-math) keep the angles within an ulp or two
// of the CPU oracle's libm.
#include "common.cuh"

namespace aspida {
namespace {

constexpr int kPrepWarps = 8;   // rows per 256-thread block

struct PrepArgs {
  const float* q;
  const float* k;
  const float* v;
  const float* q_norm;
  const float* k_norm;
  void* q_out;
  __half* Kc;
  __half* Vc;
  __half* const* Ktab;      // decode lanes: per-row caches, or null
  __half* const* Vtab;
  const int* max_len_tab;   // decode lanes: per-row bounds, or null
  const int* pos_tab;       // decode lanes / paged batch: per-row positions, or null
  const int* btab;          // paged pools: block tables, or null
  RopeArgs rope;
  float eps;
  long rows;                // P * (nq + nkv)
  int nq, nkv, hd, q_out_fp16, max_len, pos_start, max_blocks, block_size;
};

// One warp per (token, head) row; 8 rows per block. Row (t, h < nq) is query
// head h of token t; row (t, nq + j) is kv head j (K normed and rotated, V
// copied). Token t is either token t of one sequence (positions pos_start +
// t, one cache) or lane t of a decode batch (its own cache, position, bound).
// The norm's sum of squares is a warp reduction (warp_norm_row), the angle is
// evaluated once per pair (rope_pair), and every store is coalesced.
__global__ void __launch_bounds__(kPrepWarps * 32) prep_kernel(const PrepArgs a) {
  extern __shared__ float sh_all[];               // [kPrepWarps][hd]
  // a decode launched as this kernel's programmatic dependent may start now;
  // it waits for this grid before reading anything it writes
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long R = (long)blockIdx.x * kPrepWarps + warp;
  if (R >= a.rows) return;
  const int nh = a.nq + a.nkv;
  const int t = (int)(R / nh), head = (int)(R % nh), hd = a.hd;
  float* sh = sh_all + warp * hd;
  const int pos = a.pos_tab ? a.pos_tab[t] : a.pos_start + t;
  const bool is_q = head < a.nq;
  const int kvh = head - a.nq;
  const long kvd = (long)a.nkv * hd, att = (long)a.nq * hd;
  __half* Kc = a.Ktab ? a.Ktab[t] : a.Kc;
  __half* Vc = a.Vtab ? a.Vtab[t] : a.Vc;
  const int max_len = a.max_len_tab ? a.max_len_tab[t] : a.max_len;
  if (!is_q && (pos < 0 || pos >= max_len)) return;  // never write past the cache
  // cache row of this position: itself, or (paged) its block's pool row
  long crow = pos;
  if (a.btab && !is_q) {
    const int* bt = a.btab + (a.pos_tab ? (long)t * a.max_blocks : 0);
    crow = (long)bt[pos / a.block_size] * a.block_size + pos % a.block_size;
  }
  const float* x = is_q ? a.q + t * att + (long)head * hd : a.k + t * kvd + (long)kvh * hd;
  if (!is_q) {
    const float* vr = a.v + t * kvd + (long)kvh * hd;
    __half* vd = Vc + crow * kvd + (long)kvh * hd;
    if (hd <= 256) {
      float t[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) t[j] = lane + 32 * j < hd ? vr[lane + 32 * j] : 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (lane + 32 * j < hd) vd[lane + 32 * j] = __float2half_rn(t[j]);
    } else {
      for (int d = lane; d < hd; d += 32) vd[d] = __float2half_rn(vr[d]);
    }
  }
  warp_norm_row(x, is_q ? a.q_norm : a.k_norm, a.eps, hd, sh, lane);
  float* qf = nullptr;
  __half* qh = nullptr;
  __half* kd = nullptr;
  if (is_q) {
    if (a.q_out_fp16) qh = static_cast<__half*>(a.q_out) + t * att + (long)head * hd;
    else qf = static_cast<float*>(a.q_out) + t * att + (long)head * hd;
  } else {
    kd = Kc + crow * kvd + (long)kvh * hd;
  }
  auto put = [&](int d, float o) {
    if (qf) qf[d] = o;
    else if (qh) qh[d] = __float2half_rn(o);
    else kd[d] = __float2half_rn(o);
  };
  for (int i = lane; i < a.rope.rd / 2; i += 32) {
    int d1, d2;
    float o1, o2;
    rope_pair(sh, i, pos, a.rope, d1, d2, o1, o2);
    put(d1, o1);
    put(d2, o2);
  }
  for (int d = a.rope.rd + lane; d < hd; d += 32) put(d, sh[d]);
}

int launch(const PrepArgs& a, cudaStream_t st) {
  if (a.rows <= 0) return 0;
  const long blocks = (a.rows + kPrepWarps - 1) / kPrepWarps;
  if (blocks >= (1L << 31)) return record_status(ASPIDA_ERR_UNSUPPORTED);
  prep_kernel<<<(unsigned)blocks, kPrepWarps * 32, kPrepWarps * a.hd * sizeof(float), st>>>(a);
  ASPIDA_CHECK_LAUNCH();
  return 0;
}

RopeArgs rope_args(int rd, float base, float freq_scale, float m_scale, int yarn_on,
                   float corr_lo, float corr_hi, const float* ff, int use_ff, int interleaved,
                   int sec_total) {
  RopeArgs r;
  r.ff = ff; r.base = base; r.freq_scale = freq_scale; r.m_scale = m_scale;
  r.corr_lo = corr_lo; r.corr_hi = corr_hi; r.rd = rd; r.yarn_on = yarn_on;
  r.use_ff = use_ff; r.interleaved = interleaved; r.sec_total = sec_total;
  return r;
}

}  // namespace

int launch_prep(const float* q, const float* k, const float* v, int P, int nq, int nkv, int hd,
                const float* q_norm, const float* k_norm, float eps, void* q_out, int q_out_fp16,
                void* K, void* V, int max_len, int pos_start, int rd, float base,
                float freq_scale, float m_scale, int yarn_on, float corr_lo, float corr_hi,
                const float* ff, int use_ff, int interleaved, int sec_total, cudaStream_t st) {
  if (P <= 0) return 0;
  if (!q || !k || !v || !q_out || !K || !V || nq <= 0 || nkv <= 0 || nq % nkv != 0 || hd <= 0 ||
      hd > 1024 || rd < 0 || rd > hd || (rd & 1) || (use_ff && !ff) || max_len <= 0 ||
      pos_start < 0 || pos_start + P > max_len)
    return record_status(ASPIDA_ERR_ARG);
  PrepArgs a{};
  a.q = q; a.k = k; a.v = v; a.q_norm = q_norm; a.k_norm = k_norm; a.q_out = q_out;
  a.Kc = (__half*)K; a.Vc = (__half*)V; a.eps = eps;
  a.rope = rope_args(rd, base, freq_scale, m_scale, yarn_on, corr_lo, corr_hi, ff, use_ff,
                     interleaved, sec_total);
  a.rows = (long)P * (nq + nkv);
  a.nq = nq; a.nkv = nkv; a.hd = hd; a.q_out_fp16 = q_out_fp16; a.max_len = max_len;
  a.pos_start = pos_start; a.block_size = 1;
  return launch(a, st);
}

// Batched decode form: lane b appends at pos[b] into its own cache.
int launch_prep_lanes(const float* q, const float* k, const float* v, int B, int nq, int nkv,
                      int hd, void* q_out, __half* const* Ktab, __half* const* Vtab,
                      const int* pos, const int* max_len, int rd, float base, int interleaved,
                      cudaStream_t st) {
  if (B <= 0) return 0;
  if (!q || !k || !v || !q_out || !Ktab || !Vtab || !pos || !max_len || nq <= 0 || nkv <= 0 ||
      hd <= 0 || hd > 1024 || rd < 0 || rd > hd || (rd & 1))
    return record_status(ASPIDA_ERR_ARG);
  PrepArgs a{};
  a.q = q; a.k = k; a.v = v; a.q_out = q_out;
  a.Ktab = Ktab; a.Vtab = Vtab; a.max_len_tab = max_len; a.pos_tab = pos;
  a.rope = rope_args(rd, base, 1.0f, 1.0f, 0, 0.f, 0.f, nullptr, 0, interleaved, rd / 2);
  a.rows = (long)B * (nq + nkv);
  a.nq = nq; a.nkv = nkv; a.hd = hd; a.block_size = 1;
  return launch(a, st);
}

// Paged form: K/V are block pools; row t appends at pos[t] through block-table
// row t (pos != null, a decode batch) or at pos_start + t through one table.
int launch_prep_paged(const float* q, const float* k, const float* v, int P, int nq, int nkv,
                      int hd, const float* q_norm, const float* k_norm, float eps, void* q_out,
                      int q_out_fp16, void* K_pool, void* V_pool, const int* block_table,
                      int max_blocks, int block_size, int pos_start, const int* pos, int rd,
                      float base, float freq_scale, float m_scale, int yarn_on, float corr_lo,
                      float corr_hi, const float* ff, int use_ff, int interleaved, int sec_total,
                      cudaStream_t st) {
  if (P <= 0) return 0;
  if (!q || !k || !v || !q_out || !K_pool || !V_pool || !block_table || nq <= 0 || nkv <= 0 ||
      nq % nkv != 0 || hd <= 0 || hd > 1024 || rd < 0 || rd > hd || (rd & 1) ||
      (use_ff && !ff) || max_blocks <= 0 || block_size <= 0 ||
      (long)max_blocks * block_size >= (1L << 31) ||
      (!pos && (pos_start < 0 || (long)pos_start + P > (long)max_blocks * block_size)))
    return record_status(ASPIDA_ERR_ARG);
  PrepArgs a{};
  a.q = q; a.k = k; a.v = v; a.q_norm = q_norm; a.k_norm = k_norm; a.q_out = q_out;
  a.Kc = (__half*)K_pool; a.Vc = (__half*)V_pool; a.eps = eps;
  a.rope = rope_args(rd, base, freq_scale, m_scale, yarn_on, corr_lo, corr_hi, ff, use_ff,
                     interleaved, sec_total);
  a.rows = (long)P * (nq + nkv);
  a.nq = nq; a.nkv = nkv; a.hd = hd; a.q_out_fp16 = q_out_fp16;
  a.max_len = max_blocks * block_size; a.pos_start = pos_start; a.pos_tab = pos;
  a.btab = block_table; a.max_blocks = max_blocks; a.block_size = block_size;
  return launch(a, st);
}

}  // namespace aspida

extern "C" int aspida_attn_prep_paged(const float* q, const float* k, const float* v, int P,
                                      int nq, int nkv, int hd, const float* q_norm,
                                      const float* k_norm, float eps, void* q_out,
                                      int q_out_fp16, void* K_pool, void* V_pool,
                                      const int* block_table, int max_blocks, int block_size,
                                      int pos_start, const int* pos, int rd, float base,
                                      float freq_scale, float m_scale, int yarn_on,
                                      float corr_lo, float corr_hi, const float* ff, int use_ff,
                                      int interleaved, int sec_total, void* stream) {
  return aspida::launch_prep_paged(q, k, v, P, nq, nkv, hd, q_norm, k_norm, eps, q_out,
                                   q_out_fp16, K_pool, V_pool, block_table, max_blocks,
                                   block_size, pos_start, pos, rd, base, freq_scale, m_scale,
                                   yarn_on, corr_lo, corr_hi, ff, use_ff, interleaved, sec_total,
                                   (cudaStream_t)stream);
}

extern "C" int aspida_attn_prep(const float* q, const float* k, const float* v, int P, int nq,
                                int nkv, int hd, const float* q_norm, const float* k_norm,
                                float eps, void* q_out, int q_out_fp16, void* K, void* V,
                                int max_len, int pos_start, int rd, float base, float freq_scale,
                                float m_scale, int yarn_on, float corr_lo, float corr_hi,
                                const float* ff, int use_ff, int interleaved, int sec_total,
                                void* stream) {
  return aspida::launch_prep(q, k, v, P, nq, nkv, hd, q_norm, k_norm, eps, q_out, q_out_fp16, K,
                             V, max_len, pos_start, rd, base, freq_scale, m_scale, yarn_on,
                             corr_lo, corr_hi, ff, use_ff, interleaved, sec_total,
                             (cudaStream_t)stream);
}
