// prep.cu — the pre-attention step: per-head RMSNorm (optional), partial
// RoPE, and the fp16 K/V append for P consecutive tokens.
//
// Arithmetic follows LLM_RoPE.Apply_Sections (src/llm/llm_rope.adb:84-200) and
// the shim's k_fattn_prep_chunk (gpu/gpu_matvec.cu:3235-3292): theta =
// pos/base^(2i/rd) (x freq_scale, YaRN blend, / ff[i]), cos/sin x m_scale,
// NeoX split-half or interleaved pairs, pairs i >= sec_total at position 0.
// Precise powf/cosf/sinf (no fast-math) keep the angles within an ulp or two
// of the CPU oracle's libm.
#include "common.cuh"

namespace aspida {
namespace {

// grid (P, nq + nkv), block hd. Block (t, h<nq) handles query head h of token
// t; block (t, nq + j) handles kv head j (K rotated, V copied).
__global__ void prep_kernel(const float* __restrict__ q, const float* __restrict__ k,
                            const float* __restrict__ v, int nq, int nkv, int hd,
                            const float* __restrict__ q_norm, const float* __restrict__ k_norm,
                            float eps, void* __restrict__ q_out, int q_out_fp16,
                            __half* Kc, __half* Vc, __half* const* Ktab, __half* const* Vtab,
                            int max_len, const int* max_len_tab, int pos_start,
                            const int* pos_tab, int rd, float base, float freq_scale, float m_scale,
                            int yarn_on, float corr_lo, float corr_hi, const float* __restrict__ ff,
                            int use_ff, int interleaved, int sec_total,
                            const int* __restrict__ btab, int max_blocks, int block_size) {
  extern __shared__ float sh[];  // [hd]
  const int t = blockIdx.x, head = blockIdx.y, d = threadIdx.x;
  // Row t is either token t of one sequence (consecutive positions, one
  // cache) or lane t of a decode batch (its own cache, position, bound).
  const int pos = pos_tab ? pos_tab[t] : pos_start + t;
  if (Ktab) { Kc = Ktab[t]; Vc = Vtab[t]; }
  if (max_len_tab) max_len = max_len_tab[t];
  const bool is_q = head < nq;
  const int kvh = head - nq;
  const long kvd = (long)nkv * hd, att = (long)nq * hd;
  if (!is_q && (pos < 0 || pos >= max_len)) return;  // never write past the cache
  // cache row of this position: itself, or (paged) its block's pool row
  long row = pos;
  if (btab && !is_q) {
    const int* bt = btab + (pos_tab ? (long)t * max_blocks : 0);
    row = (long)bt[pos / block_size] * block_size + pos % block_size;
  }

  float x = is_q ? q[t * att + (long)head * hd + d] : k[t * kvd + (long)kvh * hd + d];
  if (!is_q) Vc[row * kvd + (long)kvh * hd + d] = __float2half_rn(v[t * kvd + (long)kvh * hd + d]);

  const float* nw = is_q ? q_norm : k_norm;
  sh[d] = x;
  __syncthreads();
  float nv = x;
  if (nw) {
    float ss = 0.0f;  // ascending sum, the CPU order
    for (int i = 0; i < hd; ++i) ss = __fadd_rn(ss, __fmul_rn(sh[i], sh[i]));
    float rms = sqrtf(ss / (float)hd + eps);
    nv = __fmul_rn(x / rms, nw[d]);
    __syncthreads();
    sh[d] = nv;
    __syncthreads();
  }
  float o = nv;
  if (d < rd) {
    const int half = rd / 2;
    int i, other;
    bool first;
    if (interleaved) {
      i = d >> 1;
      first = (d & 1) == 0;
      other = first ? d + 1 : d - 1;
    } else if (d < half) {
      i = d;
      first = true;
      other = d + half;
    } else {
      i = d - half;
      first = false;
      other = d - half;
    }
    int pos_eff = (i < sec_total) ? pos : 0;
    float th = rope_angle(i, pos_eff, rd, base, freq_scale, yarn_on, corr_lo, corr_hi, ff, use_ff);
    float c = __fmul_rn(cosf(th), m_scale), s = __fmul_rn(sinf(th), m_scale);
    float x1 = first ? nv : sh[other];
    float x2 = first ? sh[other] : nv;
    o = first ? __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s))
              : __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
  }
  if (is_q) {
    long idx = t * att + (long)head * hd + d;
    if (q_out_fp16) static_cast<__half*>(q_out)[idx] = __float2half_rn(o);
    else static_cast<float*>(q_out)[idx] = o;
  } else {
    Kc[row * kvd + (long)kvh * hd + d] = __float2half_rn(o);
  }
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
  dim3 grid(P, nq + nkv);
  prep_kernel<<<grid, hd, hd * sizeof(float), st>>>(
      q, k, v, nq, nkv, hd, q_norm, k_norm, eps, q_out, q_out_fp16, (__half*)K, (__half*)V,
      nullptr, nullptr, max_len, nullptr, pos_start, nullptr, rd, base, freq_scale, m_scale,
      yarn_on, corr_lo, corr_hi, ff, use_ff, interleaved, sec_total, nullptr, 0, 1);
  ASPIDA_CHECK_LAUNCH();
  return 0;
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
  prep_kernel<<<dim3(B, nq + nkv), hd, hd * sizeof(float), st>>>(
      q, k, v, nq, nkv, hd, nullptr, nullptr, 0.f, q_out, 0, nullptr, nullptr, Ktab, Vtab, 0,
      max_len, 0, pos, rd, base, 1.0f, 1.0f, 0, 0.f, 0.f, nullptr, 0, interleaved, rd / 2,
      nullptr, 0, 1);
  ASPIDA_CHECK_LAUNCH();
  return 0;
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
  prep_kernel<<<dim3(P, nq + nkv), hd, hd * sizeof(float), st>>>(
      q, k, v, nq, nkv, hd, q_norm, k_norm, eps, q_out, q_out_fp16, (__half*)K_pool,
      (__half*)V_pool, nullptr, nullptr, max_blocks * block_size, nullptr, pos_start, pos, rd,
      base, freq_scale, m_scale, yarn_on, corr_lo, corr_hi, ff, use_ff, interleaved, sec_total,
      block_table, max_blocks, block_size);
  ASPIDA_CHECK_LAUNCH();
  return 0;
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
