// attn_oracle.cpp — CPU restatement of Aspida's Ada attention loops.
//
// TEST INFRASTRUCTURE ONLY. This file is the checker for the CUDA library in
// aspida_b200/csrc: only tests/, __graft_entry__.smoke() and bench.py's CPU
// baseline legs load it. The product path never calls into it.
//
// The reference engine's CPU attention is Ada (GNAT), which cannot be compiled
// in this environment, so the loops are restated here in C++ with IEEE binary32
// `float`, the same loop order and the same libm elementary functions (GNAT's
// Ada.Numerics.Elementary_Functions defers to libm). Each function cites the
// Ada source it follows (paths relative to the reference project root).
//
// Build: oracle/Makefile  (-O3, no -ffast-math: the Ada build uses none).

#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>
#include <atomic>
#include <algorithm>

namespace {

// Ada `Float'First` — the initial running max in every attention loop.
constexpr float kFloatFirst = -3.40282347e38f;

// Sigmoid as in src/llm/llm_fullattn.adb:32.
inline float ada_sigmoid(float x) { return 1.0f / (1.0f + std::exp(-x)); }

// Attention-logit softcap c*tanh(s/c). The reference has no attention softcap
// (its only softcap is on final logits, src/llm/llm_gemma.adb:636-645); this is
// the textbook definition, applied after the scale and before the running max.
inline float softcap_apply(float s, float cap) {
  return cap > 0.0f ? cap * std::tanh(s / cap) : s;
}

// One query head over keys [lo, pos] — the body of Head_Op.Execute in
// src/llm/llm_llama.adb:871-898 (Llama, lo = 0), of the head loop in
// src/llm/llm_gemma.adb:541-571 (Gemma, lo = max(0, pos-win+1)), and of
// step 2 in src/llm/llm_fullattn.adb:402-444 (Qwen gated, then x sigmoid(g)).
//   pass 1: ascending-J dot, Scr(S) = Dp*AScale, running max
//   pass 2: Scr(S) = Exp(Scr(S)-Mx), ascending Den
//   pass 3: for each J, ascending-over-S Acc += (Scr(S)/Den) * V(S)(J)
// K/V rows are addressed as base + s*row_stride + kvh*hd.
void head_attend(const float* q, const float* K, const float* V, long row_stride,
                 int kvh, int hd, int lo, int pos, float scale, float softcap,
                 const float* gate, float* out, std::vector<float>& scr) {
  const int n = pos - lo + 1;
  if (n <= 0) {
    for (int j = 0; j < hd; ++j) out[j] = 0.0f;
    return;
  }
  scr.resize(n);
  float mx = kFloatFirst;
  for (int s = lo; s <= pos; ++s) {
    const float* k = K + (long)s * row_stride + (long)kvh * hd;
    float dp = 0.0f;
    for (int j = 0; j < hd; ++j) dp = dp + q[j] * k[j];
    float sc = softcap_apply(dp * scale, softcap);
    scr[s - lo] = sc;
    mx = std::max(mx, sc);
  }
  float den = 0.0f;
  for (int s = 0; s < n; ++s) {
    scr[s] = std::exp(scr[s] - mx);
    den = den + scr[s];
  }
  for (int j = 0; j < hd; ++j) {
    float acc = 0.0f;
    for (int s = lo; s <= pos; ++s)
      acc = acc + (scr[s - lo] / den) * V[(long)s * row_stride + (long)kvh * hd + j];
    out[j] = gate ? acc * ada_sigmoid(gate[j]) : acc;
  }
}

// Fan (job) ranges out over `threads` workers, as LLM_Pool.Run does with
// Number_Of_CPUs workers (src/llm/llm_pool.adb:12-15). Jobs are independent.
template <class F>
void parallel_for(int njobs, int threads, F&& f) {
  if (threads <= 1 || njobs <= 1) {
    for (int i = 0; i < njobs; ++i) f(i);
    return;
  }
  std::atomic<int> next{0};
  std::vector<std::thread> pool;
  int nt = std::min(threads, njobs);
  for (int t = 0; t < nt; ++t)
    pool.emplace_back([&] {
      for (int i = next.fetch_add(1); i < njobs; i = next.fetch_add(1)) f(i);
    });
  for (auto& th : pool) th.join();
}

}  // namespace

extern "C" {

int oracle_abi_version(void) { return 1; }

// LLM_RMSNorm.Forward (src/llm/llm_rmsnorm.adb:12-30): ascending sum of
// squares, Rms = Sqrt(Sum_Sq/N + Eps), out = x / Rms * w.
void oracle_rmsnorm(const float* x, const float* w, float* out, int n, float eps) {
  float ss = 0.0f;
  for (int i = 0; i < n; ++i) ss = ss + x[i] * x[i];
  float rms = std::sqrt(ss / (float)n + eps);
  for (int i = 0; i < n; ++i) out[i] = x[i] / rms * w[i];
}

// LLM_RoPE.Apply_Sections (src/llm/llm_rope.adb:84-200).
//   sections[4]: widths in pairs; sec_pos[4]: position per section.
//   A pair beyond every non-empty section uses position 0 (identity).
//   theta_extrap = eff_pos / base^(2i/dim); YaRN blend when yarn_on;
//   theta /= ff[i] when use_ff; cos/sin scaled by m_scale;
//   NeoX split-half pairs (i, i+dim/2) or interleaved (2i, 2i+1).
void oracle_rope_apply_sections(const float* x, float* out, int dim, float base,
                                const int* sections, const int* sec_pos,
                                int use_ff, const float* ff, int interleaved,
                                float freq_scale, int yarn_on, float corr_lo,
                                float corr_hi, float m_scale) {
  const int half = dim / 2;
  for (int i = 0; i < half; ++i) {
    int sec = -1, cum = 0;
    for (int s = 0; s < 4; ++s) {
      int w = sections[s];
      if (w <= 0) continue;
      if (i < cum + w) { sec = s; break; }
      cum += w;
    }
    int eff_pos = (sec >= 0) ? sec_pos[sec] : 0;
    float extrap = (float)eff_pos / std::pow(base, (float)(2 * i) / (float)dim);
    float theta;
    if (yarn_on) {
      float interp = freq_scale * extrap;
      float y = ((float)i - corr_lo) / std::max(0.001f, corr_hi - corr_lo);
      float ramp = 1.0f - std::min(1.0f, std::max(0.0f, y));
      theta = interp * (1.0f - ramp) + extrap * ramp;
    } else {
      theta = extrap * freq_scale;
    }
    if (use_ff) theta = theta / ff[i];
    float c = std::cos(theta) * m_scale;
    float s = std::sin(theta) * m_scale;
    if (interleaved) {
      float x1 = x[2 * i], x2 = x[2 * i + 1];
      out[2 * i] = x1 * c - x2 * s;
      out[2 * i + 1] = x2 * c + x1 * s;
    } else {
      float x1 = x[i], x2 = x[i + half];
      out[i] = x1 * c - x2 * s;
      out[i + half] = x2 * c + x1 * s;
    }
  }
}

// Norm_Rope (src/llm/llm_fullattn.adb:55-86) for one head: optional RMSNorm
// (norm_w == nullptr skips it, as Llama has no QK-norm, llm_llama.adb:826),
// then RoPE on the first rd dims with all sections at `pos` when
// sec_total >= rd/2, or the reference's section walk otherwise (pairs
// i >= sec_total get position 0 — the shim mirrors this with sec_total,
// gpu/gpu_matvec.cu:1493). Dims rd..hd-1 pass through.
void oracle_norm_rope(const float* x, const float* norm_w, float eps, float* out,
                      int hd, int rd, int pos, float base, int sec_total,
                      int use_ff, const float* ff, int interleaved,
                      float freq_scale, int yarn_on, float corr_lo,
                      float corr_hi, float m_scale) {
  std::vector<float> nrm(hd), rot(rd);
  if (norm_w) oracle_rmsnorm(x, norm_w, nrm.data(), hd, eps);
  else std::memcpy(nrm.data(), x, sizeof(float) * hd);
  int sections[4] = {sec_total, 0, 0, 0};
  int sp[4] = {pos, pos, pos, pos};
  oracle_rope_apply_sections(nrm.data(), rot.data(), rd, base, sections, sp, use_ff,
                             ff, interleaved, freq_scale, yarn_on, corr_lo, corr_hi,
                             m_scale);
  for (int i = 0; i < rd; ++i) out[i] = rot[i];
  for (int i = rd; i < hd; ++i) out[i] = nrm[i];
}

// Batched decode attention: B sequences, each with its own K/V cache
// (row stride kvd = nkv*hd floats) and its own 0-based query position pos[b]
// (keys 0..pos[b] are attended, minus the window). One (sequence x head) job
// per worker call, as LLM_Llama.Forward_Batch fans (lane x head) jobs
// (src/llm/llm_llama.adb:1089-1138). window <= 0 means none.
//   q, gate, out: [B][nq*hd]; gate may be null.
void oracle_decode_batch(const float* q, const float* gate,
                         const float* const* K, const float* const* V,
                         const int* pos, float* out, int B, int nq, int nkv, int hd,
                         float scale, int window, float softcap, int threads) {
  const int rep = nq / nkv;
  const long kvd = (long)nkv * hd, att = (long)nq * hd;
  parallel_for(B * nq, threads, [&](int job) {
    int b = job / nq, h = job % nq;
    int p = pos[b];
    int lo = window > 0 ? std::max(0, p - window + 1) : 0;
    thread_local std::vector<float> scr;
    head_attend(q + b * att + (long)h * hd, K[b], V[b], kvd, h / rep, hd, lo, p, scale,
                softcap, gate ? gate + b * att + (long)h * hd : nullptr,
                out + b * att + (long)h * hd, scr);
  });
}

// Causal prefill of P tokens at positions pos_start..pos_start+P-1 against
// one K/V cache holding rows 0..pos_start+P-1. The reference CPU path has no
// batched prefill: each prompt token goes through the single-token loop
// (LLM_Gemma.Forward_Logits, src/llm/llm_gemma.adb:668-713; LLM_FullAttn.Forward
// step 2 iterates T with keys 1..T, src/llm/llm_fullattn.adb:182-216), so this
// is the decode loop per token. Jobs are (token x head).
//   q, gate, out: [P][nq*hd]; K, V: [rows][nkv*hd].
//   rows_subset/nrows (optional): only those token indices are computed.
void oracle_prefill(const float* q, const float* gate, const float* K, const float* V,
                    float* out, int P, int pos_start, int nq, int nkv, int hd,
                    float scale, int window, float softcap, const int* rows_subset,
                    int nrows, int threads) {
  const int rep = nq / nkv;
  const long kvd = (long)nkv * hd, att = (long)nq * hd;
  const int nt = rows_subset ? nrows : P;
  parallel_for(nt * nq, threads, [&](int job) {
    int t = rows_subset ? rows_subset[job / nq] : job / nq;
    int h = job % nq;
    int p = pos_start + t;
    int lo = window > 0 ? std::max(0, p - window + 1) : 0;
    thread_local std::vector<float> scr;
    head_attend(q + t * att + (long)h * hd, K, V, kvd, h / rep, hd, lo, p, scale,
                softcap, gate ? gate + t * att + (long)h * hd : nullptr,
                out + t * att + (long)h * hd, scr);
  });
}

// Log-sum-exp merge of S partial (m, l, o) triples per row — the combine of
// flash-decoding split-K in gpu/fattn_sk.cu:84-97:
//   M = max_s m_s;  O = sum_s e^{m_s-M} o_s / sum_s e^{m_s-M} l_s
// (partials with m_s = -inf-like are skipped), then x sigmoid(gate) if given.
//   m, l: [S][rows]; o: [S][rows][hd] (unnormalised); out: [rows][hd].
void oracle_merge(const float* m, const float* l, const float* o, const float* gate,
                  float* out, int S, int rows, int hd) {
  for (int r = 0; r < rows; ++r) {
    float M = kFloatFirst;
    for (int s = 0; s < S; ++s) M = std::max(M, m[(long)s * rows + r]);
    for (int d = 0; d < hd; ++d) {
      float acc = 0.0f, L = 0.0f;
      for (int s = 0; s < S; ++s) {
        float ms = m[(long)s * rows + r];
        if (ms < -3.0e38f) continue;
        float w = std::exp(ms - M);
        acc += w * o[((long)s * rows + r) * hd + d];
        L += w * l[(long)s * rows + r];
      }
      float v = L > 0.0f ? acc / L : 0.0f;
      out[(long)r * hd + d] = gate ? v * ada_sigmoid(gate[(long)r * hd + d]) : v;
    }
  }
}

}  // extern "C"
