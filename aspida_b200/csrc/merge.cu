// merge.cu — log-sum-exp merge of S split-KV partials, the cross-GPU step of
// sequence-parallel decode. Same merge as the split-K combine in
// gpu/fattn_sk.cu:84-97: M = max_s m_s; out = sum_s e^{m_s-M} o_s /
// sum_s e^{m_s-M} l_s, partials with m_s = -3.4e38 (empty slices) skipped,
// then x sigmoid(gate) when a gate is given.
#include "common.cuh"

namespace aspida {
namespace {

// Partial s of m / l starts ml_stride floats after partial s-1; of o,
// o_stride floats after.
__global__ void merge_kernel(const float* __restrict__ m, const float* __restrict__ l,
                             const float* __restrict__ o, const float* __restrict__ gate,
                             float* __restrict__ out, int S, int rows, int hd, long ml_stride,
                             long o_stride) {
  const int r = blockIdx.x;
  for (int d = threadIdx.x; d < hd; d += blockDim.x) {
    float M = -3.402823466e38f;
    for (int s = 0; s < S; ++s) M = fmaxf(M, m[s * ml_stride + r]);
    float acc = 0.f, L = 0.f;
    for (int s = 0; s < S; ++s) {
      const float ms = m[s * ml_stride + r];
      if (ms < -3.0e38f) continue;
      const float w = expf(ms - M);
      acc += w * o[s * o_stride + (long)r * hd + d];
      L += w * l[s * ml_stride + r];
    }
    float v = L > 0.f ? acc / L : 0.f;
    const long oi = (long)r * hd + d;
    if (gate) v *= 1.f / (1.f + expf(-gate[oi]));
    out[oi] = v;
  }
}

}  // namespace

int merge(const float* m, const float* l, const float* o, const float* gate, float* out, int S,
          int rows, int hd, long ml_stride, long o_stride, cudaStream_t st) {
  if (rows <= 0) return 0;
  if (!m || !l || !o || !out || S <= 0 || hd <= 0 || ml_stride < 0 || o_stride < 0)
    return record_status(ASPIDA_ERR_ARG);
  const int threads = hd >= 256 ? 256 : ((hd + 31) / 32) * 32;
  merge_kernel<<<rows, threads, 0, st>>>(m, l, o, gate, out, S, rows, hd, ml_stride, o_stride);
  ASPIDA_CHECK_LAUNCH();
  return 0;
}

}  // namespace aspida

extern "C" int aspida_attn_merge(const float* m, const float* l, const float* o,
                                 const float* gate, float* out, int S, int rows, int hd,
                                 void* stream) {
  return aspida::merge(m, l, o, gate, out, S, rows, hd, rows, (long)rows * hd,
                       (cudaStream_t)stream);
}

extern "C" int aspida_attn_merge_strided(const float* m, const float* l, const float* o,
                                         const float* gate, float* out, int S, int rows, int hd,
                                         long part_stride, void* stream) {
  return aspida::merge(m, l, o, gate, out, S, rows, hd, part_stride, part_stride,
                       (cudaStream_t)stream);
}
