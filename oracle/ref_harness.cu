// ref_harness.cu — TEST INFRASTRUCTURE ONLY. Runs the reference's own fp32
// attention/RoPE kernels on caller-supplied inputs so their outputs can pin
// the CPU oracle. The reference sources are compiled where they lie (include
// path = the reference project root, given by oracle/Makefile.ref); nothing
// from them is copied here. Their `main`s are renamed away.
//
//   k_attn               gpu/experiments/phase1/ops.cu:39  (two-pass GQA decode)
//   k_rope               gpu/experiments/phase1/ops.cu:18  (NeoX RoPE, freq factors)
//   k_fattn_attend_chunk gpu/fattn_bench.cu:72             (gated causal chunk,
//                                                            the shim's fp32 oracle)
//
// Usage: ref_harness {attn|rope|chunk} <in.bin> <out.bin>
//   attn : i32 nh,nkv,hd,seq; f32 scale; Q[nh*hd]; K,V[seq*nkv*hd] -> O[nh*hd]
//   rope : i32 dim,pos; f32 base; x[dim]; ff[dim/2]                 -> y[dim]
//   chunk: i32 nq,nkv,hd,P,pos_start; q[P*nq*hd]; g[P*nq*hd];
//          K,V[(pos_start+P)*nkv*hd]                                -> out[P*nq*hd]
#define main aspida_ref_phase1_ops_main
#include "gpu/experiments/phase1/ops.cu"
#undef main
#define main aspida_ref_fattn_bench_main
#include "gpu/fattn_bench.cu"
#undef main

#include <cstring>
#include <string>

static std::vector<float> rd_f(FILE* f, size_t n) {
  std::vector<float> v(n);
  if (n && fread(v.data(), 4, n, f) != n) { fprintf(stderr, "short read\n"); exit(3); }
  return v;
}
static int rd_i(FILE* f) { int x; if (fread(&x, 4, 1, f) != 1) exit(3); return x; }
static float* to_dev(const std::vector<float>& h) {
  float* p = nullptr;
  CK(cudaMalloc(&p, (h.size() ? h.size() : 1) * 4));
  if (h.size()) CK(cudaMemcpy(p, h.data(), h.size() * 4, cudaMemcpyHostToDevice));
  return p;
}
static void write_out(const char* path, const float* d, size_t n) {
  std::vector<float> h(n);
  CK(cudaMemcpy(h.data(), d, n * 4, cudaMemcpyDeviceToHost));
  FILE* f = fopen(path, "wb");
  if (!f || fwrite(h.data(), 4, n, f) != n) { fprintf(stderr, "write failed\n"); exit(4); }
  fclose(f);
}

int main(int argc, char** argv) {
  if (argc != 4) { fprintf(stderr, "usage: ref_harness {attn|rope|chunk} in out\n"); return 2; }
  std::string mode = argv[1];
  FILE* f = fopen(argv[2], "rb");
  if (!f) { fprintf(stderr, "open %s\n", argv[2]); return 2; }
  if (mode == "attn") {
    int nh = rd_i(f), nkv = rd_i(f), hd = rd_i(f), seq = rd_i(f);
    float scale; if (fread(&scale, 4, 1, f) != 1) return 3;
    if (nh <= 0 || nh > 1024 || nkv <= 0 || nh % nkv || hd <= 0 || seq <= 0 || seq > 4096) return 5;
    auto Q = rd_f(f, (size_t)nh * hd), K = rd_f(f, (size_t)seq * nkv * hd),
         V = rd_f(f, (size_t)seq * nkv * hd);
    float *dQ = to_dev(Q), *dK = to_dev(K), *dV = to_dev(V), *dO = nullptr;
    CK(cudaMalloc(&dO, (size_t)nh * hd * 4));
    k_attn<<<1, nh>>>(dQ, dK, dV, dO, nh, nkv, hd, seq, scale);
    CK(cudaGetLastError()); CK(cudaDeviceSynchronize());
    write_out(argv[3], dO, (size_t)nh * hd);
  } else if (mode == "rope") {
    int dim = rd_i(f), pos = rd_i(f);
    float base; if (fread(&base, 4, 1, f) != 1) return 3;
    if (dim <= 0 || dim % 2) return 5;
    auto x = rd_f(f, dim), ff = rd_f(f, dim / 2);
    float *dx = to_dev(x), *dff = to_dev(ff), *dy = nullptr;
    CK(cudaMalloc(&dy, (size_t)dim * 4));
    k_rope<<<1, 1>>>(dx, dff, dy, dim, pos, base);
    CK(cudaGetLastError()); CK(cudaDeviceSynchronize());
    write_out(argv[3], dy, dim);
  } else if (mode == "chunk") {
    int nq = rd_i(f), nkv = rd_i(f), hd = rd_i(f), P = rd_i(f), ps = rd_i(f);
    // the kernel's tree reduction needs blockDim = hd, a power of two <= 256
    if (nq <= 0 || nkv <= 0 || nq % nkv || hd <= 0 || hd > 256 || (hd & (hd - 1)) || P <= 0 || ps < 0) return 5;
    size_t att = (size_t)nq * hd, kvd = (size_t)nkv * hd, rows = (size_t)ps + P;
    auto q = rd_f(f, P * att), g = rd_f(f, P * att), K = rd_f(f, rows * kvd), V = rd_f(f, rows * kvd);
    float *dq = to_dev(q), *dg = to_dev(g), *dK = to_dev(K), *dV = to_dev(V), *dO = nullptr;
    CK(cudaMalloc(&dO, P * att * 4));
    k_fattn_attend_chunk<<<P * nq, hd>>>(dq, dg, dK, dV, dO, nq, nkv, hd, (int)kvd, ps);
    CK(cudaGetLastError()); CK(cudaDeviceSynchronize());
    write_out(argv[3], dO, P * att);
  } else {
    return 2;
  }
  fclose(f);
  return 0;
}
