// ref_q8.cu — TEST INFRASTRUCTURE ONLY. Runs the reference's own Q8_0 KV
// kernels on caller-supplied inputs so their outputs can pin the CPU oracle's
// quantiser and the attention over dequantised caches. The reference source
// is compiled where it lies (include path = the reference project root, given
// by oracle/Makefile.ref); nothing from it is copied here. Its `main` is
// renamed away. Separate from ref_harness because both reference files define
// k_fattn_attend_chunk.
//
//   k_to_q8           gpu/fattn_kvhalf.cu:143  (Q8_0 quantiser)
//   k_gqa_kv<2,RQ,2>  gpu/fattn_kvhalf.cu:59   (gated causal GQA over a Q8_0 cache)
//
// Usage: ref_q8 {quant|gqa} <in.bin> <out.bin>
//   quant: i64 nblk; x[nblk*32] f32          -> int8 q[nblk*32], fp16 scales[nblk]
//   gqa  : i32 nq,nkv,hd,P,pos_start; q[P*nq*hd]; g[P*nq*hd];
//          K,V[(pos_start+P)*nkv*hd] f32 (quantised here by k_to_q8)
//                                            -> out[P*nq*hd] f32
#define main aspida_ref_fattn_kvhalf_main
#include "gpu/fattn_kvhalf.cu"
#undef main

#include <cstdint>
#include <string>

static std::vector<float> rd_f(FILE* f, size_t n) {
  std::vector<float> v(n);
  if (n && fread(v.data(), 4, n, f) != n) { fprintf(stderr, "short read\n"); exit(3); }
  return v;
}
static int rd_i(FILE* f) { int x; if (fread(&x, 4, 1, f) != 1) exit(3); return x; }
static void* to_dev(const void* h, size_t bytes) {
  void* p = nullptr;
  CK(cudaMalloc(&p, bytes ? bytes : 4));
  if (bytes) CK(cudaMemcpy(p, h, bytes, cudaMemcpyHostToDevice));
  return p;
}
static void write_dev(FILE* f, const void* d, size_t bytes) {
  std::vector<unsigned char> h(bytes);
  CK(cudaMemcpy(h.data(), d, bytes, cudaMemcpyDeviceToHost));
  if (fwrite(h.data(), 1, bytes, f) != bytes) { fprintf(stderr, "write failed\n"); exit(4); }
}

int main(int argc, char** argv) {
  if (argc != 4) { fprintf(stderr, "usage: ref_q8 {quant|gqa} in out\n"); return 2; }
  std::string mode = argv[1];
  FILE* f = fopen(argv[2], "rb");
  if (!f) { fprintf(stderr, "open %s\n", argv[2]); return 2; }
  FILE* o = fopen(argv[3], "wb");
  if (!o) { fprintf(stderr, "open %s\n", argv[3]); return 2; }
  if (mode == "quant") {
    long long nblk = 0;
    if (fread(&nblk, 8, 1, f) != 1 || nblk <= 0 || nblk > (1 << 22)) return 5;
    auto x = rd_f(f, (size_t)nblk * 32);
    float* dx = (float*)to_dev(x.data(), x.size() * 4);
    signed char* dq = nullptr;
    half* ds = nullptr;
    CK(cudaMalloc(&dq, (size_t)nblk * 32));
    CK(cudaMalloc(&ds, (size_t)nblk * 2));
    k_to_q8<<<(unsigned)((nblk + 255) / 256), 256>>>(dx, dq, ds, (size_t)nblk);
    CK(cudaDeviceSynchronize());
    write_dev(o, dq, (size_t)nblk * 32);
    write_dev(o, ds, (size_t)nblk * 2);
  } else if (mode == "gqa") {
    const int nq = rd_i(f), nkv = rd_i(f), hd = rd_i(f), P = rd_i(f), ps = rd_i(f);
    if (nq <= 0 || nkv <= 0 || nq % nkv || (nq / nkv) % 2 || (hd != 128 && hd != 256) ||
        P <= 0 || P > 4096 || ps < 0 || ps > 65536)
      return 5;
    const int kvd = nkv * hd, att = nq * hd, len = ps + P;
    auto q = rd_f(f, (size_t)P * att), g = rd_f(f, (size_t)P * att);
    auto K = rd_f(f, (size_t)len * kvd), V = rd_f(f, (size_t)len * kvd);
    float *dq = (float*)to_dev(q.data(), q.size() * 4), *dg = (float*)to_dev(g.data(), g.size() * 4);
    float *dK = (float*)to_dev(K.data(), K.size() * 4), *dV = (float*)to_dev(V.data(), V.size() * 4);
    const size_t nel = (size_t)len * kvd, nblk = nel / 32;
    signed char *Kq, *Vq;
    half *Ks, *Vs;
    float* dout;
    CK(cudaMalloc(&Kq, nel)); CK(cudaMalloc(&Vq, nel));
    CK(cudaMalloc(&Ks, nblk * 2)); CK(cudaMalloc(&Vs, nblk * 2));
    CK(cudaMalloc(&dout, (size_t)P * att * 4));
    k_to_q8<<<(unsigned)((nblk + 255) / 256), 256>>>(dK, Kq, Ks, nblk);
    k_to_q8<<<(unsigned)((nblk + 255) / 256), 256>>>(dV, Vq, Vs, nblk);
    // launch geometry of the reference's own bench (fattn_kvhalf.cu:162-190)
    const int TK = 16, TQW = 16;
    const size_t shm = (size_t)2 * TK * hd * 4;
    dim3 grid((P + TQW - 1) / TQW, nq / 2);
    if (hd == 256)
      k_gqa_kv<2, 8, 2><<<grid, TQW * 32, shm>>>(dq, dg, Kq, Vq, Ks, Vs, dout, nq, nkv, hd, kvd, ps, P, TK);
    else
      k_gqa_kv<2, 4, 2><<<grid, TQW * 32, shm>>>(dq, dg, Kq, Vq, Ks, Vs, dout, nq, nkv, hd, kvd, ps, P, TK);
    CK(cudaGetLastError());
    CK(cudaDeviceSynchronize());
    write_dev(o, dout, (size_t)P * att * 4);
  } else {
    return 2;
  }
  fclose(o);
  fclose(f);
  return 0;
}
