/* abi_decode.c — drives libaspida_attn.so the way the Ada binding drives the
 * shim (src/llm/llm_gpu.adb:73-149: dlopen by path, dlsym per entry point,
 * plain pointers and ints across the boundary). Creates a KV state, fills
 * its fp16 cache, runs one batched GQA decode through aspida_attn_decode and
 * checks it against a double-precision CPU loop of the Llama attention
 * (llm_llama.adb:876-898). Prints "max_abs <err>" and exits 0 when within
 * 2e-3, 1 on a mismatch, 2 on a setup failure.
 *
 * Build: gcc -O2 abi_decode.c -I<cuda>/include -L<cuda>/lib64 -lcudart -ldl -lm
 * Run:   ./abi_decode <path to libaspida_attn.so>
 */
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>

typedef int (*fattn_new_fn)(int, int, int);
typedef void (*fattn_free_fn)(int);
typedef int (*fattn_kv_fn)(int, void**, void**, int*, int*);
typedef size_t (*ws_size_fn)(int, int, int, int, int, int);
typedef int (*decode_fn)(const float*, const float*, const void* const*, const void* const*,
                         const int*, const int*, float*, int, int, int, int, float, int, float,
                         int, int, void*, size_t, void*);
typedef int (*last_error_fn)(void);

#define CHECK(x)                                                     \
  do {                                                               \
    if (!(x)) {                                                      \
      fprintf(stderr, "setup failed: %s (line %d)\n", #x, __LINE__); \
      return 2;                                                      \
    }                                                                \
  } while (0)

static unsigned long long rng = 88172645463325252ull;
static float frand(void) { /* xorshift64, uniform in [-1, 1) */
  rng ^= rng << 13;
  rng ^= rng >> 7;
  rng ^= rng << 17;
  return (float)((rng >> 11) * (1.0 / 9007199254740992.0)) * 2.f - 1.f;
}

int main(int argc, char** argv) {
  if (argc != 2) {
    fprintf(stderr, "usage: %s <libaspida_attn.so>\n", argv[0]);
    return 2;
  }
  void* lib = dlopen(argv[1], RTLD_NOW);
  CHECK(lib);
  fattn_new_fn fattn_new = (fattn_new_fn)dlsym(lib, "aspida_gpu_fattn_new");
  fattn_free_fn fattn_free = (fattn_free_fn)dlsym(lib, "aspida_gpu_fattn_free");
  fattn_kv_fn fattn_kv = (fattn_kv_fn)dlsym(lib, "aspida_gpu_fattn_kv");
  ws_size_fn ws_size = (ws_size_fn)dlsym(lib, "aspida_attn_decode_workspace_size");
  decode_fn decode = (decode_fn)dlsym(lib, "aspida_attn_decode");
  last_error_fn last_error = (last_error_fn)dlsym(lib, "aspida_gpu_last_error");
  CHECK(fattn_new && fattn_free && fattn_kv && ws_size && decode && last_error);

  enum { B = 3, NQ = 8, NKV = 2, HD = 128, MAXLEN = 600 };
  const int kvd = NKV * HD, lens[B] = {1, 257, 600};
  const float scale = 1.f / sqrtf((float)HD);
  int handles[B];
  void *Kd[B], *Vd[B];
  float* Kh[B];
  float* Vh[B];
  for (int b = 0; b < B; ++b) {
    handles[b] = fattn_new(MAXLEN, kvd, NQ);
    CHECK(handles[b] >= 0);
    int ml = 0, kv = 0;
    CHECK(fattn_kv(handles[b], &Kd[b], &Vd[b], &ml, &kv) == 0 && ml == MAXLEN && kv == kvd);
    const size_t n = (size_t)lens[b] * kvd;
    Kh[b] = (float*)malloc(n * sizeof(float));
    Vh[b] = (float*)malloc(n * sizeof(float));
    _Float16* tmp = (_Float16*)malloc(n * sizeof(_Float16));   /* IEEE binary16 */
    CHECK(Kh[b] && Vh[b] && tmp);
    for (int pass = 0; pass < 2; ++pass) {
      float* dst = pass ? Vh[b] : Kh[b];
      for (size_t i = 0; i < n; ++i) {
        tmp[i] = (_Float16)frand();
        dst[i] = (float)tmp[i];            /* the CPU check uses the fp16 values */
      }
      CHECK(cudaMemcpy(pass ? Vd[b] : Kd[b], tmp, n * sizeof(_Float16),
                       cudaMemcpyHostToDevice) == cudaSuccess);
    }
    free(tmp);
  }
  float q[B * NQ * HD], out[B * NQ * HD];
  for (int i = 0; i < B * NQ * HD; ++i) q[i] = frand();
  int pos[B];
  for (int b = 0; b < B; ++b) pos[b] = lens[b] - 1;

  float *dq, *dout;
  int* dpos;
  void **dK, **dV, *ws;
  const size_t wsb = ws_size(B, NQ, NKV, HD, MAXLEN, 0);
  CHECK(cudaMalloc((void**)&dq, sizeof q) == cudaSuccess);
  CHECK(cudaMalloc((void**)&dout, sizeof out) == cudaSuccess);
  CHECK(cudaMalloc((void**)&dpos, sizeof pos) == cudaSuccess);
  CHECK(cudaMalloc((void**)&dK, sizeof Kd) == cudaSuccess);
  CHECK(cudaMalloc((void**)&dV, sizeof Vd) == cudaSuccess);
  CHECK(cudaMalloc(&ws, wsb) == cudaSuccess);
  CHECK(cudaMemcpy(dq, q, sizeof q, cudaMemcpyHostToDevice) == cudaSuccess);
  CHECK(cudaMemcpy(dpos, pos, sizeof pos, cudaMemcpyHostToDevice) == cudaSuccess);
  CHECK(cudaMemcpy(dK, Kd, sizeof Kd, cudaMemcpyHostToDevice) == cudaSuccess);
  CHECK(cudaMemcpy(dV, Vd, sizeof Vd, cudaMemcpyHostToDevice) == cudaSuccess);

  const int rc = decode(dq, NULL, (const void* const*)dK, (const void* const*)dV, dpos, NULL,
                        dout, B, NQ, NKV, HD, scale, 0, 0.f, MAXLEN, 0, ws, wsb, NULL);
  CHECK(rc == 0);
  CHECK(cudaMemcpy(out, dout, sizeof out, cudaMemcpyDeviceToHost) == cudaSuccess);
  CHECK(last_error() == 0);

  /* CPU reference (double): softmax over keys 0..pos of each kv head's rows */
  double max_err = 0.0;
  for (int b = 0; b < B; ++b) {
    const int L = lens[b];
    double* s = (double*)malloc((size_t)L * sizeof(double));
    CHECK(s);
    for (int h = 0; h < NQ; ++h) {
      const int kh = h / (NQ / NKV);
      const float* qh = q + ((size_t)b * NQ + h) * HD;
      double mx = -1e300, den = 0.0;
      for (int j = 0; j < L; ++j) {
        double d = 0.0;
        for (int k = 0; k < HD; ++k) d += (double)qh[k] * Kh[b][(size_t)j * kvd + kh * HD + k];
        s[j] = d * scale;
        if (s[j] > mx) mx = s[j];
      }
      for (int j = 0; j < L; ++j) {
        s[j] = exp(s[j] - mx);
        den += s[j];
      }
      for (int k = 0; k < HD; ++k) {
        double acc = 0.0;
        for (int j = 0; j < L; ++j) acc += s[j] * Vh[b][(size_t)j * kvd + kh * HD + k];
        const double err = fabs(acc / den - out[((size_t)b * NQ + h) * HD + k]);
        if (err > max_err) max_err = err;
      }
    }
    free(s);
    free(Kh[b]);
    free(Vh[b]);
    fattn_free(handles[b]);
  }
  cudaFree(dq);
  cudaFree(dout);
  cudaFree(dpos);
  cudaFree(dK);
  cudaFree(dV);
  cudaFree(ws);
  printf("max_abs %.3e\n", max_err);
  return max_err <= 2e-3 ? 0 : 1;
}
