/*
 * CPU oracle for the Q4 decode hot path -- TEST INFRASTRUCTURE / CPU BASELINE.
 *
 * A C restatement of the reference's CPU arithmetic, used (a) to cross-check
 * the numpy oracle (oracle/q4.py), and (b) as the timed CPU baseline of
 * bench.py.  Nothing in the product path links or loads it.
 *
 * Semantics follow the reference's numpy oracle exactly where rounding is
 * concerned:
 *   - dequant w = bf16_rn(float(q) * float(scale_bf16))   tools/ref/gemv_q.py:32-37
 *   - gemv   y = sum_k w * x in fp32                      tools/ref/gemv_q.py:78-79
 *   - FFN    gate/up rounded to bf16, GeGLU in double
 *            from the sqrt(2/pi) factor on (numpy promotion), SwiGLU in fp32,
 *            act rounded to bf16 via float32, y = Wd act   runtime/py/model.py:687-698, 854-860
 *   - rmsnorm (gemma) fp32 mean of squares, x * (1/sqrt(var + eps))  model.py:522-529
 * Accumulation order differs from numpy/BLAS (sequential within a row), as
 * any two fp32 implementations do.  The packed-Q4 traversal (20-byte blocks
 * read in place, per-row loop) follows runtime/cpp/src/generator.cpp:69-101,
 * with the bf16 rounding of each product added to match the numpy oracle.
 * Rows are split across OpenMP threads.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* float -> bf16 round-to-nearest-even (runtime/cpp/src/bf16.cpp:7-18), widened back */
static inline float bf16r(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu)) {
    u = 0x7FC00000u;
  } else {
    u += 0x7FFFu + ((u >> 16) & 1u);
    u &= 0xFFFF0000u;
  }
  float r;
  memcpy(&r, &u, 4);
  return r;
}

static inline float bits_to_f32(uint32_t bits16) {
  uint32_t u = bits16 << 16;
  float r;
  memcpy(&r, &u, 4);
  return r;
}

int q4cpu_version(void) { return 1; }

int q4cpu_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* One row of y = W x: combined row of K/32 20-byte blocks. */
static float row_dot(const uint8_t* row, int K, const float* x) {
  float acc = 0.f;
  const int KB = K / 32;
  for (int b = 0; b < KB; ++b) {
    const uint8_t* blk = row + (size_t)b * 20;
    const float s = bits_to_f32((uint32_t)blk[16] | ((uint32_t)blk[17] << 8));
    const float* xb = x + (size_t)b * 32;
    for (int j = 0; j < 16; ++j) {
      int lo = blk[j] & 0x0F, hi = blk[j] >> 4;
      if (lo >= 8) lo -= 16;
      if (hi >= 8) hi -= 16;
      acc += bf16r((float)lo * s) * xb[2 * j];
      acc += bf16r((float)hi * s) * xb[2 * j + 1];
    }
  }
  return acc;
}

/* y[t, n] = sum_k W[n, k] x[t, k]; x (ntok, K), y (ntok, N). */
int q4cpu_gemv(const uint8_t* W, int N, int K, int ntok, const float* x, float* y, int nthreads) {
  if (!W || !x || !y || N < 0 || K % 32 || ntok < 1) return 1;
  const size_t rb = (size_t)(K / 32) * 20;
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(static)
#endif
  for (int n = 0; n < N; ++n)
    for (int t = 0; t < ntok; ++t) y[(size_t)t * N + n] = row_dot(W + (size_t)n * rb, K, x + (size_t)t * K);
  (void)nthreads;
  return 0;
}

/* GeGLU as numpy evaluates runtime/py/model.py:690-693. */
static float geglu(float g, float u) {
  const float g3 = g * g * g;
  const float inner = g + 0.044715f * g3;
  const double t = tanh(0x1.9884533d43651p-1 * (double)inner);
  const double gelu = (double)(0.5f * g) * (1.0 + t);
  return (float)(gelu * (double)u);
}

/* SwiGLU as runtime/py/model.py:857-859 (float32). */
static float swiglu(float g, float u) {
  const float e = (float)exp(-(double)g);
  const float s = 1.0f / (1.0f + e);
  return (g * s) * u;
}

/* Fused FFN: y = Wd bf16(act(bf16(Wg x), bf16(Wu x))).  act 0 = GeGLU, 1 = SwiGLU.
 * gate/up (I, H/32*20), down (H, I/32*20); x (H), y (H) fp32.  act_out (I) optional. */
int q4cpu_ffn(const uint8_t* Wg, const uint8_t* Wu, const uint8_t* Wd, int H, int I, int act, const float* x,
              float* y, float* act_out, int nthreads) {
  if (!Wg || !Wu || !Wd || !x || !y || H % 32 || I % 32) return 1;
  float* a = (float*)malloc(sizeof(float) * (size_t)I);
  if (!a) return 2;
  const size_t rbh = (size_t)(H / 32) * 20, rbi = (size_t)(I / 32) * 20;
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(static)
#endif
  for (int i = 0; i < I; ++i) {
    const float g = bf16r(row_dot(Wg + (size_t)i * rbh, H, x));
    const float u = bf16r(row_dot(Wu + (size_t)i * rbh, H, x));
    a[i] = bf16r(act == 0 ? geglu(g, u) : swiglu(g, u));
  }
#ifdef _OPENMP
#pragma omp parallel for schedule(static)
#endif
  for (int h = 0; h < H; ++h) y[h] = row_dot(Wd + (size_t)h * rbi, I, a);
  if (act_out) memcpy(act_out, a, sizeof(float) * (size_t)I);
  free(a);
  (void)nthreads;
  return 0;
}

/* Gemma RMSNorm with unit weight, bf16 result (model.py:522-529). */
static void rmsnorm_bf16(const float* x, float* out, int n, float eps) {
  float ss = 0.f;
  for (int i = 0; i < n; ++i) ss += x[i] * x[i];
  const float inv = 1.0f / sqrtf(ss / (float)n + eps);
  for (int i = 0; i < n; ++i) out[i] = bf16r(x[i] * inv);
}

/* One FFN half-block of a Gemma-4 decode layer with unit norms
 * (model.py:782-806): x <- bf16(x + bf16(rmsnorm(bf16(FFN_geglu(rmsnorm(x)))))).
 * x is (H) bf16-valued fp32, updated in place. */
int q4cpu_ffn_block(const uint8_t* Wg, const uint8_t* Wu, const uint8_t* Wd, int H, int I, float* x,
                    int nthreads) {
  float* xn = (float*)malloc(sizeof(float) * (size_t)H * 3);
  if (!xn) return 2;
  float* d = xn + H;
  float* dn = d + H;
  rmsnorm_bf16(x, xn, H, 1e-6f);
  int rc = q4cpu_ffn(Wg, Wu, Wd, H, I, 0, xn, d, NULL, nthreads);
  if (!rc) {
    for (int h = 0; h < H; ++h) d[h] = bf16r(d[h]);
    rmsnorm_bf16(d, dn, H, 1e-6f);
    for (int h = 0; h < H; ++h) x[h] = bf16r(x[h] + dn[h]);
  }
  free(xn);
  return rc;
}
