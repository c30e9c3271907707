/* abi_linear.c -- a C translation unit against include/sa3k.h (gcc, no CUDA headers): one LoRA
 * linear training step of a Q8_0 base through the C ABI with host buffers, checked against a
 * float64 loop restatement of dit_lin (src/dit.h:106-122) on the dequantized weight.
 *
 * Usage: abi_linear            -> prints the rel-L2 error of y, dx, dA, dB; exit 0 when all are
 *                                 within 1e-2 and the error paths behave, 1 otherwise. */
#include "sa3k.h"

#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

enum { S = 192, IN = 256, OUT = 320, R = 16 };

static uint64_t lcg = 0x9E3779B97F4A7C15ull;
static double unif(void) { /* U(0, 1) from a 64-bit LCG (Knuth's MMIX constants) */
  lcg = lcg * 6364136223846793005ull + 1442695040888963407ull;
  return ((double)(lcg >> 11) + 0.5) / 9007199254740992.0;
}
static float gauss(double sd) { /* Box-Muller */
  const double u = unif(), v = unif();
  return (float)(sd * sqrt(-2.0 * log(u)) * cos(6.283185307179586 * v));
}

/* GGUF Q8_0 encode of one row: per 32 values d = max|x| / 127 (stored f16), q = round(x / d). */
static void q8_0_row(const float* x, int n, unsigned char* out, double* deq) {
  for (int b = 0; b < n / 32; ++b) {
    float amax = 0.f;
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(x[b * 32 + i]));
    const _Float16 dh = (_Float16)(amax / 127.f);
    const float d = (float)dh, id = d != 0.f ? 1.f / d : 0.f;
    memcpy(out + b * 34, &dh, 2);
    for (int i = 0; i < 32; ++i) {
      const int q = (int)lrintf(x[b * 32 + i] * id);
      out[b * 34 + 2 + i] = (unsigned char)(signed char)q;
      deq[b * 32 + i] = (double)d * (double)q;
    }
  }
}

static double rel(const float* a, const double* b, long n) {
  double num = 0, den = 0;
  for (long i = 0; i < n; ++i) {
    num += ((double)a[i] - b[i]) * ((double)a[i] - b[i]);
    den += b[i] * b[i];
  }
  return sqrt(num / (den > 0 ? den : 1e-300));
}

int main(void) {
  char err[512];
  int bad = 0;
  printf("%s\n", sa3k_version());
  /* error paths: a NULL context is refused with a message, not a crash */
  if (sa3k_linear_fwd(NULL, NULL, NULL, NULL, NULL, 0, NULL, err, sizeof err) == 0 || !err[0]) bad = 1;
  sa3k_ctx* ctx = NULL;
  if (sa3k_ctx_create(0, &ctx, err, sizeof err)) {
    fprintf(stderr, "ctx: %s\n", err);
    return 1;
  }
  float* W = malloc(sizeof(float) * OUT * IN);
  double* Wd = malloc(sizeof(double) * OUT * IN);
  unsigned char* raw = malloc((size_t)OUT * IN / 32 * 34);
  for (long i = 0; i < (long)OUT * IN; ++i) W[i] = gauss(0.02);
  for (int o = 0; o < OUT; ++o) q8_0_row(W + (long)o * IN, IN, raw + (long)o * IN / 32 * 34, Wd + (long)o * IN);
  sa3k_weight* w = NULL;
  if (sa3k_weight_upload(ctx, SA3K_TYPE_Q8_0, raw, IN, OUT, &w, err, sizeof err)) {
    fprintf(stderr, "upload: %s\n", err);
    return 1;
  }
  float *x = malloc(sizeof(float) * S * IN), *dy = malloc(sizeof(float) * S * OUT);
  float *A = malloc(sizeof(float) * R * IN), *B = malloc(sizeof(float) * OUT * R);
  for (long i = 0; i < (long)S * IN; ++i) x[i] = gauss(1.0);
  for (long i = 0; i < (long)S * OUT; ++i) dy[i] = gauss(1.0);
  for (long i = 0; i < (long)R * IN; ++i) A[i] = gauss(1.0 / sqrt((double)IN));
  for (long i = 0; i < (long)OUT * R; ++i) B[i] = gauss(0.05);
  const float s = 2.0f; /* alpha / rank */
  sa3k_adapter ad = {A, B, NULL, NULL, s, R};
  float *y = malloc(sizeof(float) * S * OUT), *dx = malloc(sizeof(float) * S * IN);
  float *dA = malloc(sizeof(float) * R * IN), *dB = malloc(sizeof(float) * OUT * R);
  if (sa3k_linear_fwd_bwd_host(ctx, w, &ad, NULL, x, dy, S, y, dx, dA, dB, NULL, err, sizeof err)) {
    fprintf(stderr, "step: %s\n", err);
    return 1;
  }
  /* float64 restatement: u = x A^T, y = x W^T + s u B^T, v = dy B, dx = dy W + s v A,
   * dB = s dy^T u, dA = s v^T x */
  double *u = calloc((size_t)S * R, sizeof(double)), *v = calloc((size_t)S * R, sizeof(double));
  double *ry = calloc((size_t)S * OUT, sizeof(double)), *rdx = calloc((size_t)S * IN, sizeof(double));
  double *rdA = calloc((size_t)R * IN, sizeof(double)), *rdB = calloc((size_t)OUT * R, sizeof(double));
  for (int t = 0; t < S; ++t)
    for (int r = 0; r < R; ++r) {
      double a = 0, b = 0;
      for (int i = 0; i < IN; ++i) a += (double)x[t * IN + i] * A[r * IN + i];
      for (int o = 0; o < OUT; ++o) b += (double)dy[t * OUT + o] * B[o * R + r];
      u[t * R + r] = a;
      v[t * R + r] = b;
    }
  for (int t = 0; t < S; ++t) {
    for (int o = 0; o < OUT; ++o) {
      double a = 0;
      for (int i = 0; i < IN; ++i) a += (double)x[t * IN + i] * Wd[(long)o * IN + i];
      for (int r = 0; r < R; ++r) a += s * u[t * R + r] * B[o * R + r];
      ry[t * OUT + o] = a;
    }
    for (int i = 0; i < IN; ++i) {
      double a = 0;
      for (int o = 0; o < OUT; ++o) a += (double)dy[t * OUT + o] * Wd[(long)o * IN + i];
      for (int r = 0; r < R; ++r) a += s * v[t * R + r] * A[r * IN + i];
      rdx[t * IN + i] = a;
    }
  }
  for (int o = 0; o < OUT; ++o)
    for (int r = 0; r < R; ++r) {
      double a = 0;
      for (int t = 0; t < S; ++t) a += (double)dy[t * OUT + o] * u[t * R + r];
      rdB[o * R + r] = s * a;
    }
  for (int r = 0; r < R; ++r)
    for (int i = 0; i < IN; ++i) {
      double a = 0;
      for (int t = 0; t < S; ++t) a += v[t * R + r] * x[t * IN + i];
      rdA[r * IN + i] = s * a;
    }
  const double e_y = rel(y, ry, (long)S * OUT), e_dx = rel(dx, rdx, (long)S * IN);
  const double e_dA = rel(dA, rdA, (long)R * IN), e_dB = rel(dB, rdB, (long)OUT * R);
  printf("rel-L2 y %.3g dx %.3g dA %.3g dB %.3g\n", e_y, e_dx, e_dA, e_dB);
  if (!(e_y < 1e-2 && e_dx < 1e-2 && e_dA < 1e-2 && e_dB < 1e-2)) bad = 1;
  /* a rank above 16 is refused with an error, not run */
  sa3k_adapter big = {A, B, NULL, NULL, s, 32};
  if (sa3k_linear_fwd_bwd_host(ctx, w, &big, NULL, x, dy, S, y, dx, dA, dB, NULL, err, sizeof err) == 0) bad = 1;
  sa3k_weight_free(w);
  if (sa3k_sync(ctx, err, sizeof err)) bad = 1;
  sa3k_ctx_destroy(ctx);
  printf(bad ? "FAIL\n" : "OK\n");
  return bad;
}
