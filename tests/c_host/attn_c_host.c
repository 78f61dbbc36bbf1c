/* A plain C host calling the runtime the way MLIR-lowered code does: the
 * reference op's own form (rank-2 f32 memrefs, cf. the reference's
 * examples/MatMUL/main.c descriptor layout), causal, then checked against a
 * double-precision two-pass softmax.  Exit 0 = within 1e-4, 1 = wrong result,
 * 2 = the runtime returned an error (printed). */
#include <math.h>
#include <stdio.h>
#include <stdint.h>

#include "attn_rt.h"

enum { N = 128, D = 64 };
static float Q[N][D], K[N][D], V[N][D], O[N][D];

static float lcg(uint32_t* s) {
  *s = *s * 1664525u + 1013904223u;
  return ((*s >> 8) & 0xFFFF) / 32768.0f - 1.0f;
}

int main(void) {
  uint32_t seed = 12345u;
  for (int i = 0; i < N; ++i)
    for (int d = 0; d < D; ++d) {
      Q[i][d] = lcg(&seed);
      K[i][d] = lcg(&seed);
      V[i][d] = lcg(&seed);
    }
  AttnMemRef2D q = {Q, Q, 0, {N, D}, {D, 1}};
  AttnMemRef2D k = {K, K, 0, {N, D}, {D, 1}};
  AttnMemRef2D v = {V, V, 0, {N, D}, {D, 1}};
  AttnMemRef2D o = {O, O, 0, {N, D}, {D, 1}};
  const float scale = 0.125f;
  int rc = _mlir_ciface_attn_fused_f32_causal(&q, &k, &v, scale, &o);
  if (rc != ATTN_OK) {
    printf("attention.fused failed: %d (%s): %s\n", rc, attn_rt_status_string(rc),
           attn_rt_last_error());
    return 2;
  }
  double worst = 0.0, omax = 0.0;
  for (int i = 0; i < N; ++i) {
    double s[N], m = -INFINITY, l = 0.0;
    for (int j = 0; j <= i; ++j) {
      double acc = 0.0;
      for (int d = 0; d < D; ++d) acc += (double)Q[i][d] * K[j][d];
      s[j] = acc * scale;
      if (s[j] > m) m = s[j];
    }
    for (int j = 0; j <= i; ++j) l += exp(s[j] - m);
    for (int d = 0; d < D; ++d) {
      double r = 0.0;
      for (int j = 0; j <= i; ++j) r += exp(s[j] - m) * V[j][d];
      r /= l;
      if (fabs(r) > omax) omax = fabs(r);
      if (fabs(r - O[i][d]) > worst) worst = fabs(r - O[i][d]);
    }
  }
  printf("max_rel_err %.3e\n", worst / omax);
  return worst / omax <= 1e-4 ? 0 : 1;
}
