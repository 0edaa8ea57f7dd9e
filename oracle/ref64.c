/*
 * Float64 CPU reference of the attention forward (see ref64.h). TEST INFRASTRUCTURE ONLY.
 * Restates b4batunde/Phantom-A100 sim/harness.cu:40-64.
 */
#include "ref64.h"

#include <math.h>
#include <stdlib.h>

void phantom_ref64_attention(const float* q, const float* k, const float* v, double* o, int BH, int N, int d,
                             int causal) {
  double* s = (double*)malloc(sizeof(double) * (size_t)N);
  const double scale = 1.0 / sqrt((double)d);
  for (int bh = 0; bh < BH; ++bh) {
    const size_t base = (size_t)bh * N * d;
    for (int i = 0; i < N; ++i) {
      const float* qi = q + base + (size_t)i * d;
      const int last = causal ? i : N - 1; /* keys 0..last are visible */
      double m = -INFINITY;
      for (int j = 0; j <= last; ++j) {
        const float* kj = k + base + (size_t)j * d;
        double acc = 0.0;
        for (int c = 0; c < d; ++c) acc += (double)qi[c] * (double)kj[c];
        s[j] = acc * scale;
        if (s[j] > m) m = s[j];
      }
      double l = 0.0;
      for (int j = 0; j <= last; ++j) {
        s[j] = exp(s[j] - m);
        l += s[j];
      }
      double* oi = o + base + (size_t)i * d;
      for (int c = 0; c < d; ++c) oi[c] = 0.0;
      for (int j = 0; j <= last; ++j) {
        const float* vj = v + base + (size_t)j * d;
        for (int c = 0; c < d; ++c) oi[c] += s[j] * (double)vj[c];
      }
      for (int c = 0; c < d; ++c) oi[c] /= l;
    }
  }
  free(s);
}
