/*
 * Sequential selective scan in plain C (float32, IEEE, no fast-math), parallel over (batch, channel)
 * with OpenMP. TEST INFRASTRUCTURE ONLY: the oracle for sizes the NumPy loops cannot finish in seconds,
 * and the timed CPU baseline of bench.py.
 *
 * Per (batch b, channel d), restating experiments/09-features/test_features.py:23-43 and
 * experiments/18-prefill/verify_state_out.py:13-26 (the reference's own CPU implementation):
 *   delta' = softplus(delta) with the >20 cutoff (test_features.py:13-16)
 *   h[n] = exp(delta' * A[d,n]) * h[n] + (delta' * u) * B[b,n,t];  y = sum_n h[n] * C[b,n,t]
 *   y += D[d] * u;  y *= z / (1 + exp(-z));  last[b,d,n] = h[n] after the final step.
 */
#include <math.h>
#include <stdint.h>

#ifdef _OPENMP
#include <omp.h>
#endif

static inline float softplus_ref(float x) { return x <= 20.0f ? log1pf(expf(x)) : x; }

void mm_ref_selective_scan(const float* u, const float* delta, const float* A, const float* B, const float* C,
                           const float* D, const float* z, float* y, float* last, int64_t batch, int64_t dim,
                           int64_t dstate, int64_t seqlen, int softplus, int nthreads) {
  const int64_t rows = batch * dim;
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 1)
#endif
  for (int64_t r = 0; r < rows; ++r) {
    const int64_t b = r / dim, d = r % dim;
    float h[64];
    for (int64_t n = 0; n < dstate; ++n) h[n] = 0.0f;
    const float* ur = u + r * seqlen;
    const float* dr = delta + r * seqlen;
    const float* Bb = B + b * dstate * seqlen;
    const float* Cb = C + b * dstate * seqlen;
    const float* Ar = A + d * dstate;
    float* yr = y + r * seqlen;
    for (int64_t t = 0; t < seqlen; ++t) {
      const float dt = softplus ? softplus_ref(dr[t]) : dr[t];
      const float du = dt * ur[t];
      float acc = 0.0f;
      for (int64_t n = 0; n < dstate; ++n) {
        const float a = expf(dt * Ar[n]);
        h[n] = a * h[n] + du * Bb[n * seqlen + t];
        acc += h[n] * Cb[n * seqlen + t];
      }
      if (D) acc += D[d] * ur[t];
      if (z) {
        const float zv = z[r * seqlen + t];
        acc *= zv / (1.0f + expf(-zv));
      }
      yr[t] = acc;
    }
    if (last)
      for (int64_t n = 0; n < dstate; ++n) last[r * dstate + n] = h[n];
  }
}

int mm_ref_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
