/* TEST INFRASTRUCTURE ONLY (lfm2q oracle): exact fp32 helpers the numpy/torch restatement cannot express.
 *
 * The reference's grouped W8A8 fold (kernels/int8_gemm.cu:202-215) accumulates every 64-wide K group's int32
 * partial sum as facc = fmaf((float)part, sxT[g][m], facc): one fused multiply-add with a single rounding.
 * numpy has no fused multiply-add, so the fold is restated here with C's fmaf (correctly rounded by definition).
 * Compiled with -ffp-contract=off so no other operation is fused. Not linked into the product library. */
#include <math.h>
#include <stdint.h>

/* acc[m * N + n] = fmaf((float)part[m * N + n], s[m], acc[m * N + n]) */
void oracle_fold_group(const int32_t *part, const float *s, float *acc, int64_t M, int64_t N) {
  for (int64_t m = 0; m < M; ++m) {
    const float sm = s[m];
    const int32_t *p = part + m * N;
    float *a = acc + m * N;
    for (int64_t n = 0; n < N; ++n) a[n] = fmaf((float)p[n], sm, a[n]);
  }
}

/* out[i] = fmaf(a[i], b[i], c[i]) */
void oracle_fmaf(const float *a, const float *b, const float *c, float *out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = fmaf(a[i], b[i], c[i]);
}
