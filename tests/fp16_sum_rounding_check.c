/* Exhaustive check behind the exact attention kernel's sequential fp16 sums
 * (emx_onnx_cgen_b200/csrc/attention.cu, add_hh): for every pair of fp16
 * values a, b (NaN inputs skipped, each unordered pair once),
 *     RN16(RN32(a + b)) == RN16(a + b)
 * i.e. the reference's statement rounding (the sum in float, then to fp16)
 * equals one fp16 addition.  RN16 of the exact sum is computed from a double
 * (the sum of two fp16 values is exact in double) by rounding to the fp16
 * quantum of its binade, ties to even.  Prints the count of differing pairs
 * and exits non-zero if any differ. */
#include <immintrin.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>

static float dec[65536];

static uint16_t rn16_exact(double x) {
  double ax = fabs(x), r;
  if (ax >= 65520.0) {
    r = INFINITY;
  } else if (ax < 0x1p-14) {
    r = rint(ax * 0x1p24) * 0x1p-24;
  } else {
    int e2;
    frexp(ax, &e2);
    const double quantum = ldexp(1.0, e2 - 11);
    r = rint(ax / quantum) * quantum;
    if (r >= 65520.0) r = INFINITY;
  }
  return (uint16_t)_cvtss_sh((float)(signbit(x) ? -r : r), _MM_FROUND_TO_NEAREST_INT);
}

int main(void) {
  for (int i = 0; i < 65536; ++i) dec[i] = _cvtsh_ss((unsigned short)i);
  long long bad = 0, checked = 0;
#pragma omp parallel for reduction(+ : bad, checked) schedule(dynamic, 64)
  for (int a = 0; a < 65536; ++a) {
    if (isnan(dec[a])) continue;
    for (int b = a; b < 65536; ++b) {
      if (isnan(dec[b])) continue;
      const double exact = (double)dec[a] + (double)dec[b];
      const uint16_t twice = (uint16_t)_cvtss_sh((float)exact, _MM_FROUND_TO_NEAREST_INT);
      const uint16_t once = rn16_exact(exact);
      ++checked;
      if (twice != once && !(isnan(dec[twice]) && isnan(dec[once]))) ++bad;
    }
  }
  printf("%lld %lld\n", checked, bad);
  return bad != 0;
}
