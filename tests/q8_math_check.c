/* Host check of the Q8_0 quantiser's division-free arithmetic (the device
 * helpers q8_scale and q8_round in odiengine_b200/csrc/common.cuh):
 *   q8_scale(x) = fma(fma(-q0, 127, x), r, q0), q0 = x * r, r = RN(1/127)
 *                 must equal the IEEE quotient x / 127.0f for every
 *                 non-negative finite fp32 x (subnormals included);
 *   q8_round(t) = trunc(t + copysign(0.5 - 2^-25, t)) must equal roundf(t)
 *                 (half away from zero) for every fp32 |t| < 2^23.
 * Usage: q8_math_check [stride]; stride 1 (the default) walks every bit
 * pattern, a larger stride a regular subset.  Exit status 1 on a mismatch.
 * Build with contraction off (-ffp-contract=off) so each operation rounds. */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static float bits_to_float(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}

int main(int argc, char** argv) {
  const uint64_t stride = argc > 1 ? strtoull(argv[1], NULL, 10) : 1;
  const float r = 0x1.020408p-7f; /* RN(1/127) */
  volatile float c127 = 127.0f;   /* keeps the reference a true division */
  const float half_below = 0x1.fffffep-2f;
  long bad_div = 0, bad_round = 0;
  uint64_t n_div = 0, n_round = 0;
  if (stride == 0 || r != 1.0f / c127) return 2;
  for (uint64_t u = 0; u < 0x7F800000ull; u += stride) {
    const float x = bits_to_float((uint32_t)u);
    const float q0 = x * r;
    const float got = fmaf(fmaf(-q0, 127.0f, x), r, q0);
    const float ref = x / c127;
    ++n_div;
    if (memcmp(&got, &ref, 4) != 0) {
      if (bad_div < 5) printf("q8_scale mismatch: x=%a want %a got %a\n", x, ref, got);
      ++bad_div;
    }
  }
  /* both signs: the positive patterns below 2^23 and their negations */
  for (uint64_t u = 0; u < 0x4B000000ull; u += stride) {
    for (int sgn = 0; sgn < 2; ++sgn) {
      const float t = bits_to_float((uint32_t)u | (sgn ? 0x80000000u : 0u));
      const float got = truncf(t + copysignf(half_below, t));
      const float ref = roundf(t);
      ++n_round;
      if (got != ref) {
        if (bad_round < 5) printf("q8_round mismatch: t=%a want %a got %a\n", t, ref, got);
        ++bad_round;
      }
    }
  }
  printf("q8_scale: %llu values, %ld mismatches; q8_round: %llu values, %ld mismatches\n",
         (unsigned long long)n_div, bad_div, (unsigned long long)n_round, bad_round);
  return (bad_div || bad_round) ? 1 : 0;
}
