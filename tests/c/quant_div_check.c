/* Checks the arithmetic of the int8 activation quantiser's element step.
 *
 * The recipe (k008_int8_gemm.py:148-151) computes, per row, s = max(amax,
 * 1e-6) / 127 and per element q = round_half_even(x / s) with an IEEE fp32
 * division.  The kernel instead computes, per row, y = 1/s correctly rounded,
 * and per element
 *     q0 = x * y,   r = fma(-q0, s, x),   q1 = fma(r, y, q0)
 * (the division by a correctly rounded reciprocal with one residual
 * correction, P. Markstein, "Computation of elementary functions on the IBM
 * RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990), then rounds q1
 * half-to-even by adding 1.5 * 2^23 and keeps the low byte of the sum's bits
 * as the int8 value.
 *
 * This program compares both against the IEEE quotient x / s and rint() for
 * 16-bit inputs x (fp16 or bf16, every finite value) and every scale a row
 * can produce (s from every finite 16-bit |amax|, or a strided subset), over
 * the x a row with that maximum can hold (|x| <= amax).  Exit status 0 when
 * every int8 value matches and every quotient of a normal x is bit-identical.
 * Two kinds of quotient may differ, both ending as int8 0: a zero quotient in
 * its sign (x = -0 gives +0 here; int8 has no negative zero), and the
 * quotient of a tiny x (|x| < 2^-100; bf16 holds fp32-subnormal values),
 * where the residual underflows and the correction is inexact.  Since
 * s >= 1e-6 / 127, such quotients are below 2^-100 * 127e6 < 1e-21.
 *
 * usage: quant_div_check <f16|bf16> <amax stride> [first amax bits]
 * Build with -ffp-contract=off so that no other product is fused.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static float from_bits(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static uint32_t to_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

static float bf16_to_float(uint16_t h) { return from_bits((uint32_t)h << 16); }

static float f16_to_float(uint16_t h) {
  const uint32_t sign = (uint32_t)(h >> 15) << 31;
  const int e = (h >> 10) & 0x1f;
  const uint32_t m = h & 0x3ff;
  if (e == 0x1f) return from_bits(sign | 0x7f800000u | (m << 13));
  if (e == 0) {  /* zero or subnormal: m * 2^-24, exact in fp32 */
    const float v = ldexpf((float)m, -24);
    return sign ? -v : v;
  }
  return from_bits(sign | ((uint32_t)(e - 15 + 127) << 23) | (m << 13));
}

int main(int argc, char** argv) {
  if (argc < 3) {
    fprintf(stderr, "usage: %s <f16|bf16> <amax stride> [first amax bits]\n", argv[0]);
    return 2;
  }
  const int bf16 = strcmp(argv[1], "bf16") == 0;
  const long stride = atol(argv[2]);
  const long first = argc > 3 ? atol(argv[3]) : 0;
  float (*conv)(uint16_t) = bf16 ? bf16_to_float : f16_to_float;

  /* every finite 16-bit value, once */
  static float xs[65536];
  int nx = 0;
  for (uint32_t b = 0; b < 65536; ++b) {
    const float v = conv((uint16_t)b);
    if (isfinite(v)) xs[nx++] = v;
  }
  long pairs = 0, bad_q = 0, sub_q = 0, bad_i = 0, scales = 0;
  for (long ab = first; ab < 0x8000; ab += stride) {  /* non-negative 16-bit patterns */
    const float amax = conv((uint16_t)ab);
    if (!isfinite(amax)) continue;
    ++scales;
    const float s = fmaxf(amax, 1e-6f) / 127.0f;
    const float y = 1.0f / s;
    for (int i = 0; i < nx; ++i) {
      const float x = xs[i];
      if (fabsf(x) > amax) continue;
      ++pairs;
      const float q_ref = x / s;
      const float q0 = x * y;
      const float r = fmaf(-q0, s, x);
      const float q1 = fmaf(r, y, q0);
      /* x = -0 gives +0 here and -0 by IEEE division; both become int8 0. */
      if (to_bits(q1) != to_bits(q_ref) && !(q1 == 0.0f && q_ref == 0.0f)) {
        if (fabsf(x) < 0x1p-100f) {
          ++sub_q;
        } else {
          if (bad_q < 10)
            fprintf(stderr, "quotient differs: x=%a s=%a ieee=%a ours=%a\n", x, s, q_ref, q1);
          ++bad_q;
        }
      }
      const float t = q1 + 12582912.0f;
      const int8_t ours = (int8_t)(to_bits(t) & 0xffu);
      const int ref = (int)rintf(q_ref);
      if (ref != (int)ours) {
        if (bad_i < 10) fprintf(stderr, "int8 differs: x=%a s=%a ref=%d ours=%d\n", x, s, ref, (int)ours);
        ++bad_i;
      }
    }
  }
  printf("%s: %ld scales, %ld (x, s) pairs, %ld quotient mismatches (|x| >= 2^-100), "
         "%ld (|x| < 2^-100), %ld int8 mismatches\n",
         bf16 ? "bf16" : "f16", scales, pairs, bad_q, sub_q, bad_i);
  return (bad_q == 0 && bad_i == 0 && pairs > 0) ? 0 : 1;
}
