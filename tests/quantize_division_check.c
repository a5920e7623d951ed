/* CPU check of the divide-free e4m3 cast used on the GPU (quantize.cuh,
 * CastMarkstein) for scales 2^-60 <= s <= 2^100:
 *   L  = bf16 value >= s * 1024 (s * 1024 rounded up to bf16)
 *   x' = max(min(x, L), -L)            (bf16 min then max; a NaN x becomes L)
 *   r  = RN(1/s), q0 = RN(x' * r), e = fma(q0, -s, x'), q1 = fma(e, r, q0)
 *   t  = |q1| with the sign of x'; byte = e4m3 with saturation to +-448.
 * The reference byte is e4m3(max(-448, min(x / s, 448))) with IEEE division
 * and NaN-ignoring min/max.
 * Part 1: q1 == x / s for every (bf16 significand, fp32 significand) pair.
 * Part 2: q1 == x / s over x and s exponents at the edges of the scale window
 *         whenever |q0| >= 2^-11 (below that both bytes are a signed zero).
 * Part 3: byte equality for all 65,536 bf16 bit patterns (NaN, inf, zeros,
 *         subnormals) against sampled scales across the window.
 * Part 4: the form without the clamp that current scaling uses when the tensor
 *         holds no NaN (quant_resident_kernel): s = RN(amax / 448) for a bf16
 *         amax, byte = e4m3(q1) with the sign bit of x or'd in, for every bf16
 *         x with |x| <= amax (|x / s| stays below 449, so no clamp is needed),
 *         against sampled amax values and every binade's edges.
 * Prints the mismatch counts; exit status 0 only when all are zero. */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static float f_of(uint32_t b) { float f; memcpy(&f, &b, 4); return f; }
static uint32_t b_of(float f) { uint32_t b; memcpy(&b, &f, 4); return b; }

/* Round-to-nearest-even e4m3 (bias 7, max 448) with saturation; NaN -> 0x7F. */
static uint8_t e4m3(float v) {
  if (isnan(v)) return 0x7F;
  const uint8_t sign = signbit(v) ? 0x80 : 0x00;
  double a = fabs((double)v);
  if (a >= 448.0) return sign | 0x7E;
  if (a < 0x1p-6) return sign | (uint8_t)nearbyint(a * 512.0); /* subnormal step 2^-9; 8 -> 0x08 */
  int e;
  double m = frexp(a, &e); /* a = m * 2^e, m in [0.5, 1) */
  e -= 1;
  m *= 2.0;
  double mm = nearbyint((m - 1.0) * 8.0);
  if (mm == 8.0) { mm = 0.0; e += 1; }
  if (e > 8 || (e == 8 && mm > 6.0)) return sign | 0x7E;
  return sign | (uint8_t)(((e + 7) << 3) | (int)mm);
}

/* min / max that return the other operand when one is any NaN (quiet or
 * signalling), as the GPU's min.f32 / min.bf16x2 and numpy's fmin do; C's
 * fminf returns NaN for a signalling NaN operand. */
static float min_nn(float a, float b) { return isnan(a) ? b : isnan(b) ? a : (a < b ? a : b); }
static float max_nn(float a, float b) { return isnan(a) ? b : isnan(b) ? a : (a > b ? a : b); }

static uint8_t ref_byte(float x, float s) {
  float t = x / s;
  t = min_nn(t, 448.0f);
  t = max_nn(-448.0f, t);
  return e4m3(t);
}

static float bound_bf16(float s) {
  uint32_t b = b_of(s * 1024.0f);
  if (b & 0xFFFFu) b += 0x10000u;
  return f_of(b & 0xFFFF0000u);
}

static float markstein_q1(float x, float s, float r) {
  const float q0 = x * r;
  const float e = fmaf(q0, -s, x);
  return fmaf(e, r, q0);
}

static uint8_t new_byte(float x, float s, float r, float lb) {
  float xc = min_nn(x, lb);
  xc = max_nn(xc, -lb);
  const float q1 = markstein_q1(xc, s, r);
  return e4m3(f_of((b_of(q1) & 0x7FFFFFFFu) | (b_of(xc) & 0x80000000u)));
}

static uint8_t fast_byte(float x, float s, float r) {
  return e4m3(markstein_q1(x, s, r)) | (signbit(x) ? 0x80 : 0x00);
}

int main(int argc, char** argv) {
  const uint32_t stride2 = argc > 1 ? (uint32_t)atoi(argv[1]) : 997u;
  const uint32_t stride3 = argc > 2 ? (uint32_t)atoi(argv[2]) : 65521u;
  const uint32_t stride4 = argc > 3 ? (uint32_t)atoi(argv[3]) : 5u;
  long long bad1 = 0, bad2 = 0, bad3 = 0, bad4 = 0, n1 = 0, n2 = 0, n3 = 0, n4 = 0;
#pragma omp parallel for reduction(+ : bad1, n1) schedule(static)
  for (uint32_t sm = 0; sm < (1u << 23); ++sm) {
    const float s = f_of(0x3F800000u | sm);
    const float r = 1.0f / s;
    for (uint32_t a = 0; a < 128; ++a) {
      const float x = f_of(0x3F800000u | (a << 16));
      bad1 += b_of(markstein_q1(x, s, r)) != b_of(x / s);
      n1++;
    }
  }
  static const int es_list[] = {-60, -59, -40, -1, 0, 1, 37, 99};
  for (int ie = 0; ie < (int)(sizeof es_list / sizeof es_list[0]); ++ie) {
    const int es = es_list[ie];
    for (int k = -40; k <= 12; ++k) {
      const int ex = es + k;
      if (ex < -133 || ex > 127) continue;
#pragma omp parallel for reduction(+ : bad2, n2) schedule(static)
      for (uint32_t sm = 0; sm < (1u << 23); sm += stride2) {
        const float s = ldexpf(f_of(0x3F800000u | sm), es);
        const float r = 1.0f / s;
        for (uint32_t a = 0; a < 256; ++a) {
          float x = ldexpf(f_of(0x3F800000u | ((a & 127u) << 16)), ex);
          if (a & 128u) x = -x;
          if (fabsf(x * r) < 0x1p-11f) continue;
          bad2 += b_of(markstein_q1(x, s, r)) != b_of(x / s);
          n2++;
        }
      }
    }
  }
  for (int es = -60; es <= 100; ++es) {
#pragma omp parallel for reduction(+ : bad3, n3) schedule(static)
    for (uint32_t sm = 0; sm < (1u << 23); sm += stride3) {
      const float s = ldexpf(f_of(0x3F800000u | sm), es);
      if (s > 0x1p100f) continue;
      const float r = 1.0f / s, lb = bound_bf16(s);
      for (uint32_t xb = 0; xb < 65536u; ++xb) {
        const float x = f_of(xb << 16);
        bad3 += new_byte(x, s, r, lb) != ref_byte(x, s);
        n3++;
      }
    }
  }
#pragma omp parallel for reduction(+ : bad4, n4) schedule(dynamic, 64)
  for (uint32_t ab = 1; ab <= 0x7F7Fu; ++ab) {
    if (ab % stride4 != 0 && (ab & 0x7Fu) != 0 && (ab & 0x7Fu) != 0x7Fu && ab != 0x7F7Fu) continue;
    const float amax = f_of(ab << 16);
    const float s = amax / 448.0f;
    if (!(s >= 0x1p-60f && s <= 0x1p100f)) continue;
    const float r = 1.0f / s;
    for (uint32_t xb = 0; xb < 65536u; ++xb) {
      const float x = f_of(xb << 16);
      if (isnan(x) || fabsf(x) > amax) continue;
      bad4 += fast_byte(x, s, r) != ref_byte(x, s);
      n4++;
    }
  }
  printf("pairs %lld mismatches %lld; exponent sweep %lld mismatches %lld; bytes %lld mismatches %lld; "
         "no-clamp bytes %lld mismatches %lld\n", n1, bad1, n2, bad2, n3, bad3, n4, bad4);
  return (bad1 == 0 && bad2 == 0 && bad3 == 0 && bad4 == 0) ? 0 : 1;
}
