/* tanh_accuracy.c -- the arithmetic of the sm_100a tanh and gelu kernels
 * and of the exp / expm1 core they share with elu and mish
 * (hexir_b200/csrc/kernels/activation_f64.cu), restated in C with
 * fma() standing for the GPU's DFMA, checked against the C library's
 * 64-bit-mantissa tanhl.  The reciprocal estimate is modelled by a
 * reciprocal truncated to SEED_BITS bits (argv[1]); one Newton step and the
 * quotient correction follow, as on the GPU.
 *
 * Prints: worst ulp error against tanhl, worst ulp difference from the
 * double tanh, and the number of special values that differ from tanh's
 * sign and saturation rules.  Test infrastructure for
 * tests/test_tanh_accuracy.py. */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static double from_bits(uint64_t b) { double d; memcpy(&d, &b, 8); return d; }
static uint64_t to_bits(double d) { uint64_t b; memcpy(&b, &d, 8); return b; }

static int seed_bits = 20;

static double rcp_estimate(double d) {
  uint64_t b = to_bits(1.0 / d);
  b &= ~((1ull << (52 - seed_bits)) - 1);
  return from_bits(b);
}

/* exp_neg and expm1_neg of activation_f64.cu (the core of kernel_tanh):
 * e^z and expm1(z) for z <= 0. */
static double neg_exp_parts(double z, int32_t *k) {
  const double shifter = 0x1.8p52;
  const double t = fma(z, 0x1.71547652b82fep+0, shifter);
  const double kd = t - shifter;
  *k = (int32_t)(uint32_t)to_bits(t);
  double r = fma(-kd, 0x1.62e42fefa39efp-1, z);
  r = fma(-kd, 0x1.abc9e3b39803fp-56, r);
  double q = 0x1.6124613a86d09p-33;
  q = fma(q, r, 0x1.1eed8eff8d898p-29);
  q = fma(q, r, 0x1.ae64567f544e4p-26);
  q = fma(q, r, 0x1.27e4fb7789f5cp-22);
  q = fma(q, r, 0x1.71de3a556c734p-19);
  q = fma(q, r, 0x1.a01a01a01a01ap-16);
  q = fma(q, r, 0x1.a01a01a01a01ap-13);
  q = fma(q, r, 0x1.6c16c16c16c17p-10);
  q = fma(q, r, 0x1.1111111111111p-7);
  q = fma(q, r, 0x1.5555555555555p-5);
  q = fma(q, r, 0x1.5555555555555p-3);
  q = fma(q, r, 0.5);
  return fma(r * r, q, r);
}
static double pow2i(int32_t k) {
  return from_bits((uint64_t)(uint32_t)(k + 1023) << 52);
}
static double exp_neg(double z) {
  int32_t k;
  const double p = neg_exp_parts(z < -746.0 ? -746.0 : z, &k);
  const int32_t k1 = k >> 1;
  return ((1.0 + p) * pow2i(k1)) * pow2i(k - k1);
}
static double expm1_neg(double z) {
  int32_t k;
  const double p = neg_exp_parts(z < -40.0 ? -40.0 : z, &k);
  const double s = pow2i(k);
  return fma(s, p, s - 1.0);
}

/* GeluOp of activation_f64.cu with its table. */
static const double gelu_table[228][10] = {
#include "../hexir_b200/csrc/kernels/gelu_table.inc"
};
static double kernel_gelu(double x) {
  const double u0 = fabs(x) * 0.70710678118654752440;
  const double u = u0 > 28.5 ? 28.5 : u0;
  int j = isnan(u) ? 0 : (int)(u * 8.0);
  j = j < 0 ? 0 : (j > 227 ? 227 : j);
  const double t = fma(u, 16.0, -(double)(2 * j + 1));
  const double *c = gelu_table[j];
  double p = fma(c[9], t, c[8]);
  for (int k = 7; k >= 0; --k)
    p = fma(p, t, c[k]);
  const double uu = u * u, lo = fma(u, u, -uu);
  double e = exp_neg(-uu);
  e = fma(-lo, e, e);
  const double q = p * e;
  return x * (x < 0.0 ? q : 1.0 - q);
}

static double kernel_tanh(double x) {
  const double ax = fabs(x);
  const double y = ax > 20.0 ? 20.0 : ax;
  const double z = -2.0 * y;
  const double shifter = 0x1.8p52;
  const double t = fma(z, 0x1.71547652b82fep+0, shifter);
  const double kd = t - shifter;
  const int32_t k = (int32_t)(uint32_t)to_bits(t);
  double r = fma(-kd, 0x1.62e42fefa39efp-1, z);
  r = fma(-kd, 0x1.abc9e3b39803fp-56, r);
  double q = 0x1.6124613a86d09p-33;
  q = fma(q, r, 0x1.1eed8eff8d898p-29);
  q = fma(q, r, 0x1.ae64567f544e4p-26);
  q = fma(q, r, 0x1.27e4fb7789f5cp-22);
  q = fma(q, r, 0x1.71de3a556c734p-19);
  q = fma(q, r, 0x1.a01a01a01a01ap-16);
  q = fma(q, r, 0x1.a01a01a01a01ap-13);
  q = fma(q, r, 0x1.6c16c16c16c17p-10);
  q = fma(q, r, 0x1.1111111111111p-7);
  q = fma(q, r, 0x1.5555555555555p-5);
  q = fma(q, r, 0x1.5555555555555p-3);
  q = fma(q, r, 0.5);
  const double p = fma(r * r, q, r);
  const double s = from_bits((uint64_t)(uint32_t)(k + 1023) << 52);
  const double u = fma(s, p, s - 1.0);
  const double d = 2.0 + u;
  const double n = -u;
  double rc = rcp_estimate(d);
  rc = fma(rc, fma(-d, rc, 1.0), rc);
  const double q0 = n * rc;
  return copysign(fma(rc, fma(-d, q0, n), q0), x);
}

/* |got - want| in units of the last place of the double nearest want. */
static double ulp_error(double got, long double want) {
  const double w = (double)want;
  if (isnan(w))
    return isnan(got) ? 0.0 : INFINITY;
  double ulp = nextafter(fabs(w), INFINITY) - fabs(w);
  if (!(ulp > 0))
    ulp = 0x1p-1074;
  return (double)(fabsl((long double)got - want) / ulp);
}

static uint64_t state = 0x2545F4914F6CDD1Dull;
static uint64_t next(void) {
  state ^= state << 13;
  state ^= state >> 7;
  state ^= state << 17;
  return state;
}
static double uniform(void) { return (double)(next() >> 11) * 0x1p-53; }
static double normal(void) {
  double a = uniform(), b = uniform();
  if (a < 1e-300)
    a = 1e-300;
  return sqrt(-2.0 * log(a)) * cos(6.283185307179586 * b);
}

/* argv[1] == "exp": worst ulp errors of exp_neg against expl and of
 * expm1_neg against expm1l over z in [-750, 0]. */
static int exp_main(long n) {
  double worst_exp = 0.0, worst_expm1 = 0.0;
  for (int kind = 0; kind < 4; ++kind)
    for (long i = 0; i < n; ++i) {
      double z;
      switch (kind) {
      case 0: z = -750.0 * uniform(); break;               /* to underflow */
      case 1: z = -(708.0 + 38.0 * uniform()); break;      /* subnormal results */
      case 2: z = -45.0 * uniform(); break;
      default: z = -ldexp(uniform(), -(int)(next() % 1070)); /* tiny */
      }
      const double e = ulp_error(exp_neg(z), expl((long double)z));
      const double m = ulp_error(expm1_neg(z), expm1l((long double)z));
      if (e > worst_exp)
        worst_exp = e;
      if (m > worst_expm1)
        worst_expm1 = m;
    }
  printf("%.4f %.4f\n", worst_exp, worst_expm1);
  return 0;
}

/* argv[1] == "gelu": worst ulp errors of kernel_gelu against the formula
 * as written, (x / 2) erfc(-RN(x RN(1 / sqrt 2))), evaluated in long
 * double, and against the same formula in double with the C library's
 * erfc (the oracle's evaluation), results within 2^-1000 of the reference
 * counting as exact; then the special values that differ from the double
 * formula's. */
static int gelu_main(long n) {
  double worst = 0.0, worst_libm = 0.0;
  for (int kind = 0; kind < 5; ++kind)
    for (long i = 0; i < n; ++i) {
      double x;
      switch (kind) {
      case 0: x = normal(); break;
      case 1: x = (2.0 * uniform() - 1.0) * 45.0; break;
      case 2: x = -40.0 * uniform(); break;
      case 3: x = ldexp(2.0 * uniform() - 1.0, -(int)(next() % 1070)); break;
      default: x = (2.0 * uniform() - 1.0) * 3.0;
      }
      const double g = kernel_gelu(x);
      const double arg = -x * 0.70710678118654752440;
      const long double exact = 0.5L * (long double)x * erfcl((long double)arg);
      const double libm = (0.5 * x) * erfc(arg);
      /* Below 2^-1000 only the absolute error counts, as in the GPU tests:
       * near the subnormals e^{-u^2} carries fewer bits. */
      const double e = fabsl((long double)g - exact) <= 0x1p-1000L
                           ? 0.0 : ulp_error(g, exact);
      const double el = fabs(g - libm) <= 0x1p-1000
                            ? 0.0 : ulp_error(g, (long double)libm);
      if (e > worst)
        worst = e;
      if (el > worst_libm)
        worst_libm = el;
    }
  const double specials[] = {0.0, -0.0, 0x1p-1074, -0x1p-1074, 40.0, -40.0,
                             1e300, -1e300, INFINITY, -INFINITY, NAN};
  int bad = 0;
  for (unsigned i = 0; i < sizeof specials / sizeof *specials; ++i) {
    const double x = specials[i], g = kernel_gelu(x);
    const double want = (0.5 * x) * erfc(-x * 0.70710678118654752440);
    bad += !(isnan(want) ? isnan(g) : to_bits(g) == to_bits(want));
  }
  printf("%.4f %.4f %d\n", worst, worst_libm, bad);
  return 0;
}

int main(int argc, char **argv) {
  if (argc > 1 && strcmp(argv[1], "gelu") == 0)
    return gelu_main(argc > 2 ? atol(argv[2]) : 200000);
  if (argc > 1 && strcmp(argv[1], "exp") == 0)
    return exp_main(argc > 2 ? atol(argv[2]) : 200000);
  if (argc > 1)
    seed_bits = atoi(argv[1]);
  const long per_kind = argc > 2 ? atol(argv[2]) : 200000;
  double worst = 0.0, worst_libm = 0.0;
  for (int kind = 0; kind < 5; ++kind)
    for (long i = 0; i < per_kind; ++i) {
      double x;
      switch (kind) {
      case 0: x = normal(); break;
      case 1: x = (2.0 * uniform() - 1.0) * 25.0; break;
      case 2: x = (2.0 * uniform() - 1.0) * 0.6; break;
      case 3: x = ldexp(2.0 * uniform() - 1.0, -(int)(next() % 1070)); break;
      default: x = (2.0 * uniform() - 1.0) * 0.3 + ((next() & 1) ? 0.17 : -0.17);
      }
      const double g = kernel_tanh(x);
      const double e = ulp_error(g, tanhl((long double)x));
      const double el = ulp_error(g, (long double)tanh(x));
      if (e > worst)
        worst = e;
      if (el > worst_libm)
        worst_libm = el;
    }
  const double specials[] = {0.0, -0.0, 0x1p-1074, -0x1p-1074, 20.0, -20.0,
                             20.5, 700.0, -1e300, INFINITY, -INFINITY, NAN};
  int bad = 0;
  for (unsigned i = 0; i < sizeof specials / sizeof *specials; ++i) {
    const double x = specials[i], g = kernel_tanh(x);
    const int same = isnan(x) ? isnan(g) : to_bits(g) == to_bits(tanh(x));
    bad += !same;
  }
  printf("%.4f %.4f %d\n", worst, worst_libm, bad);
  return 0;
}
