/* gelu_table_gen.c -- writes gelu_table.inc, the coefficient table of the
 * sm_100a gelu kernel (activation_f64.cu, GeluOp).
 *
 * gelu(x) = (x / 2) erfc(-x / sqrt 2), with the argument rounded as the
 * formula is written: u = RN(|x| * RN(1 / sqrt 2)).  The kernel evaluates
 * erfc(u) / 2 = R(u) e^{-u^2}, where R(u) = erfc(u) e^{u^2} / 2 is smooth on
 * [0, 28.5] (R(0) = 1/2, R(u) ~ 1 / (2 u sqrt pi) for large u; beyond 27.3
 * erfc underflows).  [0, 28.5) is cut into 228 intervals of width 1/8; on
 * interval j, with t = 16 u - (2 j + 1) in [-1, 1], R is a degree-9
 * polynomial in t: the Chebyshev interpolant at 10 Chebyshev nodes,
 * computed in long double from the C library's erfcl and expl, turned into
 * monomial coefficients and rounded to double.  Row j holds the 10
 * coefficients from t^0 up: five 16-byte pairs.
 *
 * It also prints the worst relative error of the rounded polynomials,
 * evaluated as the kernel does (Horner in fma), against R in long double.
 *
 *   gcc -O2 -o /tmp/gelu_table_gen gelu_table_gen.c -lm &&
 *     /tmp/gelu_table_gen > gelu_table.inc
 */
#define _GNU_SOURCE
#include <math.h>
#include <stdio.h>

#define INTERVALS 228
#define DEGREE 9
#define ROW 10

typedef long double ld;

static ld r_of(ld u) { return 0.5L * erfcl(u) * expl(u * u); }

int main(void) {
  static double table[INTERVALS][ROW];
  const int n = DEGREE + 1;
  double worst = 0.0;
  for (int j = 0; j < INTERVALS; ++j) {
    const ld center = (j + 0.5L) / 8.0L, half = 1.0L / 16.0L;
    ld f[DEGREE + 1], cheb[DEGREE + 1], mono[DEGREE + 1];
    for (int i = 0; i < n; ++i)
      f[i] = r_of(center + half * cosl(M_PIl * (i + 0.5L) / n));
    for (int k = 0; k < n; ++k) {
      ld sum = 0.0L;
      for (int i = 0; i < n; ++i)
        sum += f[i] * cosl(M_PIl * k * (i + 0.5L) / n);
      cheb[k] = (k ? 2.0L : 1.0L) * sum / n;
    }
    /* T_k(t) in monomials: T_0 = 1, T_1 = t, T_k = 2 t T_{k-1} - T_{k-2}. */
    ld t_poly[DEGREE + 1][DEGREE + 1] = {{0.0L}};
    t_poly[0][0] = 1.0L;
    t_poly[1][1] = 1.0L;
    for (int k = 2; k < n; ++k)
      for (int i = 0; i < n; ++i)
        t_poly[k][i] = (i ? 2.0L * t_poly[k - 1][i - 1] : 0.0L) - t_poly[k - 2][i];
    for (int i = 0; i < n; ++i) {
      mono[i] = 0.0L;
      for (int k = 0; k < n; ++k)
        mono[i] += cheb[k] * t_poly[k][i];
      table[j][i] = (double)mono[i];
    }
    for (int q = 0; q <= 256; ++q) {
      const double t = -1.0 + q / 128.0;
      double p = table[j][DEGREE];
      for (int k = DEGREE - 1; k >= 0; --k)
        p = fma(p, t, table[j][k]);
      const ld ref = r_of(center + half * (ld)t);
      const double e = (double)fabsl(((ld)p - ref) / ref);
      if (e > worst)
        worst = e;
    }
  }
  printf("// gelu_table.inc -- written by gelu_table_gen.c; do not edit.\n");
  printf("// R(u) = erfc(u) e^{u^2} / 2 on [j/8, (j+1)/8), j = 0..%d: degree-%d\n",
         INTERVALS - 1, DEGREE);
  printf("// polynomials in t = 16 u - (2 j + 1), coefficients from t^0 up.\n");
  printf("// Worst relative error of the rounded polynomials in fma Horner\n");
  printf("// against R in long double: %.3e.\n", worst);
  for (int j = 0; j < INTERVALS; ++j) {
    printf("{");
    for (int i = 0; i < ROW; ++i)
      printf("%a%s", table[j][i], i + 1 < ROW ? ", " : "");
    printf("},\n");
  }
  return 0;
}
