/*
 * hexir_oracle.c -- CPU oracle for the hexir hot path.  TEST INFRASTRUCTURE
 * ONLY: used by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
 * leg as the checker or the timed reference.  No product code path calls it.
 *
 * A plain-C restatement of the reference runtime's CPU kernels
 * (runtime/src/kernels/reference_kernels.c):
 *
 *   oracle_matmul_f64   <- hexir_ref_matmul_f64, lines 3-13:
 *                          c[i*n+j] = sum over p = 0..k-1 of a[i*k+p]*b[p*n+j],
 *                          accumulated left to right from 0.0 with a separate
 *                          multiply and add (compile with -ffp-contract=off).
 *   oracle_add_f64      <- hexir_ref_add_f64, lines 15-18: c = a + b.
 *   oracle_relu_f64     <- hexir_ref_relu_f64, lines 20-23: x > 0 ? x : 0.
 *
 * and the activations the reference dialect declares but never lowers
 * (include/hexir/Dialect/Hexir/IR/HexirOps.td:189-308), from their op
 * descriptions, so parity for them is unpinned (no reference kernel, test or
 * golden value exists):
 *
 *   oracle_activation_f64(kind, ...)   kind = program.h kernel kind 7-14
 *     7  leaky_relu  "max(x, alpha * x)":          x > 0 ? x : 0.01 * x
 *     8  elu         "x if x > 0, else alpha * (exp(x) - 1)":
 *                                                  x > 0 ? x : 1.0 * expm1(x)
 *     9  sigmoid     "1 / (1 + exp(-x))"
 *     10 tanh        "tanh(x)"
 *     11 softmax     "normalizes values along the last dimension so that they
 *                    sum to 1": exp(x - rowmax) / sum, summed left to right
 *     12 gelu        "x * 0.5 * (1 + erf(x / sqrt(2)))", as
 *                    (0.5 * x) * erfc(-x * (1 / sqrt 2))
 *     13 swish       "x * sigmoid(x)", as x / (1 + exp(-x))
 *     14 mish        "x * tanh(softplus(x))", softplus(x) = x > 0 ?
 *                    x + log1p(exp(-x)) : log1p(exp(x))
 *
 * The ops carry no alpha, so leaky_relu and elu use the fixed 0.01 and 1.0.
 * The rewritten forms are equal in exact arithmetic and keep the relative
 * accuracy the literal ones lose (1 + erf(x) for negative x, log(1 + e^x)).
 *
 * The matmul may split ROWS over threads; every element keeps the reference's
 * sequential p order, so the result is bit-identical to the single-threaded
 * reference (pinned by tests/test_oracle.py against the reference library
 * built from its sources, oracle/_ref, and against tests/golden fixtures).
 */
#include <math.h>
#include <pthread.h>
#include <stddef.h>
#include <stdint.h>

void oracle_matmul_rows_f64(const double *a, const double *b, double *c,
                            uint32_t row_begin, uint32_t row_end, uint32_t n,
                            uint32_t k) {
  for (uint32_t i = row_begin; i < row_end; ++i) {
    for (uint32_t j = 0; j < n; ++j) {
      double acc = 0.0;
      for (uint32_t p = 0; p < k; ++p)
        acc += a[(size_t)i * k + p] * b[(size_t)p * n + j];
      c[(size_t)i * n + j] = acc;
    }
  }
}

typedef struct {
  const double *a, *b;
  double *c;
  uint32_t r0, r1, n, k;
} rows_job_t;

static void *rows_worker(void *arg) {
  rows_job_t *job = (rows_job_t *)arg;
  oracle_matmul_rows_f64(job->a, job->b, job->c, job->r0, job->r1, job->n,
                         job->k);
  return NULL;
}

void oracle_matmul_f64(const double *a, const double *b, double *c, uint32_t m,
                       uint32_t n, uint32_t k, int threads) {
  if (threads < 1)
    threads = 1;
  if ((uint32_t)threads > m)
    threads = m ? (int)m : 1;
  if (threads == 1) {
    oracle_matmul_rows_f64(a, b, c, 0, m, n, k);
    return;
  }
  enum { MAX_THREADS = 256 };
  if (threads > MAX_THREADS)
    threads = MAX_THREADS;
  pthread_t tid[MAX_THREADS];
  int joined[MAX_THREADS];
  rows_job_t jobs[MAX_THREADS];
  uint32_t per = (m + (uint32_t)threads - 1) / (uint32_t)threads;
  int count = 0;
  for (int t = 0; t < threads; ++t) {
    uint32_t r0 = (uint32_t)t * per;
    uint32_t r1 = r0 + per > m ? m : r0 + per;
    if (r0 >= r1)
      break;
    jobs[t] = (rows_job_t){a, b, c, r0, r1, n, k};
    joined[t] = pthread_create(&tid[t], NULL, rows_worker, &jobs[t]) == 0;
    if (!joined[t])
      rows_worker(&jobs[t]); /* no thread: do these rows here */
    count = t + 1;
  }
  for (int t = 0; t < count; ++t)
    if (joined[t])
      pthread_join(tid[t], NULL);
}

void oracle_add_f64(const double *a, const double *b, double *c, size_t n) {
  for (size_t i = 0; i < n; ++i)
    c[i] = a[i] + b[i];
}

void oracle_relu_f64(const double *x, double *y, size_t n) {
  for (size_t i = 0; i < n; ++i)
    y[i] = x[i] > 0.0 ? x[i] : 0.0;
}

static double oracle_softplus(double x) {
  return x > 0.0 ? x + log1p(exp(-x)) : log1p(exp(x));
}

/* Returns 0, or -1 for a kind that is not an activation. */
int oracle_activation_f64(uint32_t kind, const double *x, double *y,
                          uint64_t rows, uint64_t cols) {
  const uint64_t n = rows * cols;
  switch (kind) {
  case 7:
    for (uint64_t i = 0; i < n; ++i)
      y[i] = x[i] > 0.0 ? x[i] : 0.01 * x[i];
    return 0;
  case 8:
    for (uint64_t i = 0; i < n; ++i)
      y[i] = x[i] > 0.0 ? x[i] : 1.0 * expm1(x[i]);
    return 0;
  case 9:
    for (uint64_t i = 0; i < n; ++i)
      y[i] = 1.0 / (1.0 + exp(-x[i]));
    return 0;
  case 10:
    for (uint64_t i = 0; i < n; ++i)
      y[i] = tanh(x[i]);
    return 0;
  case 11:
    for (uint64_t r = 0; r < rows; ++r) {
      const double *xr = x + r * cols;
      double *yr = y + r * cols;
      double m = -HUGE_VAL, s = 0.0;
      for (uint64_t j = 0; j < cols; ++j)
        if (xr[j] > m)
          m = xr[j];
      for (uint64_t j = 0; j < cols; ++j) {
        yr[j] = exp(xr[j] - m);
        s += yr[j];
      }
      for (uint64_t j = 0; j < cols; ++j)
        yr[j] /= s;
    }
    return 0;
  case 12:
    for (uint64_t i = 0; i < n; ++i)
      y[i] = (0.5 * x[i]) * erfc(-x[i] * 0.70710678118654752440);
    return 0;
  case 13:
    for (uint64_t i = 0; i < n; ++i)
      y[i] = x[i] / (1.0 + exp(-x[i]));
    return 0;
  case 14:
    for (uint64_t i = 0; i < n; ++i)
      y[i] = x[i] * tanh(oracle_softplus(x[i]));
    return 0;
  }
  return -1;
}
