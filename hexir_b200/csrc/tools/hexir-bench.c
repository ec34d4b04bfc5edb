/*
 * hexir-bench -- time a module end to end and kernel only, check it, and
 * time cuBLAS on the same inputs.
 *
 * Keeps the reference tool's behaviour (bench/hexir-bench.c:123-426): the
 * first executable defines the reported shape, one untimed run whose output
 * is checked on 512 sampled elements (relative error bar 1e-12 * k, scale
 * max(|expected|, 1)), wall-clock timing of whole hexir_execute calls
 * (allocation, host->device copies, kernels, synchronisation), and a
 * kernel-only cuBLAS Dgemm on the same RODATA as the vendor line.
 *
 * Additions: the device time of the dispatches themselves (CUDA events on
 * the launching stream), --devices=N for sharded modules, --json for one
 * machine-readable line, and the relu of a matmul_relu executable applied in
 * the sampled check.
 */
#define _POSIX_C_SOURCE 200809L
#include <dlfcn.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "hexir_runtime/runtime.h"

static double now_seconds(void) {
  struct timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return (double)ts.tv_sec + (double)ts.tv_nsec * 1e-9;
}

static double gflops(uint32_t m, uint32_t n, uint32_t k, double seconds) {
  return seconds > 0.0 ? 2.0 * m * n * k / seconds / 1e9 : 0.0;
}

static int executable_at(const hexir_module_t *module, uint64_t index,
                         hexir_executable_entry_t *out) {
  const void *data = NULL;
  uint64_t size = 0;
  if (hexir_module_section(module, HEXIR_SECTION_EXECUTABLES, &data, &size) !=
      HEXIR_OK)
    return 0;
  hexir_executable_header_t header;
  if (size < sizeof(header))
    return 0;
  memcpy(&header, data, sizeof(header));
  if (index >= header.count ||
      sizeof(header) + (index + 1) * sizeof(*out) > size)
    return 0;
  memcpy(out, (const uint8_t *)data + sizeof(header) + index * sizeof(*out),
         sizeof(*out));
  return 1;
}

static int first_executable(const hexir_module_t *module,
                            hexir_executable_entry_t *out) {
  return executable_at(module, 0, out);
}

/* The last DISPATCH of "main" (whose destination hexir_execute_capture
 * returns): its executable index, and for each input that a CONST defines, a
 * pointer to the constant in RODATA (NULL for computed inputs).  When its
 * first input was computed by an earlier DISPATCH, *producer receives that
 * dispatch's executable index and producer_in its constant inputs (a relu
 * over an unfused linear).  -1 when the program cannot be read. */
static int64_t last_dispatch_inputs(const hexir_module_t *module,
                                    const double *in[3], int64_t *producer,
                                    const double *producer_in[3]) {
  const void *sym = NULL, *prog = NULL, *ro = NULL;
  uint64_t sym_size = 0, prog_size = 0, ro_size = 0;
  if (hexir_module_section(module, HEXIR_SECTION_SYMBOLS, &sym, &sym_size) !=
          HEXIR_OK ||
      hexir_module_section(module, HEXIR_SECTION_PROGRAM, &prog, &prog_size) !=
          HEXIR_OK)
    return -1;
  if (hexir_module_section(module, HEXIR_SECTION_RODATA, &ro, &ro_size) !=
      HEXIR_OK)
    ro_size = 0;
  uint64_t pc = UINT64_MAX;
  for (uint64_t i = 0; (i + 1) * sizeof(hexir_symbol_entry_t) <= sym_size; ++i) {
    hexir_symbol_entry_t e;
    memcpy(&e, (const uint8_t *)sym + i * sizeof(e), sizeof(e));
    if (strncmp(e.name, "main", HEXIR_NAME_SIZE) == 0) {
      pc = e.program_offset;
      break;
    }
  }
  if (pc == UINT64_MAX)
    return -1;
  enum { kSlots = 256 };
  const double *slot_const[kSlots] = {0};
  int64_t slot_exe[kSlots];  /* the dispatch that wrote a slot, or -1 */
  const double *slot_in[kSlots][3];
  for (int i = 0; i < kSlots; ++i)
    slot_exe[i] = -1;
  int64_t last = -1;
  *producer = -1;
  while (pc + sizeof(hexir_command_header_t) <= prog_size) {
    hexir_command_header_t h;
    memcpy(&h, (const uint8_t *)prog + pc, sizeof(h));
    pc += sizeof(h);
    if (h.operand_count > 16 || pc + 8ull * h.operand_count > prog_size)
      return -1;
    uint64_t ops[16];
    memcpy(ops, (const uint8_t *)prog + pc, 8ull * h.operand_count);
    pc += 8ull * h.operand_count;
    if (h.kind == HEXIR_CMD_END)
      break;
    if (h.kind == HEXIR_CMD_CONST && h.operand_count == 3 && ops[0] < kSlots) {
      slot_const[ops[0]] = (ops[1] % 8 == 0 && ops[1] <= ro_size &&
                            ops[2] <= ro_size - ops[1])
                               ? (const double *)((const uint8_t *)ro + ops[1])
                               : NULL;
      slot_exe[ops[0]] = -1;
    }
    if (h.kind == HEXIR_CMD_ALLOC && h.operand_count == 2 && ops[0] < kSlots) {
      slot_const[ops[0]] = NULL;
      slot_exe[ops[0]] = -1;
    }
    if (h.kind == HEXIR_CMD_DISPATCH && h.operand_count >= 3) {
      const uint64_t argc = ops[1];
      if (argc + 2 != h.operand_count || argc > 4)
        return -1;
      last = (int64_t)ops[0];
      for (uint64_t a = 0; a < 3; ++a)
        in[a] = a + 1 < argc && ops[2 + a] < kSlots ? slot_const[ops[2 + a]]
                                                    : NULL;
      const uint64_t first = ops[2];
      *producer = first < kSlots ? slot_exe[first] : -1;
      if (first < kSlots && slot_exe[first] >= 0)
        for (int a = 0; a < 3; ++a)
          producer_in[a] = slot_in[first][a];
      const uint64_t dst = ops[2 + argc - 1];
      if (dst < kSlots) {
        slot_const[dst] = NULL;
        slot_exe[dst] = last;
        for (int a = 0; a < 3; ++a)
          slot_in[dst][a] = in[a];
      }
    }
  }
  return last;
}

/* ---- cuBLAS, loaded at run time -------------------------------------- */
typedef void *cublasHandle_t;
static struct {
  void *lib;
  int (*Create)(cublasHandle_t *);
  int (*Destroy)(cublasHandle_t);
  int (*SetStream)(cublasHandle_t, void *);
  int (*Dgemm)(cublasHandle_t, int, int, int, int, int, const double *,
               const double *, int, const double *, int, const double *,
               double *, int);
} cublas;

static int cublas_load(void) {
  const char *names[] = {"libcublas.so.12", "libcublas.so", "libcublas.so.13"};
  for (size_t i = 0; i < sizeof(names) / sizeof(names[0]) && !cublas.lib; ++i)
    cublas.lib = dlopen(names[i], RTLD_NOW | RTLD_LOCAL);
  if (!cublas.lib)
    return 0;
  *(void **)(&cublas.Create) = dlsym(cublas.lib, "cublasCreate_v2");
  *(void **)(&cublas.Destroy) = dlsym(cublas.lib, "cublasDestroy_v2");
  *(void **)(&cublas.SetStream) = dlsym(cublas.lib, "cublasSetStream_v2");
  *(void **)(&cublas.Dgemm) = dlsym(cublas.lib, "cublasDgemm_v2");
  return cublas.Create && cublas.Destroy && cublas.SetStream && cublas.Dgemm;
}

/* Sampled check against the first two RODATA constants (a, then w). */
/* Sampled check of got = epilogue(a . b [+ d]) in the reference's order:
 * the sum over k, rounded, then the add, then the relu. */
static int verify_sampled(const double *a, const double *b, const double *d,
                          const double *got, uint32_t m, uint32_t n, uint32_t k,
                          int relu, int samples, double *worst_out) {
  size_t total = (size_t)m * n, stride = total / (size_t)samples;
  if (stride == 0)
    stride = 1;
  double worst = 0.0;
  for (size_t index = 0; index < total; index += stride) {
    uint32_t i = (uint32_t)(index / n), j = (uint32_t)(index % n);
    double expected = 0.0;
    for (uint32_t p = 0; p < k; ++p)
      expected += a[(size_t)i * k + p] * b[(size_t)p * n + j];
    if (d)
      expected += d[index];
    if (relu)
      expected = expected > 0.0 ? expected : 0.0;
    double scale = fabs(expected) > 1.0 ? fabs(expected) : 1.0;
    double err = fabs(got[index] - expected) / scale;
    if (err > worst)
      worst = err;
  }
  *worst_out = worst;
  return worst <= 1e-12 * (double)(k ? k : 1);
}

static int usage(void) {
  fprintf(stderr,
          "usage: hexir-bench <module.hxb> [--device=cpu|cuda|cuda:N] "
          "[--devices=N]\n"
          "                   [--iters=N] [--no-baseline] [--no-verify] "
          "[--json]\n");
  return 2;
}

int main(int argc, char **argv) {
  const char *path = NULL;
  hexir_device_kind_t kind = HEXIR_DEVICE_CUDA;
  int ordinal = 0, device_count = 0, iterations = 20;
  int want_baseline = 1, want_verify = 1, json = 0;
  for (int i = 1; i < argc; ++i) {
    if (strcmp(argv[i], "--device=cpu") == 0) {
      kind = HEXIR_DEVICE_CPU;
    } else if (strcmp(argv[i], "--device=cuda") == 0) {
      kind = HEXIR_DEVICE_CUDA;
    } else if (strncmp(argv[i], "--device=cuda:", 14) == 0) {
      kind = HEXIR_DEVICE_CUDA;
      ordinal = atoi(argv[i] + 14);
    } else if (strncmp(argv[i], "--devices=", 10) == 0) {
      device_count = atoi(argv[i] + 10);
      if (device_count < 1 || device_count > 64)
        return usage();
    } else if (strncmp(argv[i], "--iters=", 8) == 0) {
      iterations = atoi(argv[i] + 8);
      if (iterations < 1)
        return usage();
    } else if (strcmp(argv[i], "--no-baseline") == 0) {
      want_baseline = 0;
    } else if (strcmp(argv[i], "--no-verify") == 0) {
      want_verify = 0;
    } else if (strcmp(argv[i], "--json") == 0) {
      json = 1;
    } else if (argv[i][0] == '-') {
      return usage();
    } else {
      path = argv[i];
    }
  }
  if (!path)
    return usage();

  hexir_module_t *module = NULL;
  hexir_status_t status = hexir_module_load_file(path, &module);
  if (status != HEXIR_OK) {
    fprintf(stderr, "hexir-bench: cannot load '%s': %s\n", path,
            hexir_status_string(status));
    return 1;
  }
  hexir_executable_entry_t entry;
  if (!first_executable(module, &entry)) {
    fprintf(stderr, "hexir-bench: module has no executable to measure\n");
    hexir_module_release(module);
    return 1;
  }
  const int is_gemm = entry.kind == HEXIR_KERNEL_MATMUL ||
                      entry.kind == HEXIR_KERNEL_MATMUL_RELU ||
                      entry.kind == HEXIR_KERNEL_MATMUL_ADD ||
                      entry.kind == HEXIR_KERNEL_MATMUL_ADD_RELU;
  if (!json) {
    printf("module   : %s\n", path);
    printf("kernel   : %.32s  %s  built for %s  %ux%ux%u  elem=%uB\n",
           entry.name, hexir_kernel_kind_string(entry.kind),
           entry.device == 1 ? "cuda" : "cpu", entry.m, entry.n, entry.k,
           entry.elem_size);
    printf("device   : %s\n", kind == HEXIR_DEVICE_CUDA ? "cuda" : "cpu");
    printf("iters    : %d\n\n", iterations);
  }

  hexir_device_t *devices[64] = {0};
  int opened = 0;
  if (kind == HEXIR_DEVICE_CUDA && device_count > 0) {
    for (; opened < device_count; ++opened)
      if ((status = hexir_device_create_cuda(opened, &devices[opened])) !=
          HEXIR_OK)
        break;
  } else {
    status = kind == HEXIR_DEVICE_CUDA && ordinal > 0
                 ? hexir_device_create_cuda(ordinal, &devices[0])
                 : hexir_device_create(kind, &devices[0]);
    opened = status == HEXIR_OK;
  }
  if (status != HEXIR_OK) {
    fprintf(stderr, "hexir-bench: device create failed: %s\n",
            hexir_status_string(status));
    hexir_module_release(module);
    return 1;
  }

  size_t result_elems = (size_t)entry.m * entry.n;
  double *result = want_verify ? malloc(result_elems * sizeof(double)) : NULL;
  /* Untimed first run: context, module load; the run whose output is checked. */
  status = device_count > 0
               ? hexir_execute_devices(module, devices, (unsigned)device_count,
                                       "main", result,
                                       result ? result_elems * 8 : 0)
               : hexir_execute_capture(module, devices[0], "main", result,
                                       result ? result_elems * 8 : 0);
  if (status != HEXIR_OK) {
    fprintf(stderr, "hexir-bench: execution failed: %s\n",
            hexir_status_string(status));
    free(result);
    for (int i = 0; i < opened; ++i)
      hexir_device_release(devices[i]);
    hexir_module_release(module);
    return 1;
  }
  double err = -1.0;
  int correct = 1;
  /* The captured result is the last DISPATCH's: check it when that is a
   * linear (fused or not) whose inputs are all constants. */
  const double *inputs[3] = {NULL, NULL, NULL}, *prod_in[3] = {NULL, NULL, NULL};
  hexir_executable_entry_t last, prod;
  int64_t prod_index = -1;
  const int64_t last_index =
      last_dispatch_inputs(module, inputs, &prod_index, prod_in);
  int over_linear = 0;  /* a relu of an unfused linear's result */
  if (result && last_index >= 0 &&
      executable_at(module, (uint64_t)last_index, &last) &&
      last.kind == HEXIR_KERNEL_RELU && prod_index >= 0 &&
      executable_at(module, (uint64_t)prod_index, &prod) &&
      prod.kind == HEXIR_KERNEL_MATMUL && prod.m == last.m && prod.n == last.n) {
    over_linear = 1;
    last = prod;
    last.kind = HEXIR_KERNEL_MATMUL_RELU;
    for (int a = 0; a < 3; ++a)
      inputs[a] = prod_in[a];
  }
  if (result && last_index >= 0 &&
      (over_linear || executable_at(module, (uint64_t)last_index, &last)) &&
      last.m == entry.m && last.n == entry.n) {
    const int add = last.kind == HEXIR_KERNEL_MATMUL_ADD ||
                    last.kind == HEXIR_KERNEL_MATMUL_ADD_RELU;
    const int gemm = add || last.kind == HEXIR_KERNEL_MATMUL ||
                     last.kind == HEXIR_KERNEL_MATMUL_RELU;
    if (gemm && inputs[0] && inputs[1] && (!add || inputs[2])) {
      correct = verify_sampled(inputs[0], inputs[1], add ? inputs[2] : NULL,
                               result, last.m, last.n, last.k,
                               last.kind == HEXIR_KERNEL_MATMUL_RELU ||
                                   last.kind == HEXIR_KERNEL_MATMUL_ADD_RELU,
                               512, &err);
      if (!json)
        printf("verify   : hexir max relative error %.3g over 512 sampled "
               "elements (%s)\n",
               err, correct ? "ok" : "WRONG");
    }
  }
  free(result);
  if (!correct)
    fprintf(stderr, "hexir-bench: the kernel produced the wrong answer; "
                    "timings below are meaningless\n");

  double kernel_ms = 0.0;
  double start = now_seconds();
  for (int i = 0; i < iterations && status == HEXIR_OK; ++i) {
    status = device_count > 0
                 ? hexir_execute_devices(module, devices,
                                         (unsigned)device_count, "main", NULL, 0)
                 : hexir_execute(module, devices[0], "main");
    kernel_ms += hexir_last_execute_kernel_ms();
  }
  double e2e = (now_seconds() - start) / iterations;
  kernel_ms /= iterations;
  if (status != HEXIR_OK) {
    fprintf(stderr, "hexir-bench: execution failed: %s\n",
            hexir_status_string(status));
    for (int i = 0; i < opened; ++i)
      hexir_device_release(devices[i]);
    hexir_module_release(module);
    return 1;
  }
  if (!json) {
    printf("hexir    : %8.3f ms", e2e * 1e3);
    if (is_gemm)
      printf("   %10.2f GFLOP/s", gflops(entry.m, entry.n, entry.k, e2e));
    printf("   (end to end)\n");
    if (kind == HEXIR_DEVICE_CUDA) {
      printf("kernels  : %8.3f ms", kernel_ms);
      if (is_gemm)
        printf("   %10.2f GFLOP/s",
               gflops(entry.m, entry.n, entry.k, kernel_ms * 1e-3));
      printf("   (device time of the dispatches)\n");
    }
  }

  double cublas_ms = -1.0;
  if (is_gemm && kind == HEXIR_DEVICE_CUDA && want_baseline && cublas_load()) {
    const void *rodata = NULL;
    uint64_t rodata_size = 0;
    size_t a_elems = (size_t)entry.m * entry.k, b_elems = (size_t)entry.k * entry.n;
    hexir_device_t *dev = devices[0];
    hexir_buffer_t *da = NULL, *db = NULL, *dc = NULL;
    cublasHandle_t handle = NULL;
    if (hexir_module_section(module, HEXIR_SECTION_RODATA, &rodata,
                             &rodata_size) == HEXIR_OK &&
        rodata_size >= (a_elems + b_elems) * 8 &&
        hexir_buffer_allocate(dev, a_elems * 8, HEXIR_MEMORY_DEVICE_LOCAL, &da) ==
            HEXIR_OK &&
        hexir_buffer_allocate(dev, b_elems * 8, HEXIR_MEMORY_DEVICE_LOCAL, &db) ==
            HEXIR_OK &&
        hexir_buffer_allocate(dev, result_elems * 8, HEXIR_MEMORY_DEVICE_LOCAL,
                              &dc) == HEXIR_OK &&
        hexir_buffer_write(da, rodata, a_elems * 8) == HEXIR_OK &&
        hexir_buffer_write(db, (const double *)rodata + a_elems, b_elems * 8) ==
            HEXIR_OK &&
        cublas.Create(&handle) == 0) {
      cublas.SetStream(handle, hexir_device_stream(dev));
      const double alpha = 1.0, beta = 0.0;
      const double *pa = hexir_buffer_device_pointer(da);
      const double *pb = hexir_buffer_device_pointer(db);
      double *pc = hexir_buffer_device_pointer(dc);
      /* Column-major B.A is the row-major A.B on the same buffers. */
      cublas.Dgemm(handle, 0, 0, (int)entry.n, (int)entry.m, (int)entry.k,
                   &alpha, pb, (int)entry.n, pa, (int)entry.k, &beta, pc,
                   (int)entry.n);
      hexir_device_wait(dev);
      double t0 = now_seconds();
      for (int i = 0; i < iterations; ++i)
        cublas.Dgemm(handle, 0, 0, (int)entry.n, (int)entry.m, (int)entry.k,
                     &alpha, pb, (int)entry.n, pa, (int)entry.k, &beta, pc,
                     (int)entry.n);
      hexir_device_wait(dev);
      cublas_ms = (now_seconds() - t0) / iterations * 1e3;
      if (!json)
        printf("cuBLAS   : %8.3f ms   %10.2f GFLOP/s   (kernel only)\n",
               cublas_ms, gflops(entry.m, entry.n, entry.k, cublas_ms * 1e-3));
    }
    if (handle)
      cublas.Destroy(handle);
    hexir_buffer_release(da);
    hexir_buffer_release(db);
    hexir_buffer_release(dc);
  }
  if (json)
    printf("{\"module\": \"%s\", \"kernel\": \"%s\", \"m\": %u, \"n\": %u, "
           "\"k\": %u, \"iters\": %d, \"e2e_ms\": %.6f, \"kernel_ms\": %.6f, "
           "\"gflops_e2e\": %.3f, \"gflops_kernel\": %.3f, \"cublas_ms\": %.6f, "
           "\"verify_max_rel_err\": %.3g, \"verify_ok\": %s}\n",
           path, hexir_kernel_kind_string(entry.kind), entry.m, entry.n,
           entry.k, iterations, e2e * 1e3, kernel_ms,
           is_gemm ? gflops(entry.m, entry.n, entry.k, e2e) : 0.0,
           is_gemm && kernel_ms > 0 ? gflops(entry.m, entry.n, entry.k,
                                             kernel_ms * 1e-3)
                                    : 0.0,
           cublas_ms, err, correct ? "true" : "false");
  for (int i = 0; i < opened; ++i)
    hexir_device_release(devices[i]);
  hexir_module_release(module);
  return correct ? 0 : 1;
}
