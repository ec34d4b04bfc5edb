/*
 * hexir-run -- load a .hxb module and run an entry point, no compiler in the
 * process.
 *
 * Command line and output are those of the reference tool
 * (runtime/tools/hexir-run/hexir-run.c:17-143): the module report (version,
 * sections, device), results of PRINT on stdout, "--quiet" for results only,
 * "--selftest" for a HAL round trip, exit status 0 / 1 / 2.
 *
 * Additions: --device=cuda:N picks a GPU; --devices=N opens cuda:0..N-1 for
 * programs placed on several GPUs or row-sharded over them; --time prints the
 * device time of the dispatches on stderr; --repeat=N runs the entry N times
 * (PRINT output from the first run only; with --time, the median wall and
 * dispatch times of the runs); --keep-constants keeps the module's constants
 * on the GPU between those runs.
 */
#define _POSIX_C_SOURCE 200809L
#include <fcntl.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>
#include <unistd.h>

#include "hexir_runtime/runtime.h"

static int usage(void) {
  fprintf(stderr,
          "usage: hexir-run <module.hxb> [--device=cpu|cuda|cuda:N] "
          "[--devices=N]\n"
          "                 [--entry=name] [--quiet] [--time] [--repeat=N]\n"
          "                 [--keep-constants]\n"
          "       hexir-run --selftest [--device=cpu|cuda|cuda:N]\n");
  return 2;
}

static int compare_doubles(const void *x, const void *y) {
  const double a = *(const double *)x, b = *(const double *)y;
  return (a > b) - (a < b);
}

static hexir_status_t open_device(hexir_device_kind_t kind, int ordinal,
                                  hexir_device_t **out) {
  if (kind == HEXIR_DEVICE_CUDA && ordinal > 0)
    return hexir_device_create_cuda(ordinal, out);
  return hexir_device_create(kind, out);
}

/* Allocate, write, wait, read back: the HAL without a module. */
static int selftest(hexir_device_kind_t kind, int ordinal) {
  hexir_device_t *device = NULL;
  hexir_status_t status = open_device(kind, ordinal, &device);
  if (status != HEXIR_OK) {
    fprintf(stderr, "hexir-run: device create failed: %s\n",
            hexir_status_string(status));
    return 1;
  }
  printf("device        : %s\n", hexir_device_name(device));
  double in[4] = {1.0, 2.0, 3.0, 4.0};
  double out[4] = {0};
  hexir_buffer_t *buffer = NULL;
  status = hexir_buffer_allocate(device, sizeof(in), HEXIR_MEMORY_DEVICE_LOCAL,
                                 &buffer);
  if (status == HEXIR_OK)
    status = hexir_buffer_write(buffer, in, sizeof(in));
  if (status == HEXIR_OK)
    status = hexir_device_wait(device);
  if (status == HEXIR_OK)
    status = hexir_buffer_read(buffer, out, sizeof(out));
  if (status != HEXIR_OK) {
    fprintf(stderr, "hexir-run: hal selftest failed: %s\n",
            hexir_status_string(status));
    hexir_buffer_release(buffer);
    hexir_device_release(device);
    return 1;
  }
  int ok = memcmp(in, out, sizeof(in)) == 0;
  printf("hal roundtrip : %s (%zu bytes)\n", ok ? "ok" : "MISMATCH",
         hexir_buffer_size(buffer));
  hexir_buffer_release(buffer);
  hexir_device_release(device);
  return ok ? 0 : 1;
}

int main(int argc, char **argv) {
  const char *path = NULL;
  const char *entry = "main";
  hexir_device_kind_t kind = HEXIR_DEVICE_CPU;
  int ordinal = 0;
  int device_count = 0; /* --devices=N */
  int want_selftest = 0, quiet = 0, show_time = 0, keep = 0;
  long repeat = 1;

  for (int i = 1; i < argc; ++i) {
    if (strcmp(argv[i], "--quiet") == 0 || strcmp(argv[i], "-q") == 0) {
      quiet = 1;
    } else if (strcmp(argv[i], "--selftest") == 0) {
      want_selftest = 1;
    } else if (strcmp(argv[i], "--time") == 0) {
      show_time = 1;
    } else if (strcmp(argv[i], "--keep-constants") == 0) {
      keep = 1;
    } else if (strncmp(argv[i], "--repeat=", 9) == 0) {
      char *end = NULL;
      repeat = strtol(argv[i] + 9, &end, 10);
      if (!end || *end || repeat < 1 || repeat > 100000)
        return usage();
    } else if (strncmp(argv[i], "--entry=", 8) == 0) {
      entry = argv[i] + 8;
    } else if (strncmp(argv[i], "--devices=", 10) == 0) {
      char *end = NULL;
      long n = strtol(argv[i] + 10, &end, 10);
      if (!end || *end || n < 1 || n > 64)
        return usage();
      device_count = (int)n;
      kind = HEXIR_DEVICE_CUDA;
    } else if (strncmp(argv[i], "--device=", 9) == 0) {
      const char *name = argv[i] + 9;
      if (strcmp(name, "cpu") == 0) {
        kind = HEXIR_DEVICE_CPU;
      } else if (strcmp(name, "cuda") == 0 || strcmp(name, "gpu") == 0) {
        kind = HEXIR_DEVICE_CUDA;
        ordinal = 0;
      } else if (strncmp(name, "cuda:", 5) == 0 && name[5]) {
        char *end = NULL;
        long n = strtol(name + 5, &end, 10);
        if (!end || *end || n < 0 || n > 63) {
          fprintf(stderr, "hexir-run: unknown device '%s'\n", name);
          return usage();
        }
        kind = HEXIR_DEVICE_CUDA;
        ordinal = (int)n;
      } else {
        fprintf(stderr, "hexir-run: unknown device '%s'\n", name);
        return usage();
      }
    } else if (argv[i][0] == '-') {
      return usage();
    } else {
      path = argv[i];
    }
  }

  if (want_selftest)
    return selftest(kind, ordinal);
  if (!path)
    return usage();

  hexir_module_t *module = NULL;
  hexir_status_t status = hexir_module_load_file(path, &module);
  if (status != HEXIR_OK) {
    fprintf(stderr, "hexir-run: cannot load '%s': %s\n", path,
            hexir_status_string(status));
    return 1;
  }
  if (!quiet) {
    printf("module        : %s\n", path);
    printf("version       : %u\n", hexir_module_version(module));
    printf("sections      : %u\n", hexir_module_section_count(module));
    for (uint32_t i = 0; i < hexir_module_section_count(module); ++i) {
      const hexir_section_entry_t *s = hexir_module_section_at(module, i);
      printf("  [%u] %-12s offset=%-10llu size=%llu\n", i,
             hexir_section_kind_string(s->kind),
             (unsigned long long)s->offset, (unsigned long long)s->size);
    }
  }

  hexir_device_t *devices[64] = {0};
  int opened = 0;
  if (device_count > 0) {
    for (; opened < device_count; ++opened) {
      status = hexir_device_create_cuda(opened, &devices[opened]);
      if (status != HEXIR_OK)
        break;
    }
  } else {
    status = open_device(kind, ordinal, &devices[0]);
    if (status == HEXIR_OK)
      opened = 1;
  }
  if (status != HEXIR_OK) {
    fprintf(stderr, "hexir-run: device create failed: %s\n",
            hexir_status_string(status));
    for (int i = 0; i < opened; ++i)
      hexir_device_release(devices[i]);
    hexir_module_release(module);
    return 1;
  }
  if (!quiet) {
    printf("device        : %s\n", hexir_device_name(devices[0]));
    if (device_count > 0)
      printf("devices       : %d\n", device_count);
    printf("--\n");
  }
  fflush(stdout);

  if (keep && (status = hexir_module_keep_constants(module, 1)) != HEXIR_OK)
    fprintf(stderr, "hexir-run: cannot keep constants: %s\n",
            hexir_status_string(status));
  double *wall_ms = calloc((size_t)repeat, sizeof(double));
  double *kernel_ms = calloc((size_t)repeat, sizeof(double));
  int saved_stdout = -1;
  for (long run = 0; status == HEXIR_OK && run < repeat; ++run) {
    if (run == 1) {
      /* PRINT output of the first run only. */
      fflush(stdout);
      saved_stdout = dup(STDOUT_FILENO);
      int null_fd = open("/dev/null", O_WRONLY);
      if (null_fd >= 0) {
        dup2(null_fd, STDOUT_FILENO);
        close(null_fd);
      }
    }
    struct timespec t0, t1;
    clock_gettime(CLOCK_MONOTONIC, &t0);
    if (device_count > 0)
      status = hexir_execute_devices(module, devices, (unsigned)device_count,
                                     entry, NULL, 0);
    else
      status = hexir_execute(module, devices[0], entry);
    clock_gettime(CLOCK_MONOTONIC, &t1);
    fflush(stdout);
    if (wall_ms && kernel_ms) {
      wall_ms[run] = (double)(t1.tv_sec - t0.tv_sec) * 1e3 +
                     (double)(t1.tv_nsec - t0.tv_nsec) * 1e-6;
      kernel_ms[run] = hexir_last_execute_kernel_ms();
    }
  }
  if (saved_stdout >= 0) {
    dup2(saved_stdout, STDOUT_FILENO);
    close(saved_stdout);
  }
  if (status != HEXIR_OK) {
    fprintf(stderr, "hexir-run: %s failed: %s\n", entry,
            hexir_status_string(status));
  } else if (show_time && repeat == 1) {
    fprintf(stderr, "kernel time   : %.3f ms\n", hexir_last_execute_kernel_ms());
  } else if (show_time && wall_ms && kernel_ms) {
    /* Medians of the runs after the first (warm-up) one. */
    qsort(wall_ms + 1, (size_t)(repeat - 1), sizeof(double), compare_doubles);
    qsort(kernel_ms + 1, (size_t)(repeat - 1), sizeof(double), compare_doubles);
    const long mid = 1 + (repeat - 1) / 2;
    fprintf(stderr, "runs          : %ld (first one not counted)\n", repeat);
    fprintf(stderr, "execute time  : %.3f ms median\n", wall_ms[mid]);
    fprintf(stderr, "kernel time   : %.3f ms median\n", kernel_ms[mid]);
  }
  free(wall_ms);
  free(kernel_ms);

  for (int i = 0; i < opened; ++i)
    hexir_device_release(devices[i]);
  hexir_module_release(module);
  return status == HEXIR_OK ? 0 : 1;
}
