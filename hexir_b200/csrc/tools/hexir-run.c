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
 * device time of the dispatches on stderr.
 */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "hexir_runtime/runtime.h"

static int usage(void) {
  fprintf(stderr,
          "usage: hexir-run <module.hxb> [--device=cpu|cuda|cuda:N] "
          "[--devices=N]\n"
          "                 [--entry=name] [--quiet] [--time]\n"
          "       hexir-run --selftest [--device=cpu|cuda|cuda:N]\n");
  return 2;
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
  int want_selftest = 0, quiet = 0, show_time = 0;

  for (int i = 1; i < argc; ++i) {
    if (strcmp(argv[i], "--quiet") == 0 || strcmp(argv[i], "-q") == 0) {
      quiet = 1;
    } else if (strcmp(argv[i], "--selftest") == 0) {
      want_selftest = 1;
    } else if (strcmp(argv[i], "--time") == 0) {
      show_time = 1;
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

  if (device_count > 0)
    status = hexir_execute_devices(module, devices, (unsigned)device_count,
                                   entry, NULL, 0);
  else
    status = hexir_execute(module, devices[0], entry);
  fflush(stdout);
  if (status != HEXIR_OK)
    fprintf(stderr, "hexir-run: %s failed: %s\n", entry,
            hexir_status_string(status));
  else if (show_time)
    fprintf(stderr, "kernel time   : %.3f ms\n", hexir_last_execute_kernel_ms());

  for (int i = 0; i < opened; ++i)
    hexir_device_release(devices[i]);
  hexir_module_release(module);
  return status == HEXIR_OK ? 0 : 1;
}
