/*
 * hexir-run -- run an entry point of a .hxb module with no compiler in the
 * process.
 *
 * The command line and everything printed follow the reference tool
 * (runtime/tools/hexir-run/hexir-run.c:17-143), because the reference's
 * lit tests diff them: the module report (path, version, sections, device,
 * "--"), PRINT results on stdout, "--quiet" for results only, "--selftest"
 * for a HAL round trip, exit status 0 (ok), 1 (failure), 2 (usage).
 *
 * Additions: --device=cuda:N picks a GPU; --devices=N opens cuda:0..N-1 for
 * modules placed on several GPUs or row-sharded over them; --time reports
 * the device time of the dispatches on stderr; --repeat=N runs the entry N
 * times (PRINT output from the first run only; with --time, medians of the
 * runs after the first); --keep-constants keeps the module's constants on
 * the GPU between those runs.
 *
 * Layout: parse_options fills a `run_options`; a `device_set` holds the
 * opened devices; main chains the phases and owns every release.
 */
#define _POSIX_C_SOURCE 200809L
#include <fcntl.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>
#include <unistd.h>

#include "hexir_runtime/runtime.h"

enum { EXIT_OK = 0, EXIT_FAILED = 1, EXIT_USAGE = 2, MAX_DEVICES = 64 };

typedef struct {
  const char *module_path;
  const char *entry;
  hexir_device_kind_t kind;
  int ordinal;      /* --device=cuda:N */
  int gpu_count;    /* --devices=N; 0: one device */
  int selftest;
  int quiet;
  int timing;
  int keep_constants;
  long repeat;
} run_options;

typedef struct {
  hexir_device_t *dev[MAX_DEVICES];
  int count;
} device_set;

/* ---------------------------------------------------------------- options */

static int usage(void) {
  fputs("usage: hexir-run <module.hxb> [--device=cpu|cuda|cuda:N] "
        "[--devices=N]\n"
        "                 [--entry=name] [--quiet] [--time] [--repeat=N]\n"
        "                 [--keep-constants]\n"
        "       hexir-run --selftest [--device=cpu|cuda|cuda:N]\n",
        stderr);
  return EXIT_USAGE;
}

/* A whole decimal number in [lo, hi]; 0 when `text` is not one. */
static int parse_bounded(const char *text, long lo, long hi, long *out) {
  char *end = NULL;
  if (!*text)
    return 0;
  long v = strtol(text, &end, 10);
  if (*end || v < lo || v > hi)
    return 0;
  *out = v;
  return 1;
}

/* "cpu", "cuda", "gpu" (the reference's alias) or "cuda:N". */
static int parse_device(const char *name, run_options *o) {
  long n = 0;
  if (strcmp(name, "cpu") == 0) {
    o->kind = HEXIR_DEVICE_CPU;
  } else if (strcmp(name, "cuda") == 0 || strcmp(name, "gpu") == 0) {
    o->kind = HEXIR_DEVICE_CUDA;
    o->ordinal = 0;
  } else if (strncmp(name, "cuda:", 5) == 0 &&
             parse_bounded(name + 5, 0, MAX_DEVICES - 1, &n)) {
    o->kind = HEXIR_DEVICE_CUDA;
    o->ordinal = (int)n;
  } else {
    fprintf(stderr, "hexir-run: unknown device '%s'\n", name);
    return 0;
  }
  return 1;
}

/* The value after `flag` when `arg` is "flag<value>", else NULL. */
static const char *value_of(const char *arg, const char *flag) {
  const size_t n = strlen(flag);
  return strncmp(arg, flag, n) == 0 ? arg + n : NULL;
}

static int parse_options(int argc, char **argv, run_options *o) {
  memset(o, 0, sizeof(*o));
  o->entry = "main";
  o->kind = HEXIR_DEVICE_CPU;
  o->repeat = 1;
  for (int i = 1; i < argc; ++i) {
    const char *arg = argv[i], *v = NULL;
    long n = 0;
    if (!strcmp(arg, "--quiet") || !strcmp(arg, "-q"))
      o->quiet = 1;
    else if (!strcmp(arg, "--selftest"))
      o->selftest = 1;
    else if (!strcmp(arg, "--time"))
      o->timing = 1;
    else if (!strcmp(arg, "--keep-constants"))
      o->keep_constants = 1;
    else if ((v = value_of(arg, "--entry=")))
      o->entry = v;
    else if ((v = value_of(arg, "--repeat="))) {
      if (!parse_bounded(v, 1, 100000, &n))
        return 0;
      o->repeat = n;
    } else if ((v = value_of(arg, "--devices="))) {
      if (!parse_bounded(v, 1, MAX_DEVICES, &n))
        return 0;
      o->gpu_count = (int)n;
      o->kind = HEXIR_DEVICE_CUDA;
    } else if ((v = value_of(arg, "--device="))) {
      if (!parse_device(v, o))
        return 0;
    } else if (arg[0] == '-')
      return 0;
    else
      o->module_path = arg;
  }
  return o->selftest || o->module_path;
}

/* ---------------------------------------------------------------- devices */

static hexir_status_t open_one(hexir_device_kind_t kind, int ordinal,
                               hexir_device_t **out) {
  return kind == HEXIR_DEVICE_CUDA && ordinal > 0
             ? hexir_device_create_cuda(ordinal, out)
             : hexir_device_create(kind, out);
}

static void close_devices(device_set *set) {
  while (set->count > 0)
    hexir_device_release(set->dev[--set->count]);
}

/* --devices=N: cuda:0..N-1; otherwise the one device of --device. */
static hexir_status_t open_devices(const run_options *o, device_set *set) {
  set->count = 0;
  const int wanted = o->gpu_count > 0 ? o->gpu_count : 1;
  while (set->count < wanted) {
    hexir_status_t st =
        o->gpu_count > 0
            ? hexir_device_create_cuda(set->count, &set->dev[set->count])
            : open_one(o->kind, o->ordinal, &set->dev[set->count]);
    if (st != HEXIR_OK) {
      close_devices(set);
      return st;
    }
    ++set->count;
  }
  return HEXIR_OK;
}

/* --------------------------------------------------------------- selftest */

/* Through the HAL alone: a device buffer written and read back must return
 * every byte, including the bit patterns of -0.0 and a NaN payload. */
static int run_selftest(const run_options *o) {
  hexir_device_t *dev = NULL;
  hexir_status_t st = open_one(o->kind, o->ordinal, &dev);
  if (st != HEXIR_OK) {
    fprintf(stderr, "hexir-run: device create failed: %s\n",
            hexir_status_string(st));
    return EXIT_FAILED;
  }
  printf("device        : %s\n", hexir_device_name(dev));
  const uint64_t pattern[4] = {0x3ff0000000000000ull, 0x8000000000000000ull,
                               0x7ff8dead0000beefull, 0x0123456789abcdefull};
  uint64_t back[4];
  memset(back, 0xa5, sizeof(back));
  hexir_buffer_t *buf = NULL;
  st = hexir_buffer_allocate(dev, sizeof(pattern), HEXIR_MEMORY_DEVICE_LOCAL,
                             &buf);
  if (st == HEXIR_OK)
    st = hexir_buffer_write(buf, pattern, sizeof(pattern));
  if (st == HEXIR_OK)
    st = hexir_device_wait(dev);
  if (st == HEXIR_OK)
    st = hexir_buffer_read(buf, back, sizeof(back));
  int same = 0;
  if (st == HEXIR_OK) {
    same = memcmp(pattern, back, sizeof(pattern)) == 0;
    printf("hal roundtrip : %s (%zu bytes)\n", same ? "ok" : "MISMATCH",
           hexir_buffer_size(buf));
  } else {
    fprintf(stderr, "hexir-run: hal selftest failed: %s\n",
            hexir_status_string(st));
  }
  if (buf)
    hexir_buffer_release(buf);
  hexir_device_release(dev);
  return same ? EXIT_OK : EXIT_FAILED;
}

/* ----------------------------------------------------------------- report */

static void report_module(const char *path, hexir_module_t *m) {
  const uint32_t n = hexir_module_section_count(m);
  printf("module        : %s\n", path);
  printf("version       : %u\n", hexir_module_version(m));
  printf("sections      : %u\n", n);
  for (uint32_t i = 0; i < n; ++i) {
    const hexir_section_entry_t *s = hexir_module_section_at(m, i);
    printf("  [%u] %-12s offset=%-10llu size=%llu\n", i,
           hexir_section_kind_string(s->kind), (unsigned long long)s->offset,
           (unsigned long long)s->size);
  }
}

/* ------------------------------------------------------------------ runs */

/* Per-run wall and dispatch times. */
typedef struct {
  double *wall_ms;
  double *kernel_ms;
  long runs;
} run_times;

static double elapsed_ms(const struct timespec *a, const struct timespec *b) {
  return (double)(b->tv_sec - a->tv_sec) * 1e3 +
         (double)(b->tv_nsec - a->tv_nsec) * 1e-6;
}

/* stdout pointed at /dev/null; returns the saved descriptor (or -1). */
static int mute_stdout(void) {
  fflush(stdout);
  const int saved = dup(STDOUT_FILENO);
  const int sink = open("/dev/null", O_WRONLY);
  if (sink >= 0) {
    dup2(sink, STDOUT_FILENO);
    close(sink);
  }
  return saved;
}

static void restore_stdout(int saved) {
  if (saved < 0)
    return;
  fflush(stdout);
  dup2(saved, STDOUT_FILENO);
  close(saved);
}

static hexir_status_t execute_once(hexir_module_t *m, const run_options *o,
                                   device_set *set) {
  return o->gpu_count > 0
             ? hexir_execute_devices(m, set->dev, (unsigned)set->count,
                                     o->entry, NULL, 0)
             : hexir_execute(m, set->dev[0], o->entry);
}

/* The entry o->repeat times; PRINT reaches stdout from the first run only. */
static hexir_status_t run_entry(hexir_module_t *m, const run_options *o,
                                device_set *set, run_times *t) {
  hexir_status_t st = HEXIR_OK;
  int saved = -1;
  for (long r = 0; r < o->repeat && st == HEXIR_OK; ++r) {
    if (r == 1)
      saved = mute_stdout();
    struct timespec t0, t1;
    clock_gettime(CLOCK_MONOTONIC, &t0);
    st = execute_once(m, o, set);
    clock_gettime(CLOCK_MONOTONIC, &t1);
    fflush(stdout);
    if (t->wall_ms && t->kernel_ms) {
      t->wall_ms[r] = elapsed_ms(&t0, &t1);
      t->kernel_ms[r] = hexir_last_execute_kernel_ms();
      t->runs = r + 1;
    }
  }
  restore_stdout(saved);
  return st;
}

static int by_value(const void *x, const void *y) {
  const double a = *(const double *)x, b = *(const double *)y;
  return (a > b) - (a < b);
}

/* Median of v[from..n): sorts that range. */
static double median_from(double *v, long from, long n) {
  qsort(v + from, (size_t)(n - from), sizeof(double), by_value);
  return v[from + (n - from) / 2];
}

static void report_times(const run_options *o, run_times *t) {
  if (!o->timing)
    return;
  if (o->repeat == 1 || !t->wall_ms || t->runs < 2) {
    fprintf(stderr, "kernel time   : %.3f ms\n", hexir_last_execute_kernel_ms());
    return;
  }
  /* The first run warms caches and modules: medians of the others. */
  fprintf(stderr, "runs          : %ld (first one not counted)\n", t->runs);
  fprintf(stderr, "execute time  : %.3f ms median\n",
          median_from(t->wall_ms, 1, t->runs));
  fprintf(stderr, "kernel time   : %.3f ms median\n",
          median_from(t->kernel_ms, 1, t->runs));
}

/* ------------------------------------------------------------------ main */

int main(int argc, char **argv) {
  run_options opt;
  if (!parse_options(argc, argv, &opt))
    return usage();
  if (opt.selftest)
    return run_selftest(&opt);

  hexir_module_t *module = NULL;
  hexir_status_t st = hexir_module_load_file(opt.module_path, &module);
  if (st != HEXIR_OK) {
    fprintf(stderr, "hexir-run: cannot load '%s': %s\n", opt.module_path,
            hexir_status_string(st));
    return EXIT_FAILED;
  }
  if (!opt.quiet)
    report_module(opt.module_path, module);

  device_set devices = {{0}, 0};
  st = open_devices(&opt, &devices);
  if (st != HEXIR_OK) {
    fprintf(stderr, "hexir-run: device create failed: %s\n",
            hexir_status_string(st));
    hexir_module_release(module);
    return EXIT_FAILED;
  }
  if (!opt.quiet) {
    printf("device        : %s\n", hexir_device_name(devices.dev[0]));
    if (opt.gpu_count > 0)
      printf("devices       : %d\n", opt.gpu_count);
    printf("--\n");
  }
  fflush(stdout);

  if (opt.keep_constants) {
    hexir_status_t k = hexir_module_keep_constants(module, 1);
    if (k != HEXIR_OK)
      fprintf(stderr, "hexir-run: cannot keep constants: %s\n",
              hexir_status_string(k));
  }
  run_times times = {calloc((size_t)opt.repeat, sizeof(double)),
                     calloc((size_t)opt.repeat, sizeof(double)), 0};
  st = run_entry(module, &opt, &devices, &times);
  if (st != HEXIR_OK)
    fprintf(stderr, "hexir-run: %s failed: %s\n", opt.entry,
            hexir_status_string(st));
  else
    report_times(&opt, &times);
  free(times.wall_ms);
  free(times.kernel_ms);

  close_devices(&devices);
  hexir_module_release(module);
  return st == HEXIR_OK ? EXIT_OK : EXIT_FAILED;
}
