/*
 * program.h -- encoding of the PROGRAM, SYMBOLS and EXECUTABLES sections.
 *
 * Layouts and values are those of the reference format
 * (runtime/include/hexir_runtime/program.h:28-94): command kinds 0-4, kernel
 * kinds 1-3, the 80-byte executable entry and the 40-byte symbol entry.  A
 * module written by either side loads in the other.
 *
 * Extensions, all additive:
 *   - kernel kind 4, HEXIR_KERNEL_MATMUL_RELU: relu(a . b) in one kernel, the
 *     form a linear takes when its only user is a relu on the same device.  A
 *     runtime that does not know kind 4 rejects it instead of silently
 *     dropping the relu.
 *   - kernel kinds 5 and 6, HEXIR_KERNEL_MATMUL_ADD(_RELU): a . b + d (then
 *     the relu), a linear whose only user is an add (whose only user is a
 *     relu) on the same device.  DISPATCH operands: a, b, d, destination.
 *   - kernel kinds 7-14, the activations the reference dialect declares
 *     without lowering (leaky_relu, elu, sigmoid, tanh, softmax, gelu, swish,
 *     mish): y = op(x) over [m x n], softmax along each row.  DISPATCH
 *     operands: x, destination.  Written only on request
 *     (HEXIR_EMIT_ACTIVATIONS); by default the writer refuses these ops as
 *     the reference serializer does.
 *   - the LAUNCH section (module.h kind 5), one hexir_launch_entry_t per
 *     executable, in executable order.
 */
#ifndef HEXIR_RUNTIME_PROGRAM_H
#define HEXIR_RUNTIME_PROGRAM_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  HEXIR_CMD_END = 0,      /* no operands */
  HEXIR_CMD_ALLOC = 1,    /* slot, byte_size */
  HEXIR_CMD_CONST = 2,    /* slot, rodata_offset, byte_size */
  HEXIR_CMD_DISPATCH = 3, /* executable_index, arg_count, slot x arg_count;
                             the last slot is the destination */
  HEXIR_CMD_PRINT = 4,    /* slot, rows, cols */
} hexir_command_kind_t;

/* Followed by operand_count little-endian uint64_t operands. */
typedef struct {
  uint32_t kind;
  uint32_t operand_count;
} hexir_command_header_t;

typedef enum {
  HEXIR_KERNEL_MATMUL = 1,      /* c[m x n] = a[m x k] . b[k x n] */
  HEXIR_KERNEL_ADD = 2,         /* c = a + b, elementwise over m*n */
  HEXIR_KERNEL_RELU = 3,        /* y = x > 0 ? x : 0, elementwise over m*n */
  HEXIR_KERNEL_MATMUL_RELU = 4, /* extension: c = relu(a . b) */
  HEXIR_KERNEL_MATMUL_ADD = 5,  /* extension: c = a . b + d */
  HEXIR_KERNEL_MATMUL_ADD_RELU = 6, /* extension: c = relu(a . b + d) */
  HEXIR_KERNEL_LEAKY_RELU = 7,  /* extension: x > 0 ? x : 0.01 x */
  HEXIR_KERNEL_ELU = 8,         /* extension: x > 0 ? x : expm1(x) */
  HEXIR_KERNEL_SIGMOID = 9,     /* extension: 1 / (1 + exp(-x)) */
  HEXIR_KERNEL_TANH = 10,       /* extension: tanh(x) */
  HEXIR_KERNEL_SOFTMAX = 11,    /* extension: softmax along each row */
  HEXIR_KERNEL_GELU = 12,       /* extension: 0.5 x erfc(-x / sqrt 2) */
  HEXIR_KERNEL_SWISH = 13,      /* extension: x / (1 + exp(-x)) */
  HEXIR_KERNEL_MISH = 14,       /* extension: x tanh(softplus(x)) */
} hexir_kernel_kind_t;

#define HEXIR_NAME_SIZE 32

/* [u32 count][u32 reserved][entry x count][8-byte aligned images...] */
typedef struct {
  char name[HEXIR_NAME_SIZE];
  uint32_t kind;         /* hexir_kernel_kind_t */
  uint32_t device;       /* hexir_device_kind_t the op was placed on */
  uint32_t m, n, k;      /* extents; k = 0 for elementwise kernels */
  uint32_t elem_size;    /* 8 for f64 */
  uint32_t image_offset; /* from the start of EXECUTABLES */
  uint32_t image_size;   /* 0: descriptor only, the host runs the body */
  uint32_t grid_x, grid_y;
  uint32_t block_x, block_y;
} hexir_executable_entry_t; /* 80 bytes */

typedef struct {
  uint32_t count;
  uint32_t reserved;
} hexir_executable_header_t;

typedef struct {
  char name[HEXIR_NAME_SIZE];
  uint32_t program_offset; /* byte offset of the entry's first command */
  uint32_t reserved;
} hexir_symbol_entry_t; /* 40 bytes */

/* "matmul", "add", "relu", "matmul_relu", else "unknown". */
const char *hexir_kernel_kind_string(uint32_t kind);

/* ---- extension: LAUNCH section ------------------------------------------ */

#define HEXIR_LAUNCH_ABI_V1 1u

/* Image launched through the kernel library of this project (one image holds
 * every kernel; the runtime picks the variant from kind and shape). */
#define HEXIR_LAUNCH_FLAG_LIBRARY 0x1u

/* [u32 count][u32 reserved][hexir_launch_entry_t x count] */
typedef struct {
  uint32_t abi;          /* HEXIR_LAUNCH_ABI_V1 */
  uint32_t flags;        /* HEXIR_LAUNCH_FLAG_* */
  uint32_t device_first; /* first CUDA ordinal ("cuda:N" -> N) */
  uint32_t device_count; /* 1: one GPU; >1: rows of the destination split
                            over ordinals [first, first + count) */
  uint32_t reserved[4];
} hexir_launch_entry_t; /* 32 bytes */

typedef struct {
  uint32_t count;
  uint32_t reserved;
} hexir_launch_header_t;

#ifdef __cplusplus
}
#endif
#endif /* HEXIR_RUNTIME_PROGRAM_H */
