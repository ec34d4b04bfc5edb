/*
 * hexir_b200/hxb_writer.h -- build hexir programs and serialize them to .hxb.
 *
 * The reference produces .hxb with its MLIR compiler (`hexir -emit=hxb`,
 * compiler/Serialization/ModuleSerializer.cpp), which needs an unreleased
 * LLVM/MLIR to build.  This writer is the stand-in: it takes the same program
 * (hexir.constant / linear / add / relu / print in func.func bodies), the same
 * -placement= syntax (tools/hexir/hexir.cpp:229-260, compiler/Target/
 * TargetInfo.cpp:20-45) and emits the same container, byte for byte for
 * cpu-placed programs:
 *   - one executable per compute op, named <op>_<n> in walk order
 *     (compiler/Conversion/HexirToTIR/HexirToTIR.cpp:251-281);
 *   - constants with users go to RODATA, 8-byte padded, as CONST commands;
 *     splats are expanded; unused constants are dropped
 *     (ModuleSerializer.cpp:299-326);
 *   - each compute op becomes ALLOC + DISPATCH with the destination last
 *     (ModuleSerializer.cpp:328-350); print becomes PRINT; END closes;
 *   - header, section table, 8-byte aligned payloads (ModuleSerializer.cpp:
 *     375-425).
 * cuda-placed executables carry this project's sm_100a kernel image (one copy
 * shared by all entries) and a LAUNCH section (module.h) instead of an
 * MLIR-generated CUBIN.
 *
 * Placement values: cpu, cuda, gpu (alias of cuda), and the extensions cuda:N
 * (GPU N) and cuda:F-L (rows split over GPUs F..L).  Defaults are all cpu, as
 * in the reference.
 */
#ifndef HEXIR_B200_HXB_WRITER_H
#define HEXIR_B200_HXB_WRITER_H

#include <stddef.h>
#include <stdint.h>

#include "hexir_runtime/status.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct hexir_program_t hexir_program_t;

hexir_program_t *hexir_program_create(void);
void hexir_program_release(hexir_program_t *program);

/* Start a new func.func (the first op of a program starts "main" implicitly). */
hexir_status_t hexir_program_begin_function(hexir_program_t *program,
                                            const char *name);

/* Values are numbered from 0; a negative return is an error (see
 * hexir_program_last_error).  Data is row-major [rows x cols] f64 and is
 * copied. */
int32_t hexir_program_constant(hexir_program_t *program, const double *data,
                               uint32_t rows, uint32_t cols);
int32_t hexir_program_splat(hexir_program_t *program, double value,
                            uint32_t rows, uint32_t cols);
/* input [m x k] . weight [k x n] -> [m x n] */
int32_t hexir_program_linear(hexir_program_t *program, int32_t input,
                             int32_t weight);
int32_t hexir_program_add(hexir_program_t *program, int32_t lhs, int32_t rhs);
int32_t hexir_program_relu(hexir_program_t *program, int32_t input);
/* One of the activations the dialect declares without lowering
 * (include/hexir/Dialect/Hexir/IR/HexirOps.td:189-308): op is "leaky_relu",
 * "elu", "sigmoid", "tanh", "softmax", "gelu", "swish" or "mish" (a "hexir."
 * prefix is accepted).  Same shape as the input.  Serialized only with
 * HEXIR_EMIT_ACTIVATIONS. */
int32_t hexir_program_activation(hexir_program_t *program, const char *op,
                                 int32_t input);
hexir_status_t hexir_program_print(hexir_program_t *program, int32_t value);

/* Do not fuse linear -> relu into one matmul_relu executable. */
#define HEXIR_EMIT_NO_FUSE 0x1u
/* cuda-placed executables carry descriptors only (no image, no LAUNCH), as
 * the reference serializer does when it cannot compile device code. */
#define HEXIR_EMIT_NO_IMAGE 0x2u
/* Serialize the activations (kernel kinds 7-14 of hexir_runtime/program.h).
 * Without it an activation fails the emit with the reference serializer's
 * "cannot serialize this op into a host program", as the reference has no
 * kernel for them. */
#define HEXIR_EMIT_ACTIVATIONS 0x4u

/* Serialize with a -placement= string ("hexir.linear=cuda,hexir.relu=cpu";
 * NULL or "" = all cpu).  Placement errors return INVALID_ARGUMENT with the
 * reference's wording in hexir_program_last_error. */
hexir_status_t hexir_program_emit_file(hexir_program_t *program,
                                       const char *placement, uint32_t flags,
                                       const char *path);
/* Same, into a malloc'd buffer the caller frees with hexir_free. */
hexir_status_t hexir_program_emit_memory(hexir_program_t *program,
                                         const char *placement, uint32_t flags,
                                         void **data, size_t *size);
void hexir_free(void *data);

/* Parse the textual program subset (func.func, hexir.constant dense<...>,
 * linear, add, relu, print, return; `//` comments) into a new program. */
hexir_status_t hexir_program_parse(const char *text, hexir_program_t **out,
                                   char *error, size_t error_size);

const char *hexir_program_last_error(const hexir_program_t *program);

/* Seeded synthetic data.  SplitMix64 stream: state advances by
 * 0x9E3779B97F4A7C15 per draw; uniform = lo + (hi - lo) * (z >> 11) * 2^-53;
 * normal = mean + std * sqrt(-2 ln(1 - u1)) * cos(2 pi u2) (two draws per
 * value).  Successive calls on one state continue the stream, so "a then w
 * from seed s" is two calls on one state. */
typedef struct {
  uint64_t state;
} hexir_rng_t;
void hexir_rng_seed(hexir_rng_t *rng, uint64_t seed);
void hexir_rng_uniform(hexir_rng_t *rng, double *out, size_t n, double lo,
                       double hi);
void hexir_rng_normal(hexir_rng_t *rng, double *out, size_t n, double mean,
                      double stddev);

#ifdef __cplusplus
}
#endif
#endif /* HEXIR_B200_HXB_WRITER_H */
