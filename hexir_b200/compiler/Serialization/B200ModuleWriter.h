//===- B200ModuleWriter.h - host program -> .hxb for the B200 runtime -----===//
//
// The half of the compiler-side serializer that needs no MLIR.  The
// serializer (B200Serializer.cpp) walks the kernel-level IR the reference
// pipeline produces (Stage::TIR: hexir.constant, hexir.call_tir against
// hextir.prim_func carrying `hexir.kernel` and `device`, hexir.print) into a
// flat list of HostOps; this file turns that list into module bytes through
// libhexir_b200's writer C ABI (include/hexir_b200/hxb_writer.h).
//
// So `hexir -emit=hxb` writes exactly what hexir-mkhxb writes for the same
// program and placement: the reference's byte layout for cpu-placed
// programs (ModuleSerializer.cpp:47-425), and for cuda-placed ones one shared
// copy of the runtime's sm_100a kernel image (hexir_cuda_kernel_image), the
// fused kinds 4-6 (linear+relu, linear+add, linear+add+relu) and the LAUNCH
// section, instead of one MLIR-generated CUBIN per kernel.
//
// Standard C++ only; compiled and tested in this repository by
// tests/test_compiler_surface.py against the Python writer's bytes.
//
//===----------------------------------------------------------------------===//
#ifndef HEXIR_B200_COMPILER_B200MODULEWRITER_H
#define HEXIR_B200_COMPILER_B200MODULEWRITER_H

#include <cstdint>
#include <string>
#include <vector>

namespace hexir_b200 {

enum class HostOpKind {
  BeginFunction, // a func.func: `name`
  Constant,      // a dense f64 constant: rows x cols of `data`
  Splat,         // a splat f64 constant: rows x cols of `splat`
  Linear,        // operands: input, weight   (hexir.kernel = "matmul")
  Add,           // operands: lhs, rhs        (hexir.kernel = "add")
  Relu,          // operands: input           (hexir.kernel = "relu")
  Print,         // operands: value
};

// One op of the host program.  Operands name values by the index of the op
// that produced them in the list (BeginFunction and Print produce none).
struct HostOp {
  HostOpKind kind = HostOpKind::Print;
  std::string name;
  std::vector<int32_t> operands;
  uint32_t rows = 0, cols = 0;
  std::vector<double> data;
  double splat = 0.0;
  // Compute ops: the `device` attribute of the callee prim_func ("cpu",
  // "cuda", "cuda:N", "cuda:F-L").
  std::string device;
};

// The -placement string that reproduces the ops' devices: one entry per
// placeable op kind that is not on the host ("hexir.linear=cuda:0-3,...").
// The partition pass places by op kind, so all ops of a kind share a device;
// false (with *error set) if they do not, or a device is not valid.
bool placementOf(const std::vector<HostOp> &ops, std::string *placement,
                 std::string *error);

// The module bytes for `ops`, placed by their devices.  `flags` are the
// writer's HEXIR_EMIT_* flags.  False with *error set on an invalid program.
bool writeModule(const std::vector<HostOp> &ops, uint32_t flags,
                 std::string *bytes, std::string *error);

} // namespace hexir_b200

#endif // HEXIR_B200_COMPILER_B200MODULEWRITER_H
