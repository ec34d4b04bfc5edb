//===- B200Serializer.h - serializeToHXB for the B200 runtime --*- C++ -*-===//
//
// NOT COMPILED HERE: needs the reference compiler's MLIR (LLVM 24.0git).
// Written against that API for a maintainer to add to
// compiler/Serialization; patches/0001-b200-placement-and-serializer.patch
// wires it in.
//
//===----------------------------------------------------------------------===//
#ifndef HEXIR_B200_COMPILER_B200SERIALIZER_H
#define HEXIR_B200_COMPILER_B200SERIALIZER_H

#include "mlir/IR/BuiltinOps.h"
#include "mlir/Support/LLVM.h"
#include "llvm/Support/raw_ostream.h"

namespace hexir_b200 {

/// Serialize `module` (at the kernel level, Stage::TIR, as the reference's
/// serializeToHXB expects) to a .hxb the B200 runtime runs: every cuda-placed
/// kernel dispatches into the runtime's own sm_100a image, with the
/// ordinals of "cuda:N" / "cuda:F-L" placements in the LAUNCH section.
/// `flags` are the writer's HEXIR_EMIT_* flags.
mlir::LogicalResult serializeForB200(mlir::ModuleOp module,
                                     llvm::raw_ostream &os,
                                     uint32_t flags = 0);

} // namespace hexir_b200

#endif // HEXIR_B200_COMPILER_B200SERIALIZER_H
