//===- B200Serializer.cpp - serializeToHXB for the B200 runtime -----------===//
//
// NOT COMPILED HERE: needs the reference compiler's MLIR (LLVM 24.0git).
//
// The reference serializer (compiler/Serialization/ModuleSerializer.cpp:
// 128-216) lowers every cuda-placed hextir.prim_func through gpu ->
// NVVM -> CUBIN and embeds one generated image per kernel.  For the B200
// runtime that path is replaced whole: the kernels are the runtime's own
// sm_100a library, so the serializer needs no GPU lowering at all.  It reads
// the host program off the kernel-level IR -- constants, one call_tir per
// compute op with the callee's `hexir.kernel` and `device` attributes,
// prints -- and hands it to the runtime's writer (B200ModuleWriter), which
// lays the module out, fuses linear+relu / linear+add[+relu] into kinds
// 4-6, embeds the kernel image once and appends the LAUNCH section.
//
//===----------------------------------------------------------------------===//
#include "B200Serializer.h"

#include "B200ModuleWriter.h"

#include "hexir/Dialect/HexTIR/IR/HexTIRDialect.h"
#include "hexir/Dialect/Hexir/IR/HexirDialect.h"

#include "mlir/Dialect/Func/IR/FuncOps.h"
#include "mlir/IR/BuiltinAttributes.h"
#include "mlir/IR/BuiltinTypes.h"
#include "mlir/IR/SymbolTable.h"
#include "llvm/ADT/APFloat.h"
#include "llvm/ADT/DenseMap.h"

using namespace mlir;

namespace hexir_b200 {
namespace {

/// The host op of a prim func's `hexir.kernel` attribute (set by
/// hexir-lower-to-tir, compiler/Conversion/HexirToTIR/HexirToTIR.cpp:251-313).
FailureOr<HostOpKind> kindOf(hextir::PrimFuncOp fn) {
  auto kernel = fn->getAttrOfType<StringAttr>("hexir.kernel");
  if (!kernel)
    return fn.emitError("prim func has no hexir.kernel attribute; it was not "
                        "produced by hexir-lower-to-tir");
  StringRef k = kernel.getValue();
  if (k == "matmul")
    return HostOpKind::Linear;
  if (k == "add")
    return HostOpKind::Add;
  if (k == "relu")
    return HostOpKind::Relu;
  return fn.emitError("kernel '") << k << "' has no B200 kernel";
}

/// A rank-2 f64 constant: dense data, or a splat the writer expands.
FailureOr<HostOp> constantOf(mlir::hexir::ConstantOp constant) {
  auto dense = dyn_cast<DenseElementsAttr>(constant.getValue());
  auto type = dyn_cast<RankedTensorType>(constant.getType());
  if (!dense || !type || type.getRank() != 2 || !type.getElementType().isF64())
    return constant.emitError("expected a dense rank-2 f64 constant");
  HostOp op;
  op.rows = static_cast<uint32_t>(type.getShape()[0]);
  op.cols = static_cast<uint32_t>(type.getShape()[1]);
  if (dense.isSplat()) {
    op.kind = HostOpKind::Splat;
    op.splat = dense.getSplatValue<APFloat>().convertToDouble();
    return op;
  }
  op.kind = HostOpKind::Constant;
  op.data.reserve(static_cast<size_t>(op.rows) * op.cols);
  for (const APFloat &v : dense.getValues<APFloat>())
    op.data.push_back(v.convertToDouble());
  return op;
}

} // namespace

LogicalResult serializeForB200(ModuleOp module, llvm::raw_ostream &os,
                               uint32_t flags) {
  SymbolTable symbols(module);
  std::vector<HostOp> ops;
  llvm::DenseMap<Value, int32_t> producer; // SSA value -> index in `ops`

  auto operandsOf = [&](Operation *user, ValueRange values,
                        HostOp &op) -> LogicalResult {
    for (Value v : values) {
      auto it = producer.find(v);
      if (it == producer.end())
        return user->emitError("operand is not produced by a constant or a "
                               "call in this function");
      op.operands.push_back(it->second);
    }
    return success();
  };

  for (auto fn : module.getOps<func::FuncOp>()) {
    HostOp begin;
    begin.kind = HostOpKind::BeginFunction;
    begin.name = fn.getName().str();
    ops.push_back(std::move(begin));

    for (Operation &op : fn.getBody().front()) {
      if (auto constant = dyn_cast<mlir::hexir::ConstantOp>(op)) {
        // Unused constants never reach the module (the writer drops them
        // too); skipping them here saves copying their data.
        if (constant->use_empty())
          continue;
        FailureOr<HostOp> c = constantOf(constant);
        if (failed(c))
          return failure();
        producer[constant.getResult()] = static_cast<int32_t>(ops.size());
        ops.push_back(std::move(*c));
        continue;
      }
      if (auto call = dyn_cast<mlir::hexir::CallTIROp>(op)) {
        auto callee = symbols.lookup<hextir::PrimFuncOp>(call.getCallee());
        if (!callee)
          return call.emitError("callee is not a hextir.prim_func");
        FailureOr<HostOpKind> kind = kindOf(callee);
        if (failed(kind))
          return failure();
        HostOp h;
        h.kind = *kind;
        if (auto device = callee->getAttrOfType<StringAttr>("device"))
          h.device = device.getValue().str();
        if (failed(operandsOf(call, call.getArgs(), h)))
          return failure();
        producer[call.getResult()] = static_cast<int32_t>(ops.size());
        ops.push_back(std::move(h));
        continue;
      }
      if (auto print = dyn_cast<mlir::hexir::PrintOp>(op)) {
        HostOp h;
        h.kind = HostOpKind::Print;
        if (failed(operandsOf(print, print->getOperands(), h)))
          return failure();
        ops.push_back(std::move(h));
        continue;
      }
      if (isa<func::ReturnOp>(op))
        continue;
      return op.emitError("cannot serialize this op into a host program");
    }
  }

  std::string bytes, error;
  if (!writeModule(ops, flags, &bytes, &error))
    return module.emitError(error);
  os.write(bytes.data(), bytes.size());
  return success();
}

} // namespace hexir_b200
