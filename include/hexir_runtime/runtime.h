/*
 * runtime.h -- umbrella header, as in the reference
 * (runtime/include/hexir_runtime/runtime.h).  No MLIR or LLVM dependency.
 */
#ifndef HEXIR_RUNTIME_RUNTIME_H
#define HEXIR_RUNTIME_RUNTIME_H

#include "hexir_runtime/hal.h"
#include "hexir_runtime/module.h"
#include "hexir_runtime/program.h"
#include "hexir_runtime/status.h"
#include "hexir_runtime/vm.h"

#endif /* HEXIR_RUNTIME_RUNTIME_H */
