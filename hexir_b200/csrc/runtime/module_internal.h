// module_internal.h -- runtime state attached to a loaded module.
#pragma once

#include "hexir_runtime/module.h"

namespace hexir {

// The object attached to `module`, created by make(module) on first use and
// passed to detach() when the module is released (before its bytes go away).
// Thread safe.  Returns nullptr if make() returned nullptr.
void *module_attached(const hexir_module_t *module,
                      void *(*make)(const hexir_module_t *),
                      void (*detach)(void *));

}  // namespace hexir
