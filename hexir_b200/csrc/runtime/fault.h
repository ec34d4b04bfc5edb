// fault.h -- host-side fault injection (include/hexir_b200/fault.h).
//
// The runtime asks fault_hit() at each site where a real failure can occur:
// every allocation it makes (host slot storage, HAL buffers, kept
// constants, the split-K workspace), every kernel launch, and every grouped
// NCCL call of the in-process VM.  A hit makes that call fail the way the
// real failure would, so the error paths can be exercised without a GPU
// fault.  With no rule configured the check is one relaxed atomic load.
#pragma once

namespace hexir {

enum class FaultSite : int { Alloc = 0, Launch = 1, Nccl = 2 };

// Counts this call at `site`; true when a configured rule selects it.
bool fault_hit(FaultSite site);

}  // namespace hexir
