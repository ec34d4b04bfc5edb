// kernels.cu -- the single translation unit of the sm_100a kernel library.
// Built with `nvcc -cubin -gencode arch=compute_100a,code=sm_100a` into one
// CUBIN that the runtime loads with cuModuleLoadData: the copy embedded in
// libhexir_b200.so serves the kernel-level C ABI, and the writer embeds the
// same bytes in the EXECUTABLES section of every cuda-placed .hxb.

#include "common.cuh"

extern "C" __device__ unsigned int hexir_device_error_word = 0u;

#include "elementwise_f64.cu"
#include "activation_f64.cu"
#include "linear_f64.cu"
#include "linear_guarded_f64.cu"
#include "probe_f64.cu"
#include "baseline_f64.cu"
