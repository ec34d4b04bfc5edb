// baseline_f64.cu -- the reference's own GPU schedule for hexir.linear,
// restated in CUDA C as a measurement baseline.  No product path launches
// it: the VM and the kernel-level C ABI run the DMMA kernels of
// linear_f64.cu.  It exists so the reference's GPU path, whose compiler
// cannot be built here, has a number on the same GPU.
//
// The schedule hexir-lower-to-tir gives a cuda-placed linear
// (compiler/Conversion/HexirToTIR/HexirToTIR.cpp:82-170) and hextir-to-gpu
// launches (compiler/Conversion/HexTIRToGPU/HexTIRToGPU.cpp:168-263):
//   - one thread per output element c[i][j];
//   - grid (n / bs, m), block (bs, 1), bs the largest power of two <= 256
//     dividing n (1 if n is odd): blockIdx.y = i, blockIdx.x * bs +
//     threadIdx.x = j, no bounds guard (the grid covers c exactly);
//   - the k loop serial, the running sum in a register from 0.0, one store;
//   - each multiply-add contracted to one fused multiply-add, as NVVM's
//     backend contracts the separate mulf / addf it is given.
// Operands are read straight from global memory (two loads per
// multiply-add, no shared-memory reuse), as the generated kernel does.

#include "common.cuh"

extern "C" __global__ void hexir_baseline_reference_schedule_f64(
    const double *__restrict__ a, const double *__restrict__ b,
    double *__restrict__ c, uint32_t n, uint32_t k) {
  const uint64_t i = blockIdx.y;
  const uint64_t j = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const double *row = a + i * k;
  double acc = 0.0;
  for (uint32_t p = 0; p < k; ++p)
    acc = fma(row[p], b[static_cast<uint64_t>(p) * n + j], acc);
  c[i * n + j] = acc;
}
