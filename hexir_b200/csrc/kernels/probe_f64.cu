// probe_f64.cu -- FP64 tensor-core throughput probe.  Every warp runs
// `iters` rounds of 8 independent m16n8k8 f64 DMMAs on register operands (no
// memory traffic), so the launch measures what the DMMA pipe sustains on this
// GPU at its current clock: the denominator of the GEMM's roofline fraction.
//
// FLOPs per launch = blocks * (threads / 32) * iters * 8 * (2 * 16 * 8 * 8).

#include "common.cuh"

using namespace hexir;

extern "C" __global__ void __launch_bounds__(256)
    hexir_dmma_peak_probe(double *out, uint32_t iters) {
  const uint32_t lane = threadIdx.x & 31;
  double acc[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int q = 0; q < 4; ++q)
      acc[i][q] = 0.0;
  const double a0 = 1.0 + lane * 1e-3, a1 = 1.0 - lane * 1e-3;
  const double a2 = 0.5 + lane * 1e-4, a3 = 0.25 - lane * 1e-4;
  const double b0 = 1e-6 * (lane + 1), b1 = -1e-6 * (lane + 2);
  for (uint32_t it = 0; it < iters; ++it) {
#pragma unroll
    for (int i = 0; i < 8; ++i)
      dmma_16x8x8(acc[i], a0, a1, a2, a3, b0, b1);
  }
  double s = 0.0;
#pragma unroll
  for (int i = 0; i < 8; ++i)
    s += acc[i][0] + acc[i][1] + acc[i][2] + acc[i][3];
  out[(size_t)blockIdx.x * blockDim.x + threadIdx.x] = s;
}

// Failure-detection probe: one thread waits on an mbarrier that nothing ever
// arrives at.  The wait gives up after `timeout_ns`, sets
// HEXIR_KERR_WAIT_TIMEOUT in the error word and the kernel returns, so the
// host sees an error status and the context stays usable.  Nothing is in
// flight when it exits.
extern "C" __global__ void hexir_wait_timeout_probe(uint64_t timeout_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0)
    mbar_wait_bounded(&bar, 0u, timeout_ns);
}

// Marker so a loader can tell an image of this kernel library (launch ABI
// version 1) from an arbitrary CUBIN.
extern "C" __global__ void hexir_b200_abi_v1() {}
