// common.cuh -- device helpers shared by the sm_100a kernels: the error word,
// mbarrier operations with bounded waits, TMA tile loads and the f64 DMMA.
#pragma once

#include <cuda.h>
#include <stdint.h>

#include "launch_abi.h"

// One word per CUDA context that kernels OR error bits into.  The host reads
// it after a stream synchronise (runtime/kernel_lib.cc) and clears it.
extern "C" __device__ unsigned int hexir_device_error_word;

namespace hexir {

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar,
                                                      uint32_t bytes) {
  asm volatile(
      "mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(
          smem_addr(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Wait until the phase with the given parity has completed, for at most
// `timeout_ns` of wall time.  On timeout the error word gets
// HEXIR_KERR_WAIT_TIMEOUT and the caller is told to abandon its loop; no wait
// in this project spins without a bound.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar,
                                                  uint32_t parity,
                                                  uint64_t timeout_ns) {
  if (mbar_try_wait(bar, parity))
    return true;
  const uint64_t start = global_timer_ns();
  for (uint32_t spin = 1;; ++spin) {
    if (mbar_try_wait(bar, parity))
      return true;
    if ((spin & 255u) == 0u && global_timer_ns() - start > timeout_ns) {
      atomicOr(&hexir_device_error_word, HEXIR_KERR_WAIT_TIMEOUT);
      return false;
    }
  }
}

// *p += v on a shared-memory word, returning the old value, with acquire and
// release semantics at CTA scope: what this thread did before is visible to
// a thread whose later add reads the result, and what threads did before
// their earlier adds is visible to this thread after it.
__device__ __forceinline__ uint32_t atom_add_acq_rel_cta(uint32_t *p,
                                                         uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], %2;"
               : "=r"(old)
               : "r"(smem_addr(p)), "r"(v)
               : "memory");
  return old;
}

// 2-D tiled TMA load into shared memory, completing on `bar`.  The caller
// keeps x * 8 bytes a multiple of 16 (x is a multiple of 8 doubles here).
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map,
                                            int32_t x, int32_t y,
                                            uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::"
      "bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y),
      "r"(smem_addr(bar))
      : "memory");
}

// 1-D bulk copy of `bytes` from global to this CTA's shared memory,
// completing on `bar`.  Both addresses 16-byte aligned, bytes a multiple of
// 16 (the caller checks).
__device__ __forceinline__ void bulk_load(void *dst, const void *src,
                                          uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1], %2, [%3];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// Thread-block clusters.  This CTA's rank in its cluster.
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Every thread of every CTA of the cluster: writes before it (shared memory
// included) are visible to reads after it in every CTA of the cluster.  The
// hardware barrier has no timeout, so every CTA of a cluster must execute
// the same sequence of these.
__device__ __forceinline__ void cluster_sync() {
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n\t"
      "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// An f64 in the shared memory of CTA `rank` of this cluster, at the place
// `local` has in this CTA's (distributed shared memory).
__device__ __forceinline__ double ld_cluster_f64(const double *local,
                                                 uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;"
               : "=r"(remote)
               : "r"(smem_addr(local)), "r"(rank));
  double v;
  asm volatile("ld.shared::cluster.f64 %0, [%1];"
               : "=d"(v)
               : "r"(remote)
               : "memory");
  return v;
}

// Programmatic dependent launch.  launch_dependents lets the next kernel of
// the stream, when it was launched with programmatic stream serialization,
// begin launching (its CTAs take SMs as this grid's CTAs retire); griddep_wait
// in that kernel then blocks until this grid has completed and its memory
// is visible.  For a kernel launched without the attribute both are no-ops
// (stream order already holds).  Neither can wait for ever: the wait ends
// when the prerequisite grid ends, and every wait inside these kernels is
// bounded.
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void griddep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(
                   reinterpret_cast<uint64_t>(map))
               : "memory");
}

// D = A(16x8) . B(8x8) + D in f64 on the tensor cores (DMMA).  Fragment
// positions, with g = lane / 4 and t = lane % 4 (PTX ISA, mma.m16n8k8 .f64):
//   a0 (g, t)  a1 (g+8, t)  a2 (g, t+4)  a3 (g+8, t+4)
//   b0 (t, g)  b1 (t+4, g)
//   d0 (g, 2t) d1 (g, 2t+1) d2 (g+8, 2t) d3 (g+8, 2t+1)
__device__ __forceinline__ void dmma_16x8x8(double (&d)[4], double a0,
                                            double a1, double a2, double a3,
                                            double b0, double b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f64.f64.f64.f64 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+d"(d[0]), "+d"(d[1]), "+d"(d[2]), "+d"(d[3])
      : "d"(a0), "d"(a1), "d"(a2), "d"(a3), "d"(b0), "d"(b1));
}

// 256-bit global accesses (sm_100): four consecutive f64, 32-byte aligned.
__device__ __forceinline__ void stg256(double *p, double a, double b, double c,
                                       double d) {
  asm volatile("st.global.v4.f64 [%0], {%1, %2, %3, %4};" ::"l"(p), "d"(a),
               "d"(b), "d"(c), "d"(d)
               : "memory");
}

// The same with the streaming (evict-first) cache hint: for outputs nothing
// in the kernel reads again, so they do not push the operands' panels out of
// L2.
__device__ __forceinline__ void stg256_cs(double *p, double a, double b,
                                          double c, double d) {
  asm volatile("st.global.cs.v4.f64 [%0], {%1, %2, %3, %4};" ::"l"(p), "d"(a),
               "d"(b), "d"(c), "d"(d)
               : "memory");
}

__device__ __forceinline__ void ldg256(const double *p, double (&v)[4]) {
  asm volatile("ld.global.v4.f64 {%0, %1, %2, %3}, [%4];"
               : "=d"(v[0]), "=d"(v[1]), "=d"(v[2]), "=d"(v[3])
               : "l"(p));
}

__device__ __forceinline__ double2 lds128(uint32_t addr) {
  double2 v;
  asm volatile("ld.shared.v2.f64 {%0, %1}, [%2];"
               : "=d"(v.x), "=d"(v.y)
               : "r"(addr));
  return v;
}

// The reference relu (runtime/src/kernels/reference_kernels.c:20-23):
// x > 0 ? x : 0.  NaN and -0.0 both become +0.0; written as a compare and
// select so no max instruction (which treats -0.0 and NaN differently) is
// substituted.
__device__ __forceinline__ double relu_ref(double x) {
  return (x > 0.0) ? x : 0.0;
}

}  // namespace hexir
