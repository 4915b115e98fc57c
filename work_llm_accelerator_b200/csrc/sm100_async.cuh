// Thin wrappers over the sm_90+/sm_100 asynchronous-copy and mbarrier PTX used by the streaming kernels.
// Every wait is bounded: after ~2 s of polling it records an error code in a device flag and returns
// false, so a broken pipeline ends the kernel instead of hanging the GPU.
#pragma once

#include <cstdint>

namespace qb {

// Device error flag written by bounded waits that give up. Each translation unit that includes this header
// has its own copy and exports a host accessor; qwen_b200_kernel_error() combines them.
static __device__ unsigned g_kernel_error;

constexpr unsigned kErrMbarTimeout = 1u;

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// Rounds a shared-memory pointer up to a 1024-byte boundary by pointer arithmetic on the pointer itself. The
// compiler then still knows the result (and everything derived from it) lies in shared memory and emits
// shared-memory loads and stores; rounding through an integer cast loses that and gives generic accesses,
// which measured markedly slower in the latency-bound decode kernels.
__device__ __forceinline__ uint8_t* align_smem_1024(uint8_t* p) { return p + ((1024u - (smem_u32(p) & 1023u)) & 1023u); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n.reg .b64 st;\nmbarrier.arrive.shared::cta.b64 st, [%0];\n}" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("{\n.reg .b64 st;\nmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n}" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete; false (and the error flag set) after ~2 s.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (clock64() - t0 > 4000000000ll) {
      atomicExch(&g_kernel_error, kErrMbarTimeout);
      return false;
    }
  }
}

// Bulk global -> shared copy completing on an mbarrier (16-byte aligned, size a multiple of 16).
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gmem_src, unsigned bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void prefetch_l2(const void* p, unsigned bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Named barrier among `count` threads (a multiple of 32) of the CTA.
__device__ __forceinline__ void named_sync(unsigned id, unsigned count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

}  // namespace qb
