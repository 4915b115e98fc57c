// tcgen05 (5th-generation tensor core) wrappers for the int8 projections: shared-memory matrix
// descriptors, the instruction descriptor of kind::i8, MMA issue/commit, TMEM allocation and loads.
// Operand layout used throughout: K-major, 128-byte swizzle; a 128-byte K block of R rows occupies
// R * 128 bytes, row r at (r / 8) * 1024 + (r % 8) * 128, its 16-byte chunk c at ((c ^ (r % 8)) * 16).
#pragma once

#include <cstdint>

#include "sm100_async.cuh"

namespace qb {
namespace umma {

constexpr int kTileM = 128;   // weight rows per MMA tile (TMEM lanes)
constexpr int kTileN = 16;    // activation-digit rows: digit d of token t in row 4 d + t
constexpr int kKBlock = 128;  // bytes of K per 128-byte swizzle atom
constexpr int kUnitBytes = kTileM * kKBlock;   // one weight block: 16 KB
constexpr int kDigitBlockBytes = kTileN * kKBlock;  // one digit block: 2 KB

// Byte offset of (row, byte k) inside one 128-byte-swizzled K block.
__host__ __device__ __forceinline__ uint32_t sw128_offset(int row, int k) {
  return (uint32_t)((row >> 3) * 1024 + (row & 7) * 128 + (((k >> 4) ^ (row & 7)) << 4) + (k & 15));
}

// Shared-memory matrix descriptor, K-major with 128-byte swizzle (8-row core groups 1024 bytes apart).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);  // start address (16-byte units)
  d |= (uint64_t)1 << 16;                    // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;          // stride byte offset: 8 rows x 128 bytes
  d |= (uint64_t)1 << 46;                    // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                    // 128-byte swizzle
  return d;
}

// Instruction descriptor of tcgen05.mma kind::i8: D = s32, A = B = signed 8-bit, both K-major.
constexpr uint32_t idesc_i8(int m, int n) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
constexpr uint32_t kIdescI8 = idesc_i8(kTileM, kTileN);

// Instruction descriptor of tcgen05.mma kind::f16: D = f32, A = B = f16, both K-major.
constexpr uint32_t idesc_f16(int m, int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// D[tmem] (+)= A . B^T with kind::f16 operands (K = 16 elements = 32 bytes per instruction), one thread.
template <uint32_t IDESC>
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\ntcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(
          d_tmem),
      "l"(a), "l"(b), "r"(IDESC), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[128 x 32 bytes] . B[16 x 32 bytes]^T, one elected thread.
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\ntcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}" ::"r"(
          d_tmem),
      "l"(a), "l"(b), "r"(kIdescI8), "r"(accumulate)
      : "memory");
}

// Same, always accumulating (no predicate set-up on the issue path).
__device__ __forceinline__ void mma_i8_acc(uint32_t d_tmem, uint64_t a, uint64_t b) {
  asm volatile("tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, 1;" ::"r"(d_tmem), "l"(a), "l"(b), "r"(kIdescI8)
               : "memory");
}

// The mbarrier completes one arrival once every MMA this thread issued before has finished.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Generic-proxy shared-memory writes made visible to the tensor core (async proxy).
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 16 consecutive 32-bit TMEM columns of the warp's 32 lanes.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, int (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 32 consecutive 32-bit TMEM columns of the warp's 32 lanes.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Whole-warp TMEM allocation (address written to shared memory), permit release and deallocation.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(cols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}

// Balanced int8 digits of X (|X| <= 8355711): X = d0 + 256 d1 + 65536 d2, each digit in [-128, 127].
__device__ __forceinline__ void split_digits(int X, int& d0, int& d1, int& d2) {
  d0 = ((X + 128) & 255) - 128;
  const int r1 = (X - d0) >> 8;
  d1 = ((r1 + 128) & 255) - 128;
  d2 = (r1 - d1) >> 8;
}

// Largest |X| the digit split represents, as the step divisor: step = max|x| / kDigitRange.
constexpr float kDigitRange = 8355710.0f;

// The digit integer X = rint(v / step) of the reference, whose quotient is the correctly rounded binary32
// division, computed as rint(RN32(RN64(v * r))) with r = RN64(1 / step): one double multiply per element
// instead of a float division (r is formed once per row). Both give the same X for all finite v, step > 0:
// - |q| < 2^-126 (q = v / step exactly): both quotients are below 1/2 in magnitude, X = 0 either way.
// - otherwise q lies in a normal binade [2^(e+23), 2^(e+24)) with binary32 spacing 2^e; RN32 of two values
//   differs only if a rounding midpoint M = m 2^(e-1) (m odd, m > 2^24) lies between them. Write v = V 2^a,
//   step = S 2^b (V, S odd integers below 2^24). q is not a midpoint (m S is odd and above 2^24, so
//   M step = m S 2^(b+e-1) cannot equal V 2^a), and |q - M| = |v - M step| / step is a nonzero multiple of
//   2^min(a, b+e-1) over step: >= 2^(e-25) > 2^-49 |q|, or >= |q| / V > 2^-24 |q|.
//   RN64(v r) = q (1 + d1)(1 + d2), |d1|, |d2| <= 2^-53, is within 2^-51 |q| of q: on the same side of
//   every midpoint, so it rounds to RN32(q).
// v and step are binary32, so their conversions to double are exact, and |v r| stays near kDigitRange.
__device__ __forceinline__ double digit_recip(float step) { return __ddiv_rn(1.0, (double)step); }
__device__ __forceinline__ int digit_quotient(float v, double r) {
  return (int)rintf(__double2float_rn(__dmul_rn((double)v, r)));
}

}  // namespace umma
}  // namespace qb
