// Causal prefill attention on the tensor cores (tcgen05 kind::f16), the prefill context of
// hls/prefill_only/qwen_prefill_attention_kernel.cpp:204-289 (12 query heads over 2 KV heads, head_dim 128).
//
// Numerics. Every fp32 operand x (Q, K, V and the softmax weights) is written as two fp16 values
// x = hi + lo with hi = fp16(x) and lo = fp16(x - hi) (22 significant bits), and every product as
// hi.hi + hi.lo + lo.hi accumulated in fp32 in TMEM; the dropped lo.lo term is 2^-22 of the product, so
// scores and context keep fp32-level error against the reference's serial fp32 sums. The softmax keeps the
// reference's two passes: pass 1 takes the row maximum of score * scaling over the causal keys, pass 2
// recomputes the scores and accumulates e = approx_exp(score * scaling - max) (the reference's exponential,
// bit for bit), the denominator sum e and the context sum e v, and divides once: ctx = acc * (1 / denom).
// The fp16 split needs |x| < 32768 and finite values; otherwise the split kernel raises a flag, this kernel
// does nothing and the CUDA-core kernel (attention.cu) computes the context instead.
//
// Work split. CTA = (128 queries, one query head); keys in tiles of 64. Q (hi, lo) sits in TMEM as the A
// operand of S = Q K^T, which leaves shared memory for four K stages (a K tile's TMA latency is longer than
// one tile's MMAs). Warp 0 issues the TMA loads (K tiles for both passes, transposed V tiles for pass 2),
// warp 1 issues the MMAs (S into one of two TMEM score buffers; O += P V into the TMEM context
// accumulator), and
// sixteen softmax warps own one query row and 16 keys of each tile per thread: they read the scores from
// TMEM, compute the weights, and write them as fp16 (hi, lo) tiles to shared memory for the P V product.
// Query tiles are launched heaviest (longest causal prefix) first.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <mutex>

#include "attention_tc.h"
#include "umma_sm100.cuh"

namespace qb {
namespace {

using namespace umma;

constexpr int kBQ = 128;  // query rows per CTA = TMEM lanes
constexpr int kBK = 64;   // keys per tile
constexpr int kKPlaneB = kBK * kHeadDim * 2;  // fp16 [64 keys][128 dims]: two 64-dim swizzle columns
constexpr int kVPlaneB = kHeadDim * kBK * 2;  // fp16 [128 dims][64 keys]: one swizzle column
constexpr int kPPlaneB = kBQ * kBK * 2;       // fp16 [128 queries][64 keys]: one swizzle column
constexpr int kKStages = 4;                      // K tiles in flight (their TMA latency exceeds one tile's MMAs)
constexpr int kOffK = 0;                         // kKStages stages of (hi, lo)
constexpr int kOffV = kOffK + kKStages * 2 * kKPlaneB;  // two stages of (hi, lo)
constexpr int kOffP = kOffV + 2 * 2 * kVPlaneB;  // (hi, lo)
constexpr int kTileBytes = kOffP + 2 * kPPlaneB;  // 160 KB
constexpr int kSoftWarps = 16;                  // four per TMEM lane quarter
constexpr int kSoftThreads = 32 * kSoftWarps;
constexpr int kKeyGroups = kSoftWarps / 4;      // key groups of a tile (one per warp of a lane quarter)
constexpr int kKeysPer = kBK / kKeyGroups;      // keys of a tile per softmax thread
constexpr int kThreadsA = 64 + kSoftThreads;
constexpr int kBarSoft = 1;  // named barrier of the softmax warps
// TMEM columns: context accumulator 0..127, score buffers 128.., 192.., Q (the A operand of S = Q K^T)
// 256..319 (hi) and 320..383 (lo), two fp16 dims per 32-bit column
constexpr uint32_t kTmemColsA = 512;
constexpr uint32_t kColS = 128;
constexpr uint32_t kColQ = 256;
constexpr uint32_t kIdescS = idesc_f16(kBQ, kBK);
constexpr uint32_t kIdescO = idesc_f16(kBQ, kHeadDim);
constexpr float kSplitLimit = 32768.0f;

struct ACtl {
  uint64_t q_full, k_full[kKStages], k_empty[kKStages], v_full[2], v_empty[2], s_full[2], s_empty[2], p_full, p_empty,
      o_full;
  uint32_t tmem_base;
};

constexpr size_t kSmemA = 1024 + (size_t)kTileBytes + sizeof(ACtl);
static_assert(kSmemA <= 232448, "shared memory per CTA");

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int c0, int c1, int c2,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}

// fp32 -> (hi, lo) fp16 planes. Blocks [0, nvt): V tiles of 64 tokens x 64 features, transposed into
// vt [2][256][Spad]; the rest: Q [Sq][1536] -> qp [2][Sq][1536] and K [S][256] -> kp [2][S][256], four
// values per thread (Sq = S, or the Sq queries of a prefill chunk after S - Sq cached keys). A value the
// split cannot hold (|x| >= 32768, inf, nan) sets *flag.
__global__ void __launch_bounds__(256) attn_split_kernel(const float* __restrict__ q, const float* __restrict__ k,
                                                         const float* __restrict__ v, int Sq, int S, int Spad, int nvt,
                                                         __half* __restrict__ qp, __half* __restrict__ kp,
                                                         __half* __restrict__ vt, int* __restrict__ flag) {
  griddep_wait();  // inputs come from the preceding kernel (programmatic dependent launch)
  griddep_launch();
  bool bad = false;
  if ((int)blockIdx.x < nvt) {
    __shared__ float tile[64][65];
    const int tb = blockIdx.x >> 2, fb = blockIdx.x & 3;
    const int tx = threadIdx.x & 63, ty = threadIdx.x >> 6;  // 64 x 4
    for (int i = ty; i < 64; i += 4) {
      const int t = tb * 64 + i;
      const float x = t < S ? v[(size_t)t * kKvWidth + fb * 64 + tx] : 0.0f;
      bad |= !(fabsf(x) < kSplitLimit);
      tile[i][tx] = x;
    }
    __syncthreads();
    for (int i = ty; i < 64; i += 4) {
      const float x = tile[tx][i];  // token tb*64 + tx, feature fb*64 + i
      const __half h = __float2half_rn(x);
      const __half l = __float2half_rn(__fsub_rn(x, __half2float(h)));
      const size_t o = (size_t)(fb * 64 + i) * Spad + tb * 64 + tx;
      vt[o] = h;
      vt[(size_t)kKvWidth * Spad + o] = l;
    }
  } else {
    const size_t nq4 = (size_t)Sq * kHidden / 4, nk4 = (size_t)S * kKvWidth / 4;
    const size_t stride = (size_t)(gridDim.x - nvt) * blockDim.x;
    for (size_t i = (size_t)(blockIdx.x - nvt) * blockDim.x + threadIdx.x; i < nq4 + nk4; i += stride) {
      const bool isq = i < nq4;
      const size_t j = isq ? i : i - nq4;
      const float4 x = reinterpret_cast<const float4*>(isq ? q : k)[j];
      const float xs[4] = {x.x, x.y, x.z, x.w};
      __half hs[4], ls[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        bad |= !(fabsf(xs[e]) < kSplitLimit);
        hs[e] = __float2half_rn(xs[e]);
        ls[e] = __float2half_rn(__fsub_rn(xs[e], __half2float(hs[e])));
      }
      __half* dst = isq ? qp : kp;
      const size_t plane = isq ? (size_t)Sq * kHidden : (size_t)S * kKvWidth;
      uint2 hv, lv;
      hv.x = (uint32_t)__half_as_ushort(hs[0]) | ((uint32_t)__half_as_ushort(hs[1]) << 16);
      hv.y = (uint32_t)__half_as_ushort(hs[2]) | ((uint32_t)__half_as_ushort(hs[3]) << 16);
      lv.x = (uint32_t)__half_as_ushort(ls[0]) | ((uint32_t)__half_as_ushort(ls[1]) << 16);
      lv.y = (uint32_t)__half_as_ushort(ls[2]) | ((uint32_t)__half_as_ushort(ls[3]) << 16);
      reinterpret_cast<uint2*>(dst)[j] = hv;
      reinterpret_cast<uint2*>(dst + plane)[j] = lv;
    }
  }
  if (__syncthreads_or(bad) && threadIdx.x == 0) atomicOr(flag, 1);
}

// D[tmem] (+)= A[tmem] . B[smem]^T, kind::f16, A read from TMEM (row m in lane m, element k of a K step in
// column k / 2, the lower k in the low half).
template <uint32_t IDESC>
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %3, 0;\ntcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %4, p;\n}" ::"r"(
          d_tmem),
      "r"(a_tmem), "l"(b), "r"(accumulate), "r"(IDESC)
      : "memory");
}

// 16 consecutive 32-bit TMEM columns of the warp's 32 lanes <- v (then wait for the stores).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// N consecutive 32-bit TMEM columns of the warp's 32 lanes (N = 16 or 32).
template <int N>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&v)[N]) {
  static_assert(N == 16 || N == 32, "columns");
  if constexpr (N == 32) {
    tmem_ld32(taddr, v);
  } else {
    tmem_ld16(taddr, reinterpret_cast<int(&)[16]>(v));
  }
}
__device__ __forceinline__ void tmem_ld_keys(uint32_t taddr, uint32_t (&v)[kKeysPer]) { tmem_ld_cols<kKeysPer>(taddr, v); }

// (a, b) -> fp16x2 bits, a in the low half (the lower address), one conversion instruction
__device__ __forceinline__ uint32_t half2_bits(float a, float b) {
  const __half2 p = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&p);
}

__global__ void __launch_bounds__(kThreadsA, 1)
    attn_tc_kernel(const __half* __restrict__ qp, const __grid_constant__ CUtensorMap kmap,
                   const __grid_constant__ CUtensorMap vmap, int Sq, int qoff, const int* flag,
                   float* __restrict__ ctx) {
  griddep_wait();  // inputs come from the preceding kernel (programmatic dependent launch)
  griddep_launch();
  if (*reinterpret_cast<const volatile int*>(flag) != 0) return;  // values outside the split: CUDA-core kernel
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* tiles = align_smem_1024(smem_raw);
  ACtl& c = *reinterpret_cast<ACtl*>(tiles + kTileBytes);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = gridDim.x - 1 - blockIdx.x;  // heaviest query tiles first
  const int h = blockIdx.y, g = h / kGroups;
  const int q0 = qt * kBQ;  // local query rows q0 .. q0 + 127 sit at positions qoff + q0 ..
  const int S = qoff + Sq;  // keys
  const int T = (min(qoff + q0 + kBQ, S) + kBK - 1) / kBK;  // key tiles of the causal prefix
  const int G = 2 * T;                                // pass 1 tiles, then pass 2 tiles

  if (threadIdx.x == 0) {
    mbar_init(&c.q_full, kSoftWarps);  // every softmax warp stored its part of Q in TMEM
    for (int i = 0; i < kKStages; ++i) {
      mbar_init(&c.k_full[i], 1);
      mbar_init(&c.k_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&c.v_full[i], 1);
      mbar_init(&c.v_empty[i], 1);
      mbar_init(&c.s_full[i], 1);
      mbar_init(&c.s_empty[i], kSoftWarps);
    }
    mbar_init(&c.p_full, kSoftWarps);
    mbar_init(&c.p_empty, 1);
    mbar_init(&c.o_full, 1);
    mbar_fence_init();
  }
  if (warp == 1) tmem_alloc(&c.tmem_base, kTmemColsA);
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = c.tmem_base;

  if (warp == 0) {
    // ---- TMA producer
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(&kmap) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(&vmap) : "memory");
      bool ok = true;
      int kn = 0, vn = 0;
      for (int gi = 0; gi < G && ok; ++gi) {
        const int j = gi < T ? gi : gi - T;
        {
          const int st = kn % kKStages;
          if (!(ok = mbar_wait(&c.k_empty[st], ((kn / kKStages) & 1) ^ 1))) break;
          mbar_arrive_expect_tx(&c.k_full[st], 2 * kKPlaneB);
          uint8_t* dst = tiles + kOffK + st * 2 * kKPlaneB;
          for (int p = 0; p < 2; ++p)
            for (int a = 0; a < 2; ++a)
              tma_load_3d(dst + p * kKPlaneB + a * (kBK * 128), &kmap, g * kHeadDim + a * 64, j * kBK, p,
                          &c.k_full[st]);
          ++kn;
        }
        if (gi >= T) {
          const int st = vn & 1;
          if (!(ok = mbar_wait(&c.v_empty[st], ((vn >> 1) & 1) ^ 1))) break;
          mbar_arrive_expect_tx(&c.v_full[st], 2 * kVPlaneB);
          uint8_t* dst = tiles + kOffV + st * 2 * kVPlaneB;
          for (int p = 0; p < 2; ++p) tma_load_3d(dst + p * kVPlaneB, &vmap, j * kBK, g * kHeadDim, p, &c.v_full[st]);
          ++vn;
        }
      }
      // every issued stage consumed before leaving (no copy in flight at exit)
      for (int i = 0; i < kKStages && ok; ++i, ++kn) ok = mbar_wait(&c.k_empty[kn % kKStages], ((kn / kKStages) & 1) ^ 1);
      for (int i = 0; i < 2 && ok; ++i, ++vn) ok = mbar_wait(&c.v_empty[vn & 1], ((vn >> 1) & 1) ^ 1);
    }
  } else if (warp == 1) {
    // ---- MMA issuer
    if (lane == 0) {
      bool ok = mbar_wait(&c.q_full, 0);
      fence_after();
      int kn = 0, vn = 0;
      // (A plane, B plane) of the three products, cross terms first: lo.hi, hi.lo, hi.hi
      constexpr int kAp[3] = {1, 0, 0}, kBp[3] = {0, 1, 0};
      auto issue_s = [&](int gi) {
        const int st = kn % kKStages;
        ok = ok && mbar_wait(&c.k_full[st], (kn / kKStages) & 1);
        fence_after();
        if (ok) {
          const uint32_t kb = smem_u32(tiles + kOffK + st * 2 * kKPlaneB);
          const uint32_t d = tmem + kColS + 64 * (gi & 1);
#pragma unroll
          for (int t = 0; t < 3; ++t)
#pragma unroll
            for (int kk = 0; kk < kHeadDim / 16; ++kk) {
              const uint32_t off = (uint32_t)((kk & 3) * 32);  // 16 dims = 32 bytes inside the swizzle row
              const uint64_t bd = sw128_desc(kb + kBp[t] * kKPlaneB + (kk >> 2) * (kBK * 128) + off);
              mma_f16_ts<kIdescS>(d, tmem + kColQ + 64 * kAp[t] + 8 * kk, bd, (t > 0 || kk > 0) ? 1u : 0u);
            }
        }
        mma_commit(&c.k_empty[st]);
        mma_commit(&c.s_full[gi & 1]);
        ++kn;
      };
      issue_s(0);
      issue_s(1);
      for (int gi = 0; gi < G; ++gi) {
        if (gi >= T) {
          const int j = gi - T;
          const int st = vn & 1;
          ok = ok && mbar_wait(&c.p_full, j & 1);
          ok = ok && mbar_wait(&c.v_full[st], (vn >> 1) & 1);
          fence_after();
          if (ok) {
            const uint32_t pa = smem_u32(tiles + kOffP);
            const uint32_t vb = smem_u32(tiles + kOffV + st * 2 * kVPlaneB);
#pragma unroll
            for (int t = 0; t < 3; ++t)
#pragma unroll
              for (int kk = 0; kk < kBK / 16; ++kk) {
                const uint64_t ad = sw128_desc(pa + kAp[t] * kPPlaneB + kk * 32);
                const uint64_t bd = sw128_desc(vb + kBp[t] * kVPlaneB + kk * 32);
                mma_f16<kIdescO>(tmem, ad, bd, (j > 0 || t > 0 || kk > 0) ? 1u : 0u);
              }
          }
          mma_commit(&c.p_empty);
          mma_commit(&c.v_empty[st]);
          ++vn;
        }
        if (gi + 2 < G) {
          ok = ok && mbar_wait(&c.s_empty[gi & 1], (gi >> 1) & 1);
          fence_after();
          issue_s(gi + 2);
        }
      }
      mma_commit(&c.o_full);
    }
  } else {
    // ---- softmax warps: thread = one query row, kKeysPer keys of each tile
    const int quarter = warp & 3;      // the TMEM lanes this warp may access
    const int kg = (warp - 2) >> 2;    // key group of each tile
    const int r = quarter * 32 + lane;
    const int qrow = q0 + r;       // local query row (row of qp and ctx)
    const int qpos = qoff + qrow;  // its position: keys 0 .. qpos are visible
    const uint32_t lane_addr = tmem + ((uint32_t)(quarter * 32) << 16);
    // per-row exchange between the key groups, in the weight tile's space while no weight tile is live
    float* xch = reinterpret_cast<float*>(tiles + kOffP);
    bool ok = true;
    {
      // Q of this row, dims [32 kg, 32 kg + 32) of head h, both planes -> TMEM (zero past the sequence)
      uint32_t qv[16];
#pragma unroll
      for (int pl = 0; pl < 2; ++pl) {
        const uint4* src = reinterpret_cast<const uint4*>(qp + ((size_t)pl * Sq + qrow) * kHidden + h * kHeadDim + 32 * kg);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint4 u = qrow < Sq ? src[i] : make_uint4(0u, 0u, 0u, 0u);
          qv[4 * i] = u.x;
          qv[4 * i + 1] = u.y;
          qv[4 * i + 2] = u.z;
          qv[4 * i + 3] = u.w;
        }
        tmem_st16(lane_addr + kColQ + 64 * pl + 16 * kg, qv);
      }
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&c.q_full);
    }
    uint32_t v[kKeysPer];
    // pass 1: row maximum of score * scaling over keys <= qrow
    float m = -1.0e30f;
    for (int gi = 0; gi < T; ++gi) {
      ok = ok && mbar_wait(&c.s_full[gi & 1], (gi >> 1) & 1);
      fence_after();
      if (ok) tmem_ld_keys(lane_addr + kColS + 64 * (gi & 1) + kKeysPer * kg, v);
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&c.s_empty[gi & 1]);
      const int kb = gi * kBK + kKeysPer * kg;
#pragma unroll
      for (int i = 0; i < kKeysPer; ++i) {
        const float ss = __fmul_rn(__uint_as_float(v[i]), kAttentionScaling);
        if (kb + i <= qpos && ss > m) m = ss;
      }
    }
    xch[kg * kBQ + r] = m;
    named_sync(kBarSoft, kSoftThreads);
    m = xch[r];
#pragma unroll
    for (int g2 = 1; g2 < kKeyGroups; ++g2) {
      const float mg = xch[g2 * kBQ + r];
      m = mg > m ? mg : m;
    }
    named_sync(kBarSoft, kSoftThreads);  // every row maximum read before the weight tile is written
    // pass 2: weights, denominator, and the fp16 (hi, lo) weight tiles for O += P V
    const F2 nz = f2_negzero(), sc2 = f2(kAttentionScaling, kAttentionScaling), m2 = f2(-m, -m);
    F2 den2 = f2(0.0f, 0.0f);
    const uint32_t prow = smem_u32(tiles + kOffP) + (uint32_t)((r >> 3) * 1024 + (r & 7) * 128);
    for (int j = 0; j < T; ++j) {
      const int gi = T + j;
      ok = ok && mbar_wait(&c.s_full[gi & 1], (gi >> 1) & 1);
      fence_after();
      if (ok) tmem_ld_keys(lane_addr + kColS + 64 * (gi & 1) + kKeysPer * kg, v);
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&c.s_empty[gi & 1]);
      const int kb = j * kBK + kKeysPer * kg;
      // e in [0, 1]: hi = e with the low 13 mantissa bits cleared (11 significant bits, an fp16 value for
      // e >= 2^-14), lo = e - hi (exact), both converted two at a time; below 2^-14 the pair is within 2^-24
      // of e, against a denominator >= 1.
      uint32_t ph[kKeysPer / 2], pl[kKeysPer / 2];
      float e[kKeysPer];
#pragma unroll
      for (int i = 0; i < kKeysPer; i += 2) {
        // score * scaling - max for two keys (the reference's two roundings), then the exponential
        const F2 a = add2(mul2(f2(__uint_as_float(v[i]), __uint_as_float(v[i + 1])), sc2, nz), m2);
        float x0, x1;
        approx_exp_fast2(f2_lo(a), f2_hi(a), x0, x1, nz);
        e[i] = select_f32(kb + i <= qpos, x0, 0.0f);
        e[i + 1] = select_f32(kb + i + 1 <= qpos, x1, 0.0f);
        den2 = add2(den2, f2(e[i], e[i + 1]));  // even and odd keys in two running sums
      }
#pragma unroll
      for (int i = 0; i < kKeysPer; i += 2) {
        const float h0 = __uint_as_float(__float_as_uint(e[i]) & 0xFFFFE000u);
        const float h1 = __uint_as_float(__float_as_uint(e[i + 1]) & 0xFFFFE000u);
        ph[i >> 1] = half2_bits(h0, h1);
        pl[i >> 1] = half2_bits(__fsub_rn(e[i], h0), __fsub_rn(e[i + 1], h1));
      }
      if (j > 0) ok = ok && mbar_wait(&c.p_empty, (j - 1) & 1);
#pragma unroll
      for (int ch = 0; ch < kKeysPer / 8; ++ch) {
        const uint32_t off = (uint32_t)((((kg * kKeysPer / 8 + ch) ^ (r & 7))) << 4);
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(prow + off), "r"(ph[4 * ch]),
                     "r"(ph[4 * ch + 1]), "r"(ph[4 * ch + 2]), "r"(ph[4 * ch + 3])
                     : "memory");
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(prow + kPPlaneB + off), "r"(pl[4 * ch]),
                     "r"(pl[4 * ch + 1]), "r"(pl[4 * ch + 2]), "r"(pl[4 * ch + 3])
                     : "memory");
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&c.p_full);
    }
    // every P V product done (the weight tile is free again), then the row denominator over the key groups
    float den = __fadd_rn(f2_lo(den2), f2_hi(den2));
    ok = ok && mbar_wait(&c.o_full, 0);
    fence_after();
    xch[kg * kBQ + r] = den;
    named_sync(kBarSoft, kSoftThreads);
    den = xch[r];
#pragma unroll
    for (int g2 = 1; g2 < kKeyGroups; ++g2) den = __fadd_rn(den, xch[g2 * kBQ + r]);
    const float inv = den > 0.0f ? __fdiv_rn(1.0f, den) : 0.0f;
    constexpr int kCols = kHeadDim / kKeyGroups;  // context columns of this thread
    uint32_t o[kCols];
    if (ok) tmem_ld_cols<kCols>(lane_addr + kCols * kg, o);
    if (ok && qrow < Sq) {
      float4* dst = reinterpret_cast<float4*>(ctx + (size_t)qrow * kHidden + h * kHeadDim + kCols * kg);
#pragma unroll
      for (int i = 0; i < kCols / 4; ++i)
        dst[i] = make_float4(__fmul_rn(__uint_as_float(o[4 * i]), inv), __fmul_rn(__uint_as_float(o[4 * i + 1]), inv),
                             __fmul_rn(__uint_as_float(o[4 * i + 2]), inv),
                             __fmul_rn(__uint_as_float(o[4 * i + 3]), inv));
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    tmem_dealloc(tmem, kTmemColsA);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn_a() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 3D fp16 map [d2][d1][d0] (d0 contiguous), row stride s1 bytes, plane stride s2 bytes; box b0 x b1 x 1,
// 128-byte swizzle, zero fill outside the extents.
bool make_map3(CUtensorMap* m, const void* base, uint64_t d0, uint64_t d1, uint64_t s1, uint64_t s2, uint32_t b0,
               uint32_t b1) {
  auto fn = encode_fn_a();
  if (!fn) return false;
  cuuint64_t dims[3] = {(cuuint64_t)d0, (cuuint64_t)d1, 2};
  cuuint64_t strides[2] = {(cuuint64_t)s1, (cuuint64_t)s2};
  cuuint32_t box[3] = {b0, b1, 1};
  cuuint32_t es[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

size_t round256(size_t b) { return (b + 255) / 256 * 256; }
int pad64(int S) { return (S + 63) / 64 * 64; }

}  // namespace

size_t prefill_attn_tc_scratch_bytes(int S) { return prefill_attn_tc_scratch_bytes(S, S); }

size_t prefill_attn_tc_scratch_bytes(int Sq, int S) {
  return 256 + round256((size_t)2 * Sq * kHidden * 2) + round256((size_t)2 * S * kKvWidth * 2) +
         round256((size_t)2 * kKvWidth * pad64(S) * 2);
}

cudaError_t launch_prefill_attention_tc(const float* q, const float* k_cache, const float* v_cache, int Sq, float* ctx,
                                        void* scratch, size_t scratch_bytes, cudaStream_t s, int qoff) {
  const int S = qoff + Sq;  // keys
  if (Sq < 1 || qoff < 0 || !scratch || scratch_bytes < prefill_attn_tc_scratch_bytes(Sq, S) ||
      (reinterpret_cast<uintptr_t>(scratch) & 255) || (reinterpret_cast<uintptr_t>(q) & 15) ||
      (reinterpret_cast<uintptr_t>(k_cache) & 15))
    return cudaErrorInvalidValue;
  const int Spad = pad64(S);
  uint8_t* base = static_cast<uint8_t*>(scratch);
  int* flag = reinterpret_cast<int*>(base);
  __half* qp = reinterpret_cast<__half*>(base + 256);
  __half* kp = reinterpret_cast<__half*>(base + 256 + round256((size_t)2 * Sq * kHidden * 2));
  __half* vt = reinterpret_cast<__half*>(reinterpret_cast<uint8_t*>(kp) + round256((size_t)2 * S * kKvWidth * 2));
  CUtensorMap kmap, vmap;
  if (!make_map3(&kmap, kp, kKvWidth, (uint64_t)S, kKvWidth * 2, (uint64_t)S * kKvWidth * 2, 64, kBK) ||
      !make_map3(&vmap, vt, (uint64_t)S, kKvWidth, (uint64_t)Spad * 2, (uint64_t)kKvWidth * Spad * 2, kBK, kHeadDim))
    return cudaErrorInvalidValue;
  cudaError_t e = cudaMemsetAsync(flag, 0, sizeof(int), s);
  if (e != cudaSuccess) return e;
  const int nvt = (Spad / 64) * 4;
  const size_t elems4 = ((size_t)Sq * kHidden + (size_t)S * kKvWidth) / 4;
  const int nqk = (int)std::min<size_t>((elems4 + 255) / 256, 148 * 8);
  if ((e = launch_k(attn_split_kernel, dim3(nvt + nqk), dim3(256), 0, s, true, q, k_cache, v_cache, Sq, S, Spad, nvt,
                    qp, kp, vt, flag)) != cudaSuccess)
    return e;
  if ((e = ensure_smem_attr((const void*)attn_tc_kernel, kSmemA)) != cudaSuccess) return e;
  if ((e = launch_k(attn_tc_kernel, dim3((Sq + kBQ - 1) / kBQ, kHeads), dim3(kThreadsA), kSmemA, s, true,
                    static_cast<const __half*>(qp), kmap, vmap, Sq, qoff, static_cast<const int*>(flag), ctx)) !=
      cudaSuccess)
    return e;
  // values outside the fp16 split: the CUDA-core kernel computes the context (it returns at once otherwise)
  return launch_prefill_attention_gated(q, k_cache, v_cache, Sq, ctx, flag, s, qoff);
}

unsigned attn_tc_kernel_error(bool reset) {
  unsigned v = 0;
  if (cudaMemcpyFromSymbol(&v, g_kernel_error, sizeof(v)) != cudaSuccess) return 0xFFFFFFFFu;
  if (reset && v) {
    const unsigned z = 0;
    cudaMemcpyToSymbol(g_kernel_error, &z, sizeof(z));
  }
  return v;
}

}  // namespace qb
