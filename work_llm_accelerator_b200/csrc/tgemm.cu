// Many-token int8 tensor-core projections (prefill; the same kernel serves any token count).
//
// Y[t][o] = scale[o] * s_t * sum_k code(o, k) * X_t[k]: each token row of fp32 activations is written
// exactly as s_t * (d0 + 256 d1 + 65536 d2) with three int8 digit planes (24-bit fixed point per token,
// the representation the decode path's qgemm.cu uses), so the tensor cores compute three exact int32
// products per output and the result differs from the reference's fp32 dot product
// (hls/prefill_only/qwen_prefill_attention_kernel.cpp:163-202, qwen_prefill_mlp_kernel.cpp:217-254) only by
// the 24-bit rounding of x (relative ~1e-7) and the fp32 summation order.
//
// One CTA computes a 128-row x TN-token tile (TN = 16, 32 or 64 for small batches; 64 with two CTAs per SM
// for many tokens, so that one CTA's epilogue overlaps the other's main loop). Per 128-byte K block the TMA
// producer stages the weight tile (16 KB) and the three plane tiles (3 x TN x 128 bytes, back to back, i.e.
// one 3 TN-row tile); one thread issues 4 tcgen05.mma (M = 128, N = 3 TN, K = 32 bytes; accumulator column
// p TN + n = plane p of token n); four warps read the accumulators back 16 tokens at a time, combine the
// planes exactly in int64 and run the epilogue of the projection (the same operations as the CUDA-core
// prefill kernels in prefill_simt.cu).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "tgemm.h"
#include "umma_sm100.cuh"

namespace qb {
namespace {

using namespace umma;

constexpr int kPlanes = 3;
constexpr int kThreadsT = 192;
constexpr int kEpiT = 128;
constexpr int kBarT = 1;       // named barrier of the epilogue warps
constexpr int kChunkN = 16;    // tokens per TMEM read
constexpr int kMaxStages = 8;

// Token-tile geometry: TN tokens per tile (16, 32, 64 or 128 = the padded token count up to 128), so that a
// small batch does not move or multiply padding.
// ST > 0 fixes the pipeline depth (ST = 2 with TN = 64 keeps a CTA under half of the shared memory, so
// two CTAs share an SM and one's epilogue overlaps the other's main loop); ST = 0 fills ~200 KB.
// ST = kPairST selects the CTA-pair form (TN = 64): two CTAs on two SMs compute a 256-row tile with
// tcgen05.mma.cta_group::2 (M = 256, N = 192); each holds its 128 weight rows and half of the 192 digit-plane
// rows, so a stage moves 16 + 12 KB per CTA instead of 16 + 24 KB; three stages, two CTAs per SM.
constexpr int kPairST = 3;
// ST = kPairDualST: the CTA-pair form with one CTA per SM (grids of one wave): a second MMA-issuing warp
// takes every other K block into a second accumulator (the epilogue adds the two exact int32 sums), so two
// issue streams run per tile, with six stages. Each issuing thread completes about one MMA per 147 ns
// whatever N is, so a tile's main loop is bound by its MMA count per issuer when the grid is one wave.
constexpr int kPairDualST = 4;
template <int TN, int ST = 0>
struct TCfg {
  static constexpr bool kPair = ST == kPairST || ST == kPairDualST;
  static constexpr bool kDual = ST == kPairDualST;
  static constexpr int kThreads = kDual ? kThreadsT + 32 : kThreadsT;
  static constexpr int kAccStride = 256;  // TMEM columns between the two accumulators (kDual)
  static constexpr int kPlaneTile = TN * kKBlock;
  static constexpr int kStage = kUnitBytes + (kPair ? kPlanes * kPlaneTile / 2 : kPlanes * kPlaneTile);
  static constexpr int kAutoStages = (200 * 1024) / kStage > kMaxStages ? kMaxStages : (200 * 1024) / kStage;
  static constexpr int kStages = kDual ? 6 : ST > 0 ? ST : kAutoStages;
  // The three plane tiles sit back to back in a stage, which is the layout of one 3 TN-row tile: up to
  // N = 256 one MMA covers all three planes (accumulator column p TN + n = plane p, token n).
  static constexpr bool kFused = kPlanes * TN <= 256;
  static constexpr uint32_t kIdesc = idesc_i8(kPair ? 2 * kTileM : kTileM, kFused ? kPlanes * TN : TN);
  static constexpr int kTmemCols = kDual ? 512
                                   : kPlanes * TN <= 32 ? 32 : kPlanes * TN <= 64 ? 64 : kPlanes * TN <= 128 ? 128
                                   : kPlanes * TN <= 256 ? 256 : 512;
  static_assert(!kDual || kPlanes * TN <= kAccStride, "two accumulators side by side");
  static_assert(TN % 16 == 0 && TN <= 128, "token tile");
  static_assert(!kPair || TN == 64, "the pair form splits 3 x 64 plane rows into two halves of 96");
};

struct TSmem {
  uint64_t full[kMaxStages], empty[kMaxStages], acc_full;
  uint32_t tmem_base;
  float steps[128];
  float ys[kTileM][kChunkN + 1];  // partner exchange (RoPE pairs, gate|up pairs)
};

enum TEpi { kTQkv = 0, kTScale = 1, kTGateUp = 2, kTDown = 3, kTRaw = 4 };

struct TArgs {
  int nkb;           // 128-byte K blocks
  int ksplit;        // K segments = CTAs of a cluster (1: no split)
  int box_rows;      // weight rows per TMA box: 128, or 64 twice (gate|up)
  int second_row0;   // gate|up: first row of the up half
  int S, Spad, rows;
  const float* steps;
  const float* scale;
  const float* bias;
  float* out;
  const float* resid;
  bool round_out;
  int* raw;
  bool decode;  // gate|up SiLU with expf (the decode reference) instead of approx_exp (the prefill reference)
};

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Every thread of every CTA of the cluster arrives once; release/acquire order shared-memory writes.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release;\nbarrier.cluster.wait.acquire;" ::: "memory");
}
// 32-bit store into the shared memory of CTA `rank` of the cluster, at the address `saddr` has in this CTA.
__device__ __forceinline__ void st_peer(uint32_t saddr, uint32_t rank, int v) {
  uint32_t pa;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(pa) : "r"(saddr), "r"(rank));
  asm volatile("st.shared::cluster.b32 [%0], %1;" ::"r"(pa), "r"(v) : "memory");
}

// ---- CTA-pair (cta_group::2) forms ----
// Address in the shared memory of CTA `rank` of the cluster that `saddr` has in this CTA.
__device__ __forceinline__ uint32_t peer_addr(uint32_t saddr, uint32_t rank) {
  uint32_t pa;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(pa) : "r"(saddr), "r"(rank));
  return pa;
}
// Bounded wait with cluster-scope acquire (for barriers another CTA of the cluster arrives on).
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n.reg .pred p;\nmbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, unsigned parity) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if (clock64() - t0 > 4000000000ll) {
      atomicExch(&g_kernel_error, kErrMbarTimeout);
      return false;
    }
  }
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)), "r"(cols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}
// One MMA over the pair: A rows 0..127 from the leader's and 128..255 from the peer's shared memory, B rows
// split the same way, D rows in each CTA's own TMEM. Issued by the leader.
template <uint32_t IDESC>
__device__ __forceinline__ void mma_pair(uint32_t d, uint64_t a, uint64_t b, uint32_t acc) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\ntcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n}" ::"r"(d),
      "l"(a), "l"(b), "r"(IDESC), "r"(acc)
      : "memory");
}
// The mbarrier at cluster address `bar` (this CTA's or the peer's) completes one arrival once every pair
// MMA issued before has finished.
__device__ __forceinline__ void mma_commit_pair(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
// TMA load into this CTA's shared memory whose completion counts on the leader's mbarrier (cluster address).
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, int c0, int c1, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(c0), "r"(c1), "r"(bar)
      : "memory");
}

template <uint32_t IDESC>
__device__ __forceinline__ void mma_t(uint32_t d, uint64_t a, uint64_t b, uint32_t acc) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\ntcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}" ::"r"(d),
      "l"(a), "l"(b), "r"(IDESC), "r"(acc)
      : "memory");
}

template <int EPI, int TN, int ST>
__global__ void __launch_bounds__(TCfg<TN, ST>::kThreads, (ST == 2 || ST == kPairST) ? 2 : 1)
    tgemm_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap pmap, TArgs a) {
  using C = TCfg<TN, ST>;
  constexpr int kTN = TN;
  constexpr int kStagesT = C::kStages;
  constexpr int kStageBytes = C::kStage;
  constexpr int kPlaneTile = C::kPlaneTile;
  constexpr int kTmemColsT = C::kTmemCols;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* stages = align_smem_1024(smem_raw);
  TSmem& sm = *reinterpret_cast<TSmem*>(stages + (size_t)kStagesT * kStageBytes);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // split K: the ksplit CTAs of a cluster share one output tile, CTA `rank` sums K blocks [kb_lo, kb_hi)
  // (the pair form does not split K: its cluster of two is the CTA pair, `prank` 0 the leader)
  constexpr bool kPair = C::kPair;
  const int ks = kPair ? 1 : a.ksplit;
  const int rank = ks > 1 ? (int)cluster_rank() : 0;
  const int prank = kPair ? (int)cluster_rank() : 0;
  const int mtile = blockIdx.x / ks, n0 = blockIdx.y * kTN;
  const int kb_lo = rank * a.nkb / ks, kb_hi = (rank + 1) * a.nkb / ks;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStagesT; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    mbar_init(&sm.acc_full, C::kDual ? 2 : 1);
    mbar_fence_init();
  }
  if (warp == 1) {
    if constexpr (kPair)
      tmem_alloc_pair(&sm.tmem_base, kTmemColsT);
    else
      tmem_alloc(&sm.tmem_base, kTmemColsT);
  }
  fence_before();
  __syncthreads();
  if constexpr (kPair) cluster_sync_all();  // both CTAs' barriers initialised before any cross-CTA signal
  fence_after();
  const uint32_t tmem = sm.tmem_base;
  // Programmatic dependent launch: everything above is local. The weights do not depend on the preceding
  // kernel, so the producer issues the first stages' weight tiles before waiting for it; the digit planes,
  // the token steps and every global write come after the wait.
  griddep_launch();

  if (warp == 0) {
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(&wmap) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(&pmap) : "memory");
      const int row0 = a.box_rows == kTileM ? mtile * kTileM : mtile * a.box_rows;
      int s = 0;
      unsigned ph = 0;
      bool ok = true;
      // pair form: every copy completes on the leader's full barrier
      const uint32_t full0 = kPair ? peer_addr(smem_u32(&sm.full[0]), 0) : 0u;
      auto load_weights = [&](int kb, int st_i) {
        uint8_t* st = stages + (size_t)st_i * kStageBytes;
        if constexpr (kPair) {
          if (prank == 0) mbar_arrive_expect_tx(&sm.full[st_i], 2 * kStageBytes);
          const uint32_t fb = full0 + 8u * st_i;
          tma_load_2d_pair(st, &wmap, kb * kKBlock, row0, fb);
          if (a.box_rows != kTileM) tma_load_2d_pair(st + a.box_rows * kKBlock, &wmap, kb * kKBlock, row0 + a.second_row0, fb);
        } else {
          mbar_arrive_expect_tx(&sm.full[st_i], kStageBytes);
          tma_load_2d(st, &wmap, kb * kKBlock, row0, &sm.full[st_i]);
          if (a.box_rows != kTileM)
            tma_load_2d(st + a.box_rows * kKBlock, &wmap, kb * kKBlock, row0 + a.second_row0, &sm.full[st_i]);
        }
      };
      auto load_planes = [&](int kb, int st_i) {
        uint8_t* st = stages + (size_t)st_i * kStageBytes;
        if constexpr (kPair) {
          const uint32_t fb = full0 + 8u * st_i;
#pragma unroll
          for (int i = 0; i < 3; ++i) {  // plane rows 96 prank + 32 i .. + 32 (row = 64 plane + token)
            const int pr = 96 * prank + 32 * i;
            tma_load_2d_pair(st + kUnitBytes + i * 32 * kKBlock, &pmap, kb * kKBlock, (pr / 64) * a.Spad + n0 + pr % 64,
                             fb);
          }
        } else {
#pragma unroll
          for (int p = 0; p < kPlanes; ++p)
            tma_load_2d(st + kUnitBytes + p * kPlaneTile, &pmap, kb * kKBlock, p * a.Spad + n0, &sm.full[st_i]);
        }
      };
      // the first stages are free (fresh barriers): their weight tiles go out before the dependency wait
      const int pre = min(kStagesT, kb_hi - kb_lo);
      for (int i = 0; i < pre; ++i) load_weights(kb_lo + i, i);
      griddep_wait();
      for (int i = 0; i < pre; ++i) load_planes(kb_lo + i, i);
      s = pre % kStagesT;
      ph = pre == kStagesT ? 1u : 0u;
      for (int kb = kb_lo + pre; kb < kb_hi && ok; ++kb) {
        if (!(ok = kPair ? mbar_wait_cluster(&sm.empty[s], ph ^ 1) : mbar_wait(&sm.empty[s], ph ^ 1))) break;
        load_weights(kb, s);
        load_planes(kb, s);
        if (++s == kStagesT) {
          s = 0;
          ph ^= 1;
        }
      }
      // every issued stage consumed before leaving (no copy in flight at exit)
      for (int i = 0; i < kStagesT && ok; ++i) {
        ok = kPair ? mbar_wait_cluster(&sm.empty[s], ph ^ 1) : mbar_wait(&sm.empty[s], ph ^ 1);
        if (++s == kStagesT) {
          s = 0;
          ph ^= 1;
        }
      }
    }
  } else if (warp == 1 || (C::kDual && warp == 6)) {
    // issuer 0 (warp 1) takes every K block, or with kDual the even ones (K block index from kb_lo) into the
    // first accumulator and issuer 1 (warp 6) the odd ones into the second
    const int iss = warp == 1 ? 0 : 1;
    if (lane == 0 && (!kPair || prank == 0)) {
      int s = 0;
      unsigned ph = 0;
      bool ok = true, first = true;
      const uint32_t dacc = tmem + (uint32_t)(iss * C::kAccStride);
      for (int kb = kb_lo; kb < kb_hi; ++kb) {
        if (!C::kDual || ((kb - kb_lo) & 1) == iss) {
          ok = ok && mbar_wait(&sm.full[s], ph);
          fence_after();
          if (ok) {
            const uint32_t sb = smem_u32(stages + (size_t)s * kStageBytes);
            const uint64_t ad = sw128_desc(sb);
#pragma unroll
            for (int p = 0; p < (C::kFused ? 1 : kPlanes); ++p) {
              const uint64_t bd = sw128_desc(sb + kUnitBytes + p * kPlaneTile);
#pragma unroll
              for (int j = 0; j < kKBlock / 32; ++j) {
                if constexpr (kPair)
                  mma_pair<C::kIdesc>(dacc + p * kTN, ad + 2 * j, bd + 2 * j, (!first || j > 0) ? 1u : 0u);
                else
                  mma_t<C::kIdesc>(dacc + p * kTN, ad + 2 * j, bd + 2 * j, (!first || j > 0) ? 1u : 0u);
              }
            }
          }
          first = false;
          if constexpr (kPair) {  // both CTAs' stage s is free once the pair MMAs finished
            mma_commit_pair(smem_u32(&sm.empty[s]));
            mma_commit_pair(peer_addr(smem_u32(&sm.empty[s]), 1));
          } else {
            mma_commit(&sm.empty[s]);
          }
        }
        if (++s == kStagesT) {
          s = 0;
          ph ^= 1;
        }
      }
      if constexpr (kPair) {
        mma_commit_pair(smem_u32(&sm.acc_full));
        mma_commit_pair(peer_addr(smem_u32(&sm.acc_full), 1));
      } else {
        mma_commit(&sm.acc_full);
      }
    }
  }
  // ---- epilogue: thread = one tile row (TMEM lane), 16 tokens per read
  // Split K: the tile's tokens are shared out over the cluster (CTA `rank` finishes tokens [tb, te)); once
  // every main loop is done each CTA pushes the partial sums of the other CTAs' tokens into their shared
  // memory (inbox [source rank][plane][token][row], in the then idle stage buffers), and after a second
  // cluster barrier sums its inbox in rank order (exact integers).
  const int q = warp & 3, r = q * 32 + lane;
  const int tp = kTN / ks;  // tokens per CTA of the cluster
  const int tb = rank * tp, te = tb + tp;
  const int* inbox = reinterpret_cast<const int*>(stages);
  bool ok = true;
  // Epilogue constants and the global loads of a chunk (the residual) do not depend on the accumulators:
  // the first chunk's are issued before the wait, behind the main loop.
  int row = 0;
  float sc = 0.f, bb = 0.f;
  float res[kChunkN];
  const int S_hi = min(a.S, n0 + te);  // tokens that exist and belong to this CTA
  auto chunk_loads = [&](int c0) {
    if constexpr (EPI == kTDown) {
#pragma unroll
      for (int c = 0; c < kChunkN; ++c) {
        const int n = n0 + c0 + c;
        res[c] = n < S_hi ? __ldg(a.resid + (size_t)n * kHidden + row) : 0.f;
      }
    }
  };
  if (warp >= 2 && warp < 6) {
    if constexpr (EPI == kTGateUp) {
      row = r < 64 ? mtile * 64 + r : a.second_row0 + mtile * 64 + (r - 64);
    } else {
      row = mtile * kTileM + r;
    }
    if constexpr (EPI != kTRaw) sc = __ldg(a.scale + row);
    if constexpr (EPI == kTQkv) bb = __ldg(a.bias + row);
    griddep_wait();  // the token steps (and the residual) come from earlier kernels
    if (r < kTN) sm.steps[r] = a.steps[n0 + r];
    named_sync(kBarT, kEpiT);
    if (tb < te && n0 + tb < a.S) chunk_loads(tb);
    ok = kPair ? mbar_wait_cluster(&sm.acc_full, 0) : mbar_wait(&sm.acc_full, 0);
    fence_after();
  }
  if (ks > 1) {
    cluster_sync_all();  // every CTA's main loop done: the cluster's stage memory is free
    if (warp >= 2 && warp < 6) {
      const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
      const uint32_t ib = smem_u32(stages);
      for (int c0 = 0; c0 < kPlanes * kTN; c0 += kChunkN) {
        int v[16];
        if (ok) {
          tmem_ld16(lane_base + c0, v);
        } else {
#pragma unroll
          for (int c = 0; c < 16; ++c) v[c] = 0;
        }
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const int col = c0 + c, pl = col / kTN, t = col % kTN;
          const int dst = t / tp, cc = t - dst * tp;
          st_peer(ib + (uint32_t)((((rank * kPlanes + pl) * tp + cc) * kTileM + r) * 4), dst, v[c]);
        }
      }
    }
    cluster_sync_all();  // every partial delivered
  }
  if (warp >= 2 && warp < 6) {
    const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
    for (int c0 = tb; c0 < te && n0 + c0 < a.S; c0 += kChunkN) {  // chunks holding real tokens only
      if (c0 != tb) chunk_loads(c0);
      int v0[16], v1[16], v2[16];
      if (ks > 1) {
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          v0[c] = v1[c] = v2[c] = 0;
          const int cc = c0 + c - tb;
          if (cc < tp) {
            for (int src = 0; src < ks; ++src) {
              const int* bx = inbox + ((src * kPlanes) * tp + cc) * kTileM + r;
              v0[c] += bx[0];
              v1[c] += bx[tp * kTileM];
              v2[c] += bx[2 * tp * kTileM];
            }
          }
        }
      } else if (ok) {
        tmem_ld16(lane_base + c0, v0);
        tmem_ld16(lane_base + kTN + c0, v1);
        tmem_ld16(lane_base + 2 * kTN + c0, v2);
        if constexpr (C::kDual) {  // the second issuer's K blocks (every issuer has at least one)
          int u[16];
          tmem_ld16(lane_base + C::kAccStride + c0, u);
#pragma unroll
          for (int c = 0; c < 16; ++c) v0[c] += u[c];
          tmem_ld16(lane_base + C::kAccStride + kTN + c0, u);
#pragma unroll
          for (int c = 0; c < 16; ++c) v1[c] += u[c];
          tmem_ld16(lane_base + C::kAccStride + 2 * kTN + c0, u);
#pragma unroll
          for (int c = 0; c < 16; ++c) v2[c] += u[c];
        }
      } else {
#pragma unroll
        for (int c = 0; c < 16; ++c) v0[c] = v1[c] = v2[c] = 0;
      }
      if constexpr (EPI == kTRaw) {
#pragma unroll
        for (int c = 0; c < kChunkN; ++c) {
          const int n = n0 + c0 + c;
          if (n < S_hi) {
            a.raw[((size_t)0 * a.S + n) * a.rows + row] = v0[c];
            a.raw[((size_t)1 * a.S + n) * a.rows + row] = v1[c];
            a.raw[((size_t)2 * a.S + n) * a.rows + row] = v2[c];
          }
        }
        continue;
      } else {
        float yv[kChunkN];
#pragma unroll
        for (int c = 0; c < kChunkN; ++c) {
          const long long tot = (long long)v0[c] + 256ll * (long long)v1[c] + 65536ll * (long long)v2[c];
          yv[c] = (float)((double)tot * (double)sm.steps[c0 + c]);
        }
        // every global load of the chunk is issued before any result is used (one round trip per chunk)
        if constexpr (EPI == kTScale || EPI == kTDown) {
#pragma unroll
          for (int c = 0; c < kChunkN; ++c) {
            const int n = n0 + c0 + c;
            float y = sc * yv[c];
            if constexpr (EPI == kTDown) {
              y = __fadd_rn(res[c], y);
              if (a.round_out) y = round_bf16(y);
            }
            if (n < S_hi) a.out[(size_t)n * kHidden + row] = y;
          }
        } else if constexpr (EPI == kTQkv) {
          // biased q|k|v rows [S][2048]; RoPE and the K/V row writes follow in qkv_rope_kernel
#pragma unroll
          for (int c = 0; c < kChunkN; ++c) {
            const int n = n0 + c0 + c;
            if (n < S_hi) a.out[(size_t)n * kQkvRows + row] = __fmaf_rn(sc, yv[c], bb);
          }
        } else {  // gate|up: tile rows 0..63 gate rows 64 j.., 64..127 the matching up rows
#pragma unroll
          for (int c = 0; c < kChunkN; ++c) sm.ys[r][c] = sc * yv[c];
          named_sync(kBarT, kEpiT);
          // all 128 threads: gate row (r & 63), tokens (r >> 6) * 8 .. +8 of the chunk
          const int gr = r & 63, cb = (r >> 6) * (kChunkN / 2);
#pragma unroll
          for (int c = cb; c < cb + kChunkN / 2; ++c) {
            const int n = n0 + c0 + c;
            const float gv = sm.ys[gr][c], uv = sm.ys[gr + 64][c];
            const float silu = __fdiv_rn(gv, __fadd_rn(1.0f, a.decode ? expf(-gv) : approx_exp_fast(-gv)));
            if (n < S_hi) a.out[(size_t)n * kInter + mtile * 64 + gr] = __fmul_rn(silu, uv);
          }
          named_sync(kBarT, kEpiT);
        }
      }
    }
  }
  fence_before();
  __syncthreads();
  if constexpr (kPair) cluster_sync_all();  // neither CTA leaves while the pair still uses its memory
  if (warp == 1) {
    fence_after();
    if constexpr (kPair)
      tmem_dealloc_pair(tmem, kTmemColsT);
    else
      tmem_dealloc(tmem, kTmemColsT);
  }
}

// One CTA per token row: per-token step and the three digit planes; padded rows become zero.
constexpr int kDigitVec = 9;  // float4 per thread: rows up to 9216 floats
__global__ void __launch_bounds__(256) digitize_kernel(const float* __restrict__ x, int S, int K, int Spad,
                                                       int8_t* __restrict__ planes, float* __restrict__ steps) {
  griddep_wait();  // inputs come from the preceding kernel (programmatic dependent launch)
  griddep_launch();
  const int t = blockIdx.x;
  __shared__ float red[8];
  int8_t* p0 = planes + (size_t)t * K;
  int8_t* p1 = planes + ((size_t)Spad + t) * K;
  int8_t* p2 = planes + ((size_t)2 * Spad + t) * K;
  if (t >= S) {
    for (int k = threadIdx.x * 4; k < K; k += 1024) {
      *reinterpret_cast<uint32_t*>(p0 + k) = 0u;
      *reinterpret_cast<uint32_t*>(p1 + k) = 0u;
      *reinterpret_cast<uint32_t*>(p2 + k) = 0u;
    }
    if (threadIdx.x == 0) steps[t] = 1.0f;
    return;
  }
  // the row is read once and held in registers (four values per float4, up to kDigitVec per thread)
  const float* row = x + (size_t)t * K;
  float4 v[kDigitVec];
  float m = 0.f;
#pragma unroll
  for (int i = 0; i < kDigitVec; ++i) {
    const int k = 4 * ((int)threadIdx.x + 256 * i);
    if (k < K) {
      v[i] = *reinterpret_cast<const float4*>(row + k);
      m = fmaxf(m, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  float mx = 0.f;
  for (int i = 0; i < 8; ++i) mx = fmaxf(mx, red[i]);
  const float st = mx > 0.0f ? mx / kDigitRange : 1.0f;
  if (threadIdx.x == 0) steps[t] = st;
  const double rst = digit_recip(st);
#pragma unroll
  for (int i = 0; i < kDigitVec; ++i) {
    const int k = 4 * ((int)threadIdx.x + 256 * i);
    if (k >= K) break;
    const float vv[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
    uint32_t w0 = 0, w1 = 0, w2 = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      int d0, d1, d2;
      split_digits(digit_quotient(vv[e], rst), d0, d1, d2);
      w0 |= (uint32_t)(d0 & 255) << (8 * e);
      w1 |= (uint32_t)(d1 & 255) << (8 * e);
      w2 |= (uint32_t)(d2 & 255) << (8 * e);
    }
    *reinterpret_cast<uint32_t*>(p0 + k) = w0;
    *reinterpret_cast<uint32_t*>(p1 + k) = w1;
    *reinterpret_cast<uint32_t*>(p2 + k) = w2;
  }
}

// Prefill RMSNorm (hls/prefill_only/qwen_prefill_attention_kernel.cpp:47-57,112-126) followed by the digit
// planes of the normalised rows, in one kernel: the same values as prefill_rmsnorm_kernel (prefill_simt.cu)
// followed by digitize_kernel, without writing the normalised rows to global memory. CTA = 2 token rows
// (so that short prompts still spread the digit divisions over many SMs), staged in shared memory by
// asynchronous 16-byte copies; lanes 0..1 of warp 0 run the reference's serial fp32 sums of squares, the
// rows are normalised in place, then every thread digitizes 12 values of each row.
constexpr int kPNormTok = 2, kPNormPad = kHidden + 4;  // rows padded by four floats: aligned, conflict-free
constexpr size_t kPNormSmem = (size_t)kPNormTok * kPNormPad * 4 + kPNormTok * 4 + 4 * kPNormTok * 4;

__global__ void __launch_bounds__(128) prefill_rmsnorm_digitize_kernel(const float* __restrict__ x,
                                                                       const float* __restrict__ w, int S, int Spad,
                                                                       int8_t* __restrict__ planes,
                                                                       float* __restrict__ steps) {
  griddep_wait();  // inputs come from the preceding kernel (programmatic dependent launch)
  griddep_launch();
  extern __shared__ __align__(16) float psm[];
  float* rows = psm;                            // [kPNormTok][kPNormPad]
  float* inv_s = psm + kPNormTok * kPNormPad;   // [kPNormTok]
  float* redm = inv_s + kPNormTok;              // [4 warps][kPNormTok]
  const int t0 = blockIdx.x * kPNormTok, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n = max(0, min(kPNormTok, S - t0));
  for (int i = tid; i < n * (kHidden / 4); i += 128) {
    const int r = i / (kHidden / 4), f = i % (kHidden / 4);
    const unsigned dst = (unsigned)__cvta_generic_to_shared(rows + r * kPNormPad + 4 * f);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(x + (size_t)(t0 + r) * kHidden + 4 * f)
                 : "memory");
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();
  if (tid < n) {
    const float* row = rows + tid * kPNormPad;
    float ms = 0.0f;
#pragma unroll 16
    for (int d = 0; d < kHidden; ++d) ms = __fadd_rn(ms, __fmul_rn(row[d], row[d]));
    ms = __fdiv_rn(ms, (float)kHidden);
    inv_s[tid] = __fdiv_rn(1.0f, approx_sqrt(__fadd_rn(ms, kEps)));
  }
  __syncthreads();
  // thread = values 4 tid + 512 j (j < 3) of every row: normalise (in registers), row maxima
  float v[kPNormTok][3][4];
#pragma unroll
  for (int r = 0; r < kPNormTok; ++r) {
    float m = 0.f;
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      const int k = 4 * tid + 512 * j;
      const float4 xv = *reinterpret_cast<const float4*>(rows + r * kPNormPad + k);
      const float4 wv = __ldg(reinterpret_cast<const float4*>(w + k));
      const float iv = r < n ? inv_s[r] : 0.f;
      v[r][j][0] = __fmul_rn(__fmul_rn(xv.x, iv), wv.x);
      v[r][j][1] = __fmul_rn(__fmul_rn(xv.y, iv), wv.y);
      v[r][j][2] = __fmul_rn(__fmul_rn(xv.z, iv), wv.z);
      v[r][j][3] = __fmul_rn(__fmul_rn(xv.w, iv), wv.w);
#pragma unroll
      for (int e = 0; e < 4; ++e) m = fmaxf(m, fabsf(v[r][j][e]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) redm[warp * kPNormTok + r] = m;
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < kPNormTok; ++r) {
    const int t = t0 + r;
    int8_t* p0 = planes + (size_t)t * kHidden;
    int8_t* p1 = planes + ((size_t)Spad + t) * kHidden;
    int8_t* p2 = planes + ((size_t)2 * Spad + t) * kHidden;
    if (r >= n) {  // padded token rows: zero digits, step 1
#pragma unroll
      for (int j = 0; j < 3; ++j) {
        const int k = 4 * tid + 512 * j;
        *reinterpret_cast<uint32_t*>(p0 + k) = 0u;
        *reinterpret_cast<uint32_t*>(p1 + k) = 0u;
        *reinterpret_cast<uint32_t*>(p2 + k) = 0u;
      }
      if (tid == 0) steps[t] = 1.0f;
      continue;
    }
    const float mx = fmaxf(fmaxf(redm[r], redm[kPNormTok + r]), fmaxf(redm[2 * kPNormTok + r], redm[3 * kPNormTok + r]));
    const float st = mx > 0.0f ? mx / kDigitRange : 1.0f;
    if (tid == 0) steps[t] = st;
    const double rst = digit_recip(st);
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      const int k = 4 * tid + 512 * j;
      uint32_t w0 = 0, w1 = 0, w2 = 0;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        int d0, d1, d2;
        split_digits(digit_quotient(v[r][j][e], rst), d0, d1, d2);
        w0 |= (uint32_t)(d0 & 255) << (8 * e);
        w1 |= (uint32_t)(d1 & 255) << (8 * e);
        w2 |= (uint32_t)(d2 & 255) << (8 * e);
      }
      *reinterpret_cast<uint32_t*>(p0 + k) = w0;
      *reinterpret_cast<uint32_t*>(p1 + k) = w1;
      *reinterpret_cast<uint32_t*>(p2 + k) = w2;
    }
  }
}

// Decode RMSNorm of n token rows (hls/decode_only/qwen_decode_attention_kernel.cpp:13-27): double sum of
// squares, inv = 1 / sqrt(ms + eps) in double, out = float(x * inv * w). 128 threads per token with the
// element assignment and reduction order of the persistent decode kernel (thread tid sums elements
// 512 j + 4 tid + e, xor-shuffle within the warp, the four warps in order), so both give identical rows.
__global__ void __launch_bounds__(128) decode_rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                             float* __restrict__ out) {
  griddep_wait();  // inputs come from the preceding kernel (programmatic dependent launch)
  griddep_launch();
  __shared__ double red[4];
  const int t = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const float* row = x + (size_t)t * kHidden;
  float v[3][4];
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const float4 f = *reinterpret_cast<const float4*>(row + 512 * j + 4 * tid);
    v[j][0] = f.x;
    v[j][1] = f.y;
    v[j][2] = f.z;
    v[j][3] = f.w;
  }
  double ss = 0.0;
#pragma unroll
  for (int j = 0; j < 3; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) ss += (double)v[j][e] * (double)v[j][e];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  const double tot = red[0] + red[1] + red[2] + red[3];
  const double inv = 1.0 / sqrt(tot / (double)kHidden + (double)kEps);
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const float4 wv = *reinterpret_cast<const float4*>(w + 512 * j + 4 * tid);
    float4 o;
    o.x = (float)((double)v[j][0] * inv * (double)wv.x);
    o.y = (float)((double)v[j][1] * inv * (double)wv.y);
    o.z = (float)((double)v[j][2] * inv * (double)wv.z);
    o.w = (float)((double)v[j][3] * inv * (double)wv.w);
    *reinterpret_cast<float4*>(out + (size_t)t * kHidden + 512 * j + 4 * tid) = o;
  }
}

// Decode RMSNorm (as decode_rmsnorm_kernel: same element assignment, double sums, reduction order) fused
// with the digit planes of the normalised row (as digitize_kernel: step = max|xn| / 8355710, digits of
// rint(xn / step)), one CTA of 128 threads per token; padded rows become zero.
__global__ void __launch_bounds__(128) rmsnorm_digitize_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                               int S, int Spad, int8_t* __restrict__ planes,
                                                               float* __restrict__ steps) {
  griddep_wait();  // inputs come from the preceding kernel (programmatic dependent launch)
  griddep_launch();
  __shared__ double red[4];
  __shared__ float redm[4];
  const int t = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  int8_t* p0 = planes + (size_t)t * kHidden;
  int8_t* p1 = planes + ((size_t)Spad + t) * kHidden;
  int8_t* p2 = planes + ((size_t)2 * Spad + t) * kHidden;
  if (t >= S) {
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      const int k = 512 * j + 4 * tid;
      *reinterpret_cast<uint32_t*>(p0 + k) = 0u;
      *reinterpret_cast<uint32_t*>(p1 + k) = 0u;
      *reinterpret_cast<uint32_t*>(p2 + k) = 0u;
    }
    if (tid == 0) steps[t] = 1.0f;
    return;
  }
  const float* row = x + (size_t)t * kHidden;
  float v[3][4];
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const float4 f = *reinterpret_cast<const float4*>(row + 512 * j + 4 * tid);
    v[j][0] = f.x;
    v[j][1] = f.y;
    v[j][2] = f.z;
    v[j][3] = f.w;
  }
  double ss = 0.0;
#pragma unroll
  for (int j = 0; j < 3; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) ss += (double)v[j][e] * (double)v[j][e];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  const double tot = red[0] + red[1] + red[2] + red[3];
  const double inv = 1.0 / sqrt(tot / (double)kHidden + (double)kEps);
  float m = 0.f;
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const float4 wv = *reinterpret_cast<const float4*>(w + 512 * j + 4 * tid);
    v[j][0] = (float)((double)v[j][0] * inv * (double)wv.x);
    v[j][1] = (float)((double)v[j][1] * inv * (double)wv.y);
    v[j][2] = (float)((double)v[j][2] * inv * (double)wv.z);
    v[j][3] = (float)((double)v[j][3] * inv * (double)wv.w);
#pragma unroll
    for (int e = 0; e < 4; ++e) m = fmaxf(m, fabsf(v[j][e]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) redm[warp] = m;
  __syncthreads();
  const float mx = fmaxf(fmaxf(redm[0], redm[1]), fmaxf(redm[2], redm[3]));
  const float st = mx > 0.0f ? mx / kDigitRange : 1.0f;
  if (tid == 0) steps[t] = st;
  const double rst = digit_recip(st);
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    uint32_t w0 = 0, w1 = 0, w2 = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      int d0, d1, d2;
      split_digits(digit_quotient(v[j][e], rst), d0, d1, d2);
      w0 |= (uint32_t)(d0 & 255) << (8 * e);
      w1 |= (uint32_t)(d1 & 255) << (8 * e);
      w2 |= (uint32_t)(d2 & 255) << (8 * e);
    }
    const int k = 512 * j + 4 * tid;
    *reinterpret_cast<uint32_t*>(p0 + k) = w0;
    *reinterpret_cast<uint32_t*>(p1 + k) = w1;
    *reinterpret_cast<uint32_t*>(p2 + k) = w2;
  }
}

// RoPE of the biased q|k|v rows and their destinations, one CTA of 256 threads per token. A thread takes the
// partner rows (d, d + 64) of a head: q and k heads rotate (d < 64: y_d = x_d cos - x_{d+64} sin,
// y_{d+64} = x_{d+64} cos + x_d sin, the reference's operations and order), v rows pass through. Prefill:
// position = token index, K/V rows into flat caches; decode: position pos[t], K/V rows through the paged view
// at (seq[t], pos[t]).
__global__ void __launch_bounds__(256) qkv_rope_kernel(const float* __restrict__ raw, const float* __restrict__ cosv,
                                                       const float* __restrict__ sinv, bool decode,
                                                       const int* __restrict__ posv, const int* __restrict__ seqv,
                                                       KvView kv, float* __restrict__ k_cache, float* __restrict__ v_cache,
                                                       float* __restrict__ q_out) {
  griddep_wait();  // inputs come from the preceding kernel (programmatic dependent launch)
  griddep_launch();
  const int t = blockIdx.x;
  const int pos = decode ? posv[t] : t;
  const float* x = raw + (size_t)t * kQkvRows;
  float* kdst = decode ? kv_row(kv, seqv[t], pos, 0) : k_cache + (size_t)t * kKvWidth;
  float* vdst = decode ? kv_row(kv, seqv[t], pos, 1) : v_cache + (size_t)t * kKvWidth;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int pr = threadIdx.x + 256 * i;  // pair index: head pr / 64, dims d and d + 64
    const int head = pr >> 6, d = pr & 63;
    const int r0 = head * kHeadDim + d, r1 = r0 + 64;
    const float x0 = x[r0], x1 = x[r1];
    float y0 = x0, y1 = x1;
    if (head < kHeads + kKvHeads) {
      const float c = cosv[(size_t)pos * 64 + d], sn = sinv[(size_t)pos * 64 + d];
      y0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
      y1 = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, sn));
    }
    if (head < kHeads) {
      q_out[(size_t)t * kHidden + r0] = y0;
      q_out[(size_t)t * kHidden + r1] = y1;
    } else if (head < kHeads + kKvHeads) {
      kdst[r0 - kHidden] = y0;
      kdst[r1 - kHidden] = y1;
    } else {
      vdst[r0 - kHidden - kKvWidth] = y0;
      vdst[r1 - kHidden - kKvWidth] = y1;
    }
  }
}

// ---------------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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

// 2D int8 map over [rows][k_bytes], box 128 bytes x box_rows, 128-byte swizzle
bool make_map(CUtensorMap* m, const void* base, uint64_t rows, uint64_t k_bytes, uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)k_bytes, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)k_bytes};
  cuuint32_t box[2] = {(cuuint32_t)kKBlock, box_rows};
  cuuint32_t es[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int EPI, int TN, int ST = 0>
cudaError_t run_tgemm_tn(const uint8_t* w, int rows_total, int K, int mtiles, int box_rows, int second_row0,
                         const DigitPlanes& x, TArgs a, cudaStream_t s, int ksplit = 1) {
  using C = TCfg<TN, ST>;
  if (x.K != K || K % kKBlock || x.Spad % TN || x.S < 1 || x.S > x.Spad) return cudaErrorInvalidValue;
  // split K: 1, 2, 4 or 8 CTAs per cluster, each with at least one K block; the inbox uses the stage memory
  if ((ksplit != 1 && ksplit != 2 && ksplit != 4 && ksplit != 8) || ksplit > K / kKBlock ||
      (ksplit > 1 && (size_t)C::kStages * C::kStage < (size_t)kPlanes * TN * kTileM * 4))
    return cudaErrorInvalidValue;
  a.ksplit = ksplit;
  CUtensorMap wmap, pmap;
  if (C::kPair && ((mtiles & 1) || ksplit != 1 || K / kKBlock < C::kStages)) return cudaErrorInvalidValue;
  if (C::kDual && K / kKBlock < 2) return cudaErrorInvalidValue;  // each issuer needs a K block
  if (!make_map(&wmap, w, (uint64_t)rows_total, (uint64_t)K, (uint32_t)box_rows) ||
      !make_map(&pmap, x.planes, (uint64_t)kPlanes * x.Spad, (uint64_t)K, C::kPair ? 32u : (uint32_t)TN))
    return cudaErrorInvalidValue;
  a.nkb = K / kKBlock;
  a.box_rows = box_rows;
  a.second_row0 = second_row0;
  a.S = x.S;
  a.Spad = x.Spad;
  a.steps = x.steps;
  auto kern = tgemm_kernel<EPI, TN, ST>;
  const size_t smem = 1024 + (size_t)C::kStages * C::kStage + sizeof(TSmem);
  static std::mutex mu;
  static unsigned long long attr_set = 0;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (dev < 64 && !((attr_set >> dev) & 1ull)) {
      if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)) != cudaSuccess)
        return e;
      attr_set |= 1ull << dev;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(mtiles * ksplit, x.Spad / TN);
  cfg.blockDim = dim3(C::kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  at[1].id = cudaLaunchAttributeClusterDimension;
  at[1].val.clusterDim.x = C::kPair ? 2 : ksplit;
  at[1].val.clusterDim.y = 1;
  at[1].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = (C::kPair || ksplit > 1) ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kern, wmap, pmap, a);
}

// K segments for a grid of `tiles` output tiles: as many (1, 2, 4 or 8, <= K blocks) as keep the grid within one
// wave of 148 SMs, so that projections with few row tiles (q|k|v, o_proj, down at small token counts) fill
// the GPU; 1 when the tiles alone fill it.
int pick_ksplit(int tiles, int nkb) {
  int k = 1;
  while (k < 8 && 2 * k <= nkb && tiles * 2 * k <= 148) k *= 2;
  return k;
}

template <int EPI>
cudaError_t run_tgemm(const uint8_t* w, int rows_total, int K, int mtiles, int box_rows, int second_row0,
                      const DigitPlanes& x, TArgs a, cudaStream_t s) {
  const int nkb = K / kKBlock;
  // 33-64 tokens: every row tile re-reads the token digit planes, which already outweigh its weights, so
  // the planes' traffic sets the time: CTA pairs (each CTA stages half of the planes) where the row tiles
  // pair up; K split (long K only: measured slower for the short-K projections) for the down projection.
  // A grid of CTA pairs that fits one wave of the 148 SMs takes the two-issuer form (one CTA per SM).
  const bool one_wave = mtiles * (x.Spad / 64) <= 148;
  if (x.Spad == 64) {
    const int ks = nkb >= 32 ? pick_ksplit(mtiles, nkb) : 1;
    if (ks == 1 && (mtiles & 1) == 0 && one_wave && nkb >= TCfg<64, kPairDualST>::kStages)
      return run_tgemm_tn<EPI, 64, kPairDualST>(w, rows_total, K, mtiles, box_rows, second_row0, x, a, s);
    if (ks == 1 && (mtiles & 1) == 0 && nkb >= TCfg<64, kPairST>::kStages)
      return run_tgemm_tn<EPI, 64, kPairST>(w, rows_total, K, mtiles, box_rows, second_row0, x, a, s);
    return run_tgemm_tn<EPI, 64>(w, rows_total, K, mtiles, box_rows, second_row0, x, a, s, ks);
  }
  if (x.Spad >= 128) {  // many tokens: 64-token tiles, two CTAs per SM unless K is split (long K only)
    const int ks = nkb >= 32 ? pick_ksplit(mtiles * (x.Spad / 64), nkb) : 1;
    if (ks > 1) return run_tgemm_tn<EPI, 64>(w, rows_total, K, mtiles, box_rows, second_row0, x, a, s, ks);
    if ((mtiles & 1) == 0 && one_wave && nkb >= TCfg<64, kPairDualST>::kStages)
      return run_tgemm_tn<EPI, 64, kPairDualST>(w, rows_total, K, mtiles, box_rows, second_row0, x, a, s);
    if ((mtiles & 1) == 0 && nkb >= TCfg<64, kPairST>::kStages)  // CTA pairs: 256-row tiles
      return run_tgemm_tn<EPI, 64, kPairST>(w, rows_total, K, mtiles, box_rows, second_row0, x, a, s);
    return run_tgemm_tn<EPI, 64, 2>(w, rows_total, K, mtiles, box_rows, second_row0, x, a, s);
  }
  // few tokens: split the long-K projection (down); measured slower for the short-K ones
  const int ks = nkb >= 32 ? pick_ksplit(mtiles, nkb) : 1;
  switch (x.Spad) {
    case 16: return run_tgemm_tn<EPI, 16>(w, rows_total, K, mtiles, box_rows, second_row0, x, a, s, ks);
    case 32: return run_tgemm_tn<EPI, 32>(w, rows_total, K, mtiles, box_rows, second_row0, x, a, s, ks);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

cudaError_t tgemm_rmsnorm_digitize(const float* x, const float* w, DigitPlanes d, cudaStream_t s) {
  if (d.K != kHidden || d.Spad != tgemm_pad(d.S) || d.S < 1) return cudaErrorInvalidValue;
  return launch_k(rmsnorm_digitize_kernel, dim3(d.Spad), dim3(128), 0, s, true, x, w, d.S, d.Spad, d.planes, d.steps);
}

cudaError_t tgemm_prefill_rmsnorm_digitize(const float* x, const float* w, DigitPlanes d, cudaStream_t s) {
  if (d.K != kHidden || d.Spad != tgemm_pad(d.S) || d.S < 1 || (reinterpret_cast<uintptr_t>(x) & 15))
    return cudaErrorInvalidValue;
  const cudaError_t attr = cudaFuncSetAttribute(prefill_rmsnorm_digitize_kernel,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPNormSmem);
  if (attr != cudaSuccess) return attr;
  return launch_k(prefill_rmsnorm_digitize_kernel, dim3(d.Spad / kPNormTok), dim3(128), kPNormSmem, s, true, x, w,
                  d.S, d.Spad, d.planes, d.steps);
}

cudaError_t tgemm_digitize(const float* x, DigitPlanes d, cudaStream_t s) {
  if (d.K % 4 || d.K > 4 * 256 * kDigitVec || d.Spad != tgemm_pad(d.S) || d.S < 1) return cudaErrorInvalidValue;
  return launch_k(digitize_kernel, dim3(d.Spad), dim3(256), 0, s, true, x, d.S, d.K, d.Spad, d.planes, d.steps);
}

cudaError_t tgemm_qkv(const LayerDev& L, const DigitPlanes& x, const float* rope_cos, const float* rope_sin, float* q_out,
                      float* k_cache, float* v_cache, float* raw, cudaStream_t s) {
  TArgs a{};
  a.scale = L.qkv_s;
  a.bias = L.qkv_b;
  a.out = raw;
  cudaError_t e = run_tgemm<kTQkv>(L.qkv_w, kQkvRows, kHidden, kQkvRows / kTileM, kTileM, 0, x, a, s);
  if (e != cudaSuccess) return e;
  return launch_k(qkv_rope_kernel, dim3(x.S), dim3(256), 0, s, true, static_cast<const float*>(raw), rope_cos, rope_sin,
                  false, static_cast<const int*>(nullptr), static_cast<const int*>(nullptr), KvView{}, k_cache, v_cache,
                  q_out);
}

cudaError_t tgemm_o(const LayerDev& L, const DigitPlanes& x, float* out, cudaStream_t s) {
  TArgs a{};
  a.scale = L.o_s;
  a.out = out;
  return run_tgemm<kTScale>(L.o_w, kHidden, kHidden, kHidden / kTileM, kTileM, 0, x, a, s);
}

cudaError_t tgemm_gateup(const LayerDev& L, const DigitPlanes& x, float* h, cudaStream_t s) {
  TArgs a{};
  a.scale = L.gu_s;
  a.out = h;
  return run_tgemm<kTGateUp>(L.gu_w, 2 * kInter, kHidden, kInter / 64, 64, kInter, x, a, s);
}

cudaError_t tgemm_down(const LayerDev& L, const DigitPlanes& x, const float* resid, float* out, bool round_out,
                       cudaStream_t s) {
  TArgs a{};
  a.scale = L.down_s;
  a.resid = resid;
  a.out = out;
  a.round_out = round_out;
  return run_tgemm<kTDown>(L.down_w, kHidden, kInter, kHidden / kTileM, kTileM, 0, x, a, s);
}

cudaError_t tgemm_qkv_decode(const LayerDev& L, const DigitPlanes& x, const int* pos, const int* seq, KvView kv,
                             const float* rope_cos, const float* rope_sin, float* q_out, float* raw, cudaStream_t s) {
  TArgs a{};
  a.scale = L.qkv_s;
  a.bias = L.qkv_b;
  a.out = raw;
  cudaError_t e = run_tgemm<kTQkv>(L.qkv_w, kQkvRows, kHidden, kQkvRows / kTileM, kTileM, 0, x, a, s);
  if (e != cudaSuccess) return e;
  return launch_k(qkv_rope_kernel, dim3(x.S), dim3(256), 0, s, true, static_cast<const float*>(raw), rope_cos, rope_sin,
                  true, pos, seq, kv, static_cast<float*>(nullptr), static_cast<float*>(nullptr), q_out);
}

cudaError_t tgemm_gateup_decode(const LayerDev& L, const DigitPlanes& x, float* h, cudaStream_t s) {
  TArgs a{};
  a.scale = L.gu_s;
  a.out = h;
  a.decode = true;
  return run_tgemm<kTGateUp>(L.gu_w, 2 * kInter, kHidden, kInter / 64, 64, kInter, x, a, s);
}

cudaError_t tgemm_raw(const uint8_t* codes, int rows, const DigitPlanes& x, int* acc, cudaStream_t s) {
  if (rows % kTileM) return cudaErrorInvalidValue;
  TArgs a{};
  a.raw = acc;
  a.rows = rows;
  return run_tgemm<kTRaw>(codes, rows, x.K, rows / kTileM, kTileM, 0, x, a, s);
}

cudaError_t decode_rmsnorm(const float* x, const float* w, int n, float* out, cudaStream_t s) {
  if (n < 1) return cudaErrorInvalidValue;
  return launch_k(decode_rmsnorm_kernel, dim3(n), dim3(128), 0, s, true, x, w, out);
}

unsigned tgemm_kernel_error(bool reset) {
  unsigned v = 0;
  if (cudaMemcpyFromSymbol(&v, g_kernel_error, sizeof(v)) != cudaSuccess) return 0xFFFFFFFFu;
  if (reset && v) {
    const unsigned z = 0;
    cudaMemcpyToSymbol(g_kernel_error, &z, sizeof(z));
  }
  return v;
}

}  // namespace qb
