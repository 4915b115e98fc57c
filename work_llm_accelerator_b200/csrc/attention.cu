// GQA attention kernels (12 query heads over 2 KV heads, head_dim 128).
//
// Decode (hls/decode_only/qwen_decode_attention_kernel.cpp:113-162): the reference makes two passes over
// the whole history (max, then expf(s - max)). Here the history is split into 64-token chunks (one KV
// page each) and every (token, KV head, chunk) is one work item handling the 6 query heads that share the
// KV head, so each K/V row is read once for all six. The kernel is persistent: one CTA per SM walks a
// contiguous range of the flattened item list while a producer warp streams each item's K rows, V rows
// and query heads into shared-memory rings with tensor-map copies, so the HBM reads of later items
// overlap the arithmetic of the current one. Each chunk keeps its own max and writes a partial; a small
// follow-up kernel merges each (token, KV head)'s chunks in chunk order (rescaling by expf(m_c - M)), so
// the result equals the two-pass value up to rounding, is deterministic and does not depend on how items
// are spread over CTAs; a history of one chunk writes the context directly.
//
// Prefill (hls/prefill_only/qwen_prefill_attention_kernel.cpp:204-289): approx_exp(a) * approx_exp(b) is
// not approx_exp(a + b), so online rescaling would change results; the kernel keeps the reference's two
// passes: pass 1 takes the causal max of the scaled scores, pass 2 recomputes each score and accumulates
// approx_exp(score * scale - max). Scores, max and every exp value are bit-identical to the reference;
// only the order of the denominator and context sums differs.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>
#include <vector>

#include "qwen_kernels.cuh"
#include "sm100_async.cuh"

namespace qb {
namespace {

constexpr int kChunk = 64;                 // decode keys per work item (one KV page)
constexpr int kPartStride = 2 + kHeadDim;  // m, l, acc[128]
constexpr int kQHalf = kHeadDim / 2 + 4;   // padded half query row
constexpr int kStages = 3;                 // depth of the K ring and of the V ring
constexpr int kGroupThreads = 64;          // the score group (warps 0-1) and the P.V group (warps 2-3)
constexpr int kAttnThreads = 2 * kGroupThreads + 32;  // + warp 4: the loads
constexpr int kProducerWarp = 2 * kGroupThreads / 32;
constexpr int kMaxTokens = 1024;           // tokens per launch (prefix table); larger batches are split
// named barriers (0 is __syncthreads): score group, P.V group, weights full / empty by item parity
constexpr unsigned kBarScore = 1, kBarEsFull = 3, kBarEsEmpty = 5;

// K ring stage: four 32-float column blocks of 64 rows x 128 bytes with the 128-byte swizzle (16-byte chunk c
// of row r stored at chunk c ^ (r & 7): the score loop's column reads of consecutive keys are conflict-free)
// and the six query heads as padded half rows. V ring stage: 64 dense 512-byte rows.
struct DecodeAttnSmem {
  float ks[kStages][4][kChunk][32];  // 1024-byte aligned (swizzle atoms)
  float vs[kStages][kChunk][kHeadDim];
  float qs[kStages][kGroups][2][kQHalf];  // query head h, dims 64 * half ..
  float es[2][kGroups][kChunk];   // softmax weights, head-major; by item parity
  float xch[2][2][3][kChunk];     // score halves handed between the two score warps; by item parity
  float ms[2][kGroups], ls[2][kGroups];
  int prefix[kMaxTokens + 1];  // work items before token t (2 KV heads x its chunks)
  int len[kMaxTokens + 1];     // history length of token t including its new row (entry nt unused)
  uint64_t kfull[kStages], kempty[kStages], vfull[kStages], vempty[kStages];
  volatile int abort;  // a bounded wait gave up: every role stops working but keeps its barrier steps
};
constexpr size_t kDecodeAttnSmem = sizeof(DecodeAttnSmem) + 1024;  // + alignment slack
static_assert(kDecodeAttnSmem <= 232448, "shared memory per CTA");
constexpr unsigned kKStageBytes = 4 * kChunk * 128 + kGroups * kHeadDim * 4;
constexpr unsigned kVStageBytes = kChunk * kHeadDim * 4;

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void bar_arrive(unsigned id, unsigned count) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Hint: stream `bytes` of the next kernels' weights into L2 while this latency-bound kernel runs; the
// region is split evenly over the grid's CTAs.
__device__ __forceinline__ void prefetch_region(const uint8_t* pf, size_t bytes, unsigned cta, unsigned ctas,
                                                unsigned lane, unsigned lanes) {
  if (pf == nullptr || bytes == 0) return;
  const size_t per = ((bytes + ctas - 1) / ctas + 15) & ~size_t(15);
  const size_t b0 = (size_t)cta * per;
  const size_t b1 = min(bytes, b0 + per);
  for (size_t off = b0 + (size_t)lane * 16384; off < b1; off += (size_t)lanes * 16384)
    prefetch_l2(pf + off, (unsigned)min((size_t)16384, b1 - off));
}

// Work item j -> (token, KV head, chunk), items ordered by token, then head, then chunk.
struct Item {
  int t, g, c, L;
};

__device__ __forceinline__ Item item_of(const int* prefix, const int* len, int nt, int j) {
  int lo = 0, hi = nt - 1;  // last t with prefix[t] <= j
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (prefix[mid] <= j) lo = mid;
    else hi = mid - 1;
  }
  Item it;
  it.t = lo;
  it.L = len[lo];
  const int nch = (prefix[lo + 1] - prefix[lo]) >> 1;
  const int local = j - prefix[lo];
  it.g = local >= nch ? 1 : 0;
  it.c = local - it.g * nch;
  return it;
}

// The item after `it` in the (token, head, chunk) order.
__device__ __forceinline__ void item_next(Item& it, const int* len) {
  if (++it.c * kChunk < it.L) return;
  it.c = 0;
  if (++it.g < kKvHeads) return;
  it.g = 0;
  it.L = len[++it.t];
}

// Where one item's rows come from (resolved by one producer lane, handed to the others by shuffles).
struct ItemSrc {
  int ky, vy;       // tensor-map row of the chunk's K row 0 and V row 0
  int x;            // tensor-map column of this KV head (0 or 128)
  const float* qp;  // the six query heads of this KV head
  int dep;          // 1 if the chunk holds the new token's row (written by the preceding kernel)
};

__device__ __forceinline__ ItemSrc shfl_src(const ItemSrc& mine, int src) {
  ItemSrc r;
  r.ky = __shfl_sync(0xffffffffu, mine.ky, src);
  r.vy = __shfl_sync(0xffffffffu, mine.vy, src);
  r.x = __shfl_sync(0xffffffffu, mine.x, src);
  r.qp = reinterpret_cast<const float*>(__shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(mine.qp), src));
  r.dep = __shfl_sync(0xffffffffu, mine.dep, src);
  return r;
}

// Bounded wait that also gives up at once when another role has aborted.
__device__ __forceinline__ bool stage_wait(DecodeAttnSmem& sm, uint64_t* bar, unsigned parity) {
  if (sm.abort) return false;
  if (mbar_wait(bar, parity)) return true;
  sm.abort = 1;
  return false;
}

// The kernel is a three-role pipeline per CTA:
//   warp 4 (loads)   : K rows + query heads of item i into the K ring, V rows into the V ring (tensor-map and
//                      bulk copies), as ring slots free up;
//   warps 0-1 (score): item i's scores and softmax -> weights es[i & 1]; lane l owns keys l and l + 32 and
//                      warp w the 64-dim half w of every dot product, so each broadcast query float4 feeds
//                      two keys and the softmax runs from registers in the lane layout of the reference
//                      order (keys l and l + 32 per lane, then a butterfly over the warp);
//   warps 2-3 (P.V)  : item i-1's weighted V sums (lane = two dims, six heads), chunk partial / context, run
//                      publication and the merge.
// The two compute groups hand the weights over through named barriers (full: score arrives, P.V waits;
// empty: the reverse), so scores of one item overlap the P.V of the previous one. Shared-memory reads
// (the L1 data pipe) rather than arithmetic bound the compute roles, so the layout minimises broadcasts.
// kmap / vmap: 2D maps over the K and V rows (256 floats each; paged: every row of the pool, K and V alike).
__global__ void __launch_bounds__(kAttnThreads, 1) decode_attn_kernel(const __grid_constant__ CUtensorMap kmap,
                                                                      const __grid_constant__ CUtensorMap vmap,
                                                                      const float* __restrict__ q, KvView kv,
                                                                      DecodeTokens tok, int max_chunks,
                                                                      float* __restrict__ ctx,
                                                                      float* __restrict__ part,
                                                                      const uint8_t* pf, size_t pf_bytes) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  DecodeAttnSmem& sm = *reinterpret_cast<DecodeAttnSmem*>(smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023));
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int nt = tok.nt;

  // Positions were written before the preceding kernel started, so the item table is built before the
  // grid-dependency wait: prefix[t] = items of the tokens before t.
  for (int t = tid; t < nt; t += kAttnThreads) {
    const int L = tok.pos[t] + 1;
    sm.len[t] = L;
    sm.prefix[t + 1] = kKvHeads * ((L + kChunk - 1) / kChunk);
  }
  if (tid == 0) {
    sm.prefix[0] = 0;
    sm.abort = 0;
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&sm.kfull[i], 1);
      mbar_init(&sm.vfull[i], 1);
      mbar_init(&sm.kempty[i], kGroupThreads / 32);
      mbar_init(&sm.vempty[i], kGroupThreads / 32);
    }
    mbar_fence_init();
  }
  __syncthreads();
  if (warp == 0) {
    const int per = (nt + 31) / 32, a = min(nt, lane * per), b = min(nt, a + per);
    int sum = 0;
    for (int i = a; i < b; ++i) sum += sm.prefix[i + 1];
    int incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    int run = incl - sum;
    for (int i = a; i < b; ++i) {
      run += sm.prefix[i + 1];
      sm.prefix[i + 1] = run;
    }
  }
  __syncthreads();
  const int total = sm.prefix[nt];
  const int j0 = (int)((long long)blockIdx.x * total / gridDim.x);
  const int j1 = (int)((long long)(blockIdx.x + 1) * total / gridDim.x);
  const int count = j1 - j0;

  if (warp == kProducerWarp) {
    // ---------------- loads ----------------
    prefetch_region(pf, pf_bytes, blockIdx.x, gridDim.x, lane, 32);
    // lane l resolves item base + l (sequence, page-table lookups) so a batch of 32 costs one round trip
    auto resolve = [&](int i) {
      ItemSrc r = {0, 0, 0, nullptr, 0};
      if (i < count) {
        const Item it = item_of(sm.prefix, sm.len, nt, j0 + i);
        const int k0 = it.c * kChunk;
        if (kv.page_table == nullptr) {
          r.ky = r.vy = k0;
        } else {
          const int page = kv.page_table[tok.seq[it.t] * kv.max_pages + it.c];
          r.ky = ((page * kLayers + kv.layer) * 2) * kPage;
          r.vy = r.ky + kPage;
        }
        r.x = it.g * kHeadDim;
        r.qp = q + (size_t)it.t * kHidden + it.g * kGroups * kHeadDim;
        r.dep = (it.L - 1 - k0) < kChunk;
      }
      return r;
    };
    // one item's copies (elected lanes): phase 0 = K/V of a chunk without the new token's row (issued before
    // the grid-dependency wait), phase 1 = q and the remaining K/V (after it), phase 2 = everything
    auto issue_k = [&](int i, const ItemSrc& it, int phase) {
      const int s = i % kStages;
      if (phase != 1 && lane == 0) mbar_arrive_expect_tx(&sm.kfull[s], kKStageBytes);
      __syncwarp();
      const bool now = phase == 2 || (phase == 0) != (it.dep != 0);
      if (now && lane < 4) tma_load_2d(&sm.ks[s][lane][0][0], &kmap, it.x + 32 * lane, it.ky, &sm.kfull[s]);
      if (phase != 0 && lane >= 8 && lane < 8 + 2 * kGroups)
        bulk_g2s(&sm.qs[s][(lane - 8) >> 1][(lane - 8) & 1][0], it.qp + (lane - 8) * (kHeadDim / 2), kHeadDim * 2,
                 &sm.kfull[s]);
    };
    auto issue_v = [&](int i, const ItemSrc& it, int phase) {
      const int s = i % kStages;
      if (phase != 1 && lane == 0) mbar_arrive_expect_tx(&sm.vfull[s], kVStageBytes);
      __syncwarp();
      const bool now = phase == 2 || (phase == 0) != (it.dep != 0);
      if (now && lane == 0) tma_load_2d(&sm.vs[s][0][0], &vmap, it.x, it.vy, &sm.vfull[s]);
    };
    ItemSrc mine = resolve(lane);
    const int first = min(count, kStages);
    for (int i = 0; i < first; ++i) {
      const ItemSrc it = shfl_src(mine, i);
      issue_k(i, it, 0);
      issue_v(i, it, 0);
    }
    griddep_wait();
    griddep_launch();
    for (int i = 0; i < first; ++i) {
      const ItemSrc it = shfl_src(mine, i);
      issue_k(i, it, 1);
      issue_v(i, it, 1);
    }
    int k_issued = first, v_issued = first;
    for (int i = kStages; i < count; ++i) {
      if ((i & 31) == 0) mine = resolve(i + lane);
      const ItemSrc it = shfl_src(mine, i & 31);
      if (!stage_wait(sm, &sm.kempty[i % kStages], ((i / kStages) - 1) & 1)) break;
      issue_k(i, it, 2);
      k_issued = i + 1;
      if (!stage_wait(sm, &sm.vempty[i % kStages], ((i / kStages) - 1) & 1)) break;
      issue_v(i, it, 2);
      v_issued = i + 1;
    }
    // copies still in flight land before the CTA may exit (bounded waits, also after an abort)
    for (int i = max(0, k_issued - kStages); i < k_issued; ++i) mbar_wait(&sm.kfull[i % kStages], (i / kStages) & 1);
    for (int i = max(0, v_issued - kStages); i < v_issued; ++i) mbar_wait(&sm.vfull[i % kStages], (i / kStages) & 1);
    return;
  }

  griddep_wait();
  griddep_launch();
  Item it = item_of(sm.prefix, sm.len, nt, j0);

  if (warp < kGroupThreads / 32) {
    // ---------------- score group: lane = keys l and l + 32, warp = 64-dim half ----------------
    // Each score is the sum of two 64-dim halves (FMA chains over dims 0..63 and 64..127, each float4
    // consumed w, z, y, x), the order the persistent decode kernel uses, so both paths round alike. Warp
    // `half` computes its half of all six heads; warp 0 finishes heads 0-2, warp 1 heads 3-5.
    const float scaling = kAttentionScaling;  // == float(1 / sqrt(128)), qwen_decode_attention_kernel.cpp:119
    const int half = warp;
    const int sw = lane & 7;  // swizzle row of keys lane and lane + 32
    for (int i = 0; i < count; ++i, item_next(it, sm.len)) {
      const int s = i % kStages, b = i & 1;
      const int n = min(kChunk, it.L - it.c * kChunk);
      const bool ok_k = stage_wait(sm, &sm.kfull[s], (i / kStages) & 1);
      float pa[kGroups], pb[kGroups];
#pragma unroll
      for (int h = 0; h < kGroups; ++h) pa[h] = pb[h] = 0.f;
      if (ok_k) {
#pragma unroll 4
        for (int f = 0; f < 16; ++f) {
          const int F = 16 * half + f;
          const float4 ka = *reinterpret_cast<const float4*>(&sm.ks[s][F >> 3][lane][4 * ((F & 7) ^ sw)]);
          const float4 kb = *reinterpret_cast<const float4*>(&sm.ks[s][F >> 3][lane + 32][4 * ((F & 7) ^ sw)]);
#pragma unroll
          for (int h = 0; h < kGroups; ++h) {
            const float4 qq = *reinterpret_cast<const float4*>(&sm.qs[s][h][half][4 * f]);
            pa[h] = fmaf(qq.x, ka.x, fmaf(qq.y, ka.y, fmaf(qq.z, ka.z, fmaf(qq.w, ka.w, pa[h]))));
            pb[h] = fmaf(qq.x, kb.x, fmaf(qq.y, kb.y, fmaf(qq.z, kb.z, fmaf(qq.w, kb.w, pb[h]))));
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.kempty[s]);  // this warp is done with the K stage
      // hand the halves of the other warp's heads over
      float ka[3], kb2[3];  // this warp's halves of the heads it finishes (3 * half + j)
#pragma unroll
      for (int j = 0; j < 3; ++j) {
        sm.xch[b][half][j][lane] = half ? pa[j] : pa[3 + j];
        sm.xch[b][half][j][lane + 32] = half ? pb[j] : pb[3 + j];
        ka[j] = half ? pa[3 + j] : pa[j];
        kb2[j] = half ? pb[3 + j] : pb[j];
      }
      named_sync(kBarScore, kGroupThreads);
      if (i >= 2) named_sync(kBarEsEmpty + b, 2 * kGroupThreads);  // P.V is done with es[b] (item i - 2)
      if (ok_k && !sm.abort) {
        // the three heads' reductions are interleaved (independent shuffle chains)
        float a[3], bb[3], m[3], ea[3], eb[3], l[3];
#pragma unroll
        for (int j = 0; j < 3; ++j) {
          const float oa = sm.xch[b][1 - half][j][lane], ob = sm.xch[b][1 - half][j][lane + 32];
          a[j] = lane < n ? __fadd_rn(ka[j], oa) * scaling : -INFINITY;
          bb[j] = lane + 32 < n ? __fadd_rn(kb2[j], ob) * scaling : -INFINITY;
          m[j] = fmaxf(a[j], bb[j]);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
          for (int j = 0; j < 3; ++j) m[j] = fmaxf(m[j], __shfl_xor_sync(0xffffffffu, m[j], o));
#pragma unroll
        for (int j = 0; j < 3; ++j) {
          m[j] = fmaxf(m[j], -1.0e30f);  // the reference's initial max
          ea[j] = lane < n ? expf(a[j] - m[j]) : 0.f;
          eb[j] = lane + 32 < n ? expf(bb[j] - m[j]) : 0.f;
          sm.es[b][3 * half + j][lane] = ea[j];
          sm.es[b][3 * half + j][lane + 32] = eb[j];
          l[j] = ea[j] + eb[j];
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
          for (int j = 0; j < 3; ++j) l[j] += __shfl_xor_sync(0xffffffffu, l[j], o);
        if (lane == 0) {
#pragma unroll
          for (int j = 0; j < 3; ++j) {
            sm.ms[b][3 * half + j] = m[j];
            sm.ls[b][3 * half + j] = l[j];
          }
        }
      }
      bar_arrive(kBarEsFull + b, 2 * kGroupThreads);  // weights of item i are in es[b]
    }
    return;
  }

  // ---------------- P.V group: lane = dims d, d + 1 (warp 2: 0..63, warp 3: 64..127), six heads ----------------
  const int d = 2 * (tid - kGroupThreads);
  for (int i = 0; i < count; ++i, item_next(it, sm.len)) {
    const int s = i % kStages, b = i & 1;
    const int n = min(kChunk, it.L - it.c * kChunk);
    const int nchunks = (it.L + kChunk - 1) / kChunk;
    named_sync(kBarEsFull + b, 2 * kGroupThreads);
    const bool ok_v = stage_wait(sm, &sm.vfull[s], (i / kStages) & 1);
    const bool work = ok_v && !sm.abort;
    // keys in order; keys past the history have weight 0 and their V rows (whatever the page holds there)
    // are replaced by 0, so they leave the sums unchanged
    float a0[kGroups], a1[kGroups];
#pragma unroll
    for (int h = 0; h < kGroups; ++h) a0[h] = a1[h] = 0.f;
    if (work) {
#pragma unroll 2
      for (int k0 = 0; k0 < kChunk; k0 += 4) {
        float4 e[kGroups];
#pragma unroll
        for (int h = 0; h < kGroups; ++h) e[h] = *reinterpret_cast<const float4*>(&sm.es[b][h][k0]);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const float2 vr = *reinterpret_cast<const float2*>(&sm.vs[s][k0 + kk][d]);
          const bool ok = k0 + kk < n;
          const float v0 = ok ? vr.x : 0.0f, v1 = ok ? vr.y : 0.0f;
#pragma unroll
          for (int h = 0; h < kGroups; ++h) {
            const float w = kk == 0 ? e[h].x : kk == 1 ? e[h].y : kk == 2 ? e[h].z : e[h].w;
            a0[h] = fmaf(w, v0, a0[h]);
            a1[h] = fmaf(w, v1, a1[h]);
          }
        }
      }
    }
    float lsum[kGroups];
#pragma unroll
    for (int h = 0; h < kGroups; ++h) lsum[h] = sm.ls[b][h];
    const int hl = tid - kGroupThreads;  // 0..63: threads 0..5 write the six heads' m and l
    const float mine_m = hl < kGroups ? sm.ms[b][hl] : 0.f;
    const float mine_l = hl < kGroups ? sm.ls[b][hl] : 0.f;
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.vempty[s]);  // this warp is done with the V stage
    if (i + 2 < count) bar_arrive(kBarEsEmpty + b, 2 * kGroupThreads);  // es[b] may take item i + 2
    if (!work) continue;

    float* out_base = ctx + (size_t)it.t * kHidden + it.g * kGroups * kHeadDim + d;
    if (nchunks == 1) {
#pragma unroll
      for (int h = 0; h < kGroups; ++h) {
        const float inv = lsum[h] > 0.0f ? 1.0f / lsum[h] : 0.0f;
        *reinterpret_cast<float2*>(out_base + h * kHeadDim) = make_float2(a0[h] * inv, a1[h] * inv);
      }
      continue;
    }
    const size_t tg = (size_t)it.t * kKvHeads + it.g;
    float* my = part + (tg * max_chunks + it.c) * kGroups * kPartStride;
#pragma unroll
    for (int h = 0; h < kGroups; ++h)
      *reinterpret_cast<float2*>(my + h * kPartStride + 2 + d) = make_float2(a0[h], a1[h]);
    if (hl < kGroups) {
      my[hl * kPartStride + 0] = mine_m;
      my[hl * kPartStride + 1] = mine_l;
    }
  }
}

// Merge of one (token, KV head)'s chunk partials, in chunk order (deterministic, the same operations as the
// persistent decode kernel): M' = max(M, m_c), o = o e^(M - M') + acc_c e^(m_c - M'), L likewise. The
// rescale factors depend only on the chunk maxima, so one thread per head computes them once; then every
// (head, dim) chain folds its chunks with all of its loads in flight together. Runs after the attention
// kernel (programmatic dependent launch: its prologue overlaps that kernel's tail).
constexpr int kMergeThreads = kGroups * kHeadDim;  // 768: thread = (head, dim)
constexpr int kMergeLoads = 16;                    // chunk values loaded together per chain

__global__ void __launch_bounds__(kMergeThreads) decode_attn_merge_kernel(DecodeTokens tok, int max_chunks,
                                                                          float* __restrict__ ctx,
                                                                          const float* __restrict__ part) {
  extern __shared__ float msm[];  // m[6][nc], l[6][nc], sa[6][nc], sb[6][nc], inv[6]
  const int t = blockIdx.x, g = blockIdx.y, tid = threadIdx.x;
  const int L = tok.pos[t] + 1;
  const int nc = (L + kChunk - 1) / kChunk;
  griddep_wait();  // the attention kernel's partials
  griddep_launch();
  if (nc <= 1) return;  // that kernel wrote the context directly
  float* mv = msm;
  float* lv = mv + kGroups * nc;
  float* sa = lv + kGroups * nc;
  float* sb = sa + kGroups * nc;
  float* inv = sb + kGroups * nc;
  const float* base = part + ((size_t)t * kKvHeads + g) * max_chunks * kGroups * kPartStride;
  const int h = tid / kHeadDim, d = tid % kHeadDim;
  const float* src = base + (size_t)h * kPartStride + 2 + d;
  // the first chunks' values do not depend on the rescale factors: their loads go out first
  float av[kMergeLoads];
#pragma unroll
  for (int k = 0; k < kMergeLoads; ++k) av[k] = __ldcg(src + (size_t)min(k, nc - 1) * kGroups * kPartStride);
  for (int i = tid; i < kGroups * nc; i += kMergeThreads) {
    const int c = i / kGroups, hh = i % kGroups;
    mv[hh * nc + c] = __ldcg(base + ((size_t)c * kGroups + hh) * kPartStride);
    lv[hh * nc + c] = __ldcg(base + ((size_t)c * kGroups + hh) * kPartStride + 1);
  }
  __syncthreads();
  if (tid < kGroups) {
    float M = -INFINITY, Lsum = 0.f;
    for (int c = 0; c < nc; ++c) {
      const float Mn = fmaxf(M, mv[tid * nc + c]);
      const float fa = expf(M - Mn), fb = expf(mv[tid * nc + c] - Mn);
      sa[tid * nc + c] = fa;
      sb[tid * nc + c] = fb;
      Lsum = __fadd_rn(__fmul_rn(Lsum, fa), __fmul_rn(lv[tid * nc + c], fb));
      M = Mn;
    }
    inv[tid] = Lsum > 0.0f ? 1.0f / Lsum : 0.0f;
  }
  __syncthreads();
  float o = 0.f;
  for (int c0 = 0; c0 < nc; c0 += kMergeLoads) {
    if (c0 > 0) {
#pragma unroll
      for (int k = 0; k < kMergeLoads; ++k)
        av[k] = __ldcg(src + (size_t)min(c0 + k, nc - 1) * kGroups * kPartStride);
    }
#pragma unroll
    for (int k = 0; k < kMergeLoads; ++k)
      if (c0 + k < nc) o = __fadd_rn(__fmul_rn(o, sa[h * nc + c0 + k]), __fmul_rn(av[k], sb[h * nc + c0 + k]));
  }
  ctx[(size_t)t * kHidden + (g * kGroups + h) * kHeadDim + d] = o * inv[h];
}

// ------------------------------------------------------------------------------------------------
// prefill: CTA = (block of 16 queries, KV head); 8 warps; K/V tiles of 32 keys in shared memory
// ------------------------------------------------------------------------------------------------
constexpr int kPQ = 16;                 // queries per CTA
constexpr int kPK = 32;                 // keys per tile
constexpr int kPairs = kPQ * kGroups;   // 96 (query, head) pairs
constexpr int kPad = kHeadDim + 1;      // padded row length (bank-conflict free column walks)

struct PrefillSmem {
  float qs[kPairs][kPad];
  float ks[kPK][kPad];
  float vs[kPK][kHeadDim];
  float es[kPairs][kPK];
  float mx[kPairs];
  float den[kPairs];
};

// Queries q0 + qi (local rows of q and ctx) sit at positions qoff + q0 + qi and see keys 0 .. that position
// (qoff > 0: a prefill chunk after qoff cached tokens; kc / vc then hold qoff + S rows).
__global__ void __launch_bounds__(256) prefill_attn_kernel(const float* __restrict__ q, const float* __restrict__ kc,
                                                           const float* __restrict__ vc, int S, int qoff,
                                                           float* __restrict__ ctx, const int* only_if) {
  griddep_wait();  // inputs come from the preceding kernel (programmatic dependent launch)
  griddep_launch();
  if (only_if != nullptr && *reinterpret_cast<const volatile int*>(only_if) == 0) return;
  extern __shared__ float4 smem4[];
  PrefillSmem& sm = *reinterpret_cast<PrefillSmem*>(smem4);
  const int q0 = blockIdx.x * kPQ, g = blockIdx.y;
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int nq = min(kPQ, S - q0);

  // load Q pairs: pair p = qi * 6 + h
  for (int i = tid; i < kPairs * kHeadDim; i += 256) {
    const int p = i / kHeadDim, d = i % kHeadDim;
    const int qi = p / kGroups, h = p % kGroups;
    sm.qs[p][d] = qi < nq ? q[(size_t)(q0 + qi) * kHidden + (g * kGroups + h) * kHeadDim + d] : 0.0f;
  }
  if (tid < kPairs) {
    sm.mx[tid] = -1.0e30f;
    sm.den[tid] = 0.0f;
  }
  const int kend = qoff + q0 + nq;  // keys [0, kend)
  const int ntiles = (kend + kPK - 1) / kPK;

  // pass 1: causal max of the scaled scores
  for (int tile = 0; tile < ntiles; ++tile) {
    const int k0 = tile * kPK;
    __syncthreads();
    for (int i = tid; i < kPK * kHeadDim; i += 256) {
      const int jj = i / kHeadDim, d = i % kHeadDim;
      sm.ks[jj][d] = (k0 + jj) < kend ? kc[(size_t)(k0 + jj) * kKvWidth + g * kHeadDim + d] : 0.0f;
    }
    __syncthreads();
    for (int p = warp; p < kPairs; p += 8) {
      const int qi = p / kGroups;
      const int key = k0 + lane;
      float s = 0.0f;
      for (int d = 0; d < kHeadDim; ++d) s = __fadd_rn(s, __fmul_rn(sm.qs[p][d], sm.ks[lane][d]));
      const float ss = __fmul_rn(s, kAttentionScaling);
      float m = (qi < nq && key <= qoff + q0 + qi) ? ss : -INFINITY;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      if (lane == 0) sm.mx[p] = m > sm.mx[p] ? m : sm.mx[p];
    }
  }
  __syncthreads();

  // pass 2: e = approx_exp(score * scale - max), denominator and context
  const int d = tid % kHeadDim;   // output dim owned by this thread
  const int ph = tid / kHeadDim;  // pairs ph, ph+2, ph+4, ...
  float acc[kPairs / 2];
#pragma unroll
  for (int i = 0; i < kPairs / 2; ++i) acc[i] = 0.0f;
  for (int tile = 0; tile < ntiles; ++tile) {
    const int k0 = tile * kPK;
    __syncthreads();
    for (int i = tid; i < kPK * kHeadDim; i += 256) {
      const int jj = i / kHeadDim, dd = i % kHeadDim;
      const bool ok = (k0 + jj) < kend;
      sm.ks[jj][dd] = ok ? kc[(size_t)(k0 + jj) * kKvWidth + g * kHeadDim + dd] : 0.0f;
      sm.vs[jj][dd] = ok ? vc[(size_t)(k0 + jj) * kKvWidth + g * kHeadDim + dd] : 0.0f;
    }
    __syncthreads();
    for (int p = warp; p < kPairs; p += 8) {
      const int qi = p / kGroups;
      const int key = k0 + lane;
      float s = 0.0f;
      for (int dd = 0; dd < kHeadDim; ++dd) s = __fadd_rn(s, __fmul_rn(sm.qs[p][dd], sm.ks[lane][dd]));
      const float ss = __fmul_rn(s, kAttentionScaling);
      const bool valid = qi < nq && key <= qoff + q0 + qi;
      const float e = valid ? approx_exp(__fsub_rn(ss, sm.mx[p])) : 0.0f;
      sm.es[p][lane] = e;
      float l = e;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
      if (lane == 0) sm.den[p] += l;
    }
    __syncthreads();
#pragma unroll 4
    for (int jj = 0; jj < kPK; ++jj) {
      const float vv = sm.vs[jj][d];
#pragma unroll
      for (int i = 0; i < kPairs / 2; ++i) acc[i] = fmaf(sm.es[ph + 2 * i][jj], vv, acc[i]);
    }
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < kPairs / 2; ++i) {
    const int p = ph + 2 * i;
    const int qi = p / kGroups, h = p % kGroups;
    if (qi < nq) {
      const float den = sm.den[p];
      const float inv = den > 0.0f ? 1.0f / den : 0.0f;
      ctx[(size_t)(q0 + qi) * kHidden + (g * kGroups + h) * kHeadDim + d] = acc[i] * inv;
    }
  }
}

}  // namespace

size_t attn_partial_floats(int nt, int max_len) {
  const int max_chunks = (max_len + kChunk - 1) / kChunk;
  return (size_t)nt * kKvHeads * max_chunks * kGroups * kPartStride;
}

namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn_d() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &qr) == cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// fp32 rows of 256 floats (1 KB apart), `rows` of them; K boxes 32 floats x 64 rows with the 128-byte
// swizzle, V boxes 128 floats x 64 rows dense. Rows past the extent read as zeros. Encoded maps are cached.
bool kv_map(CUtensorMap* out, const float* base, uint64_t rows, bool k_layout) {
  struct Entry {
    const float* base;
    uint64_t rows;
    bool k;
    CUtensorMap map;
  };
  static std::mutex mu;
  static std::vector<Entry> cache;
  std::lock_guard<std::mutex> lock(mu);
  for (const Entry& e : cache)
    if (e.base == base && e.rows == rows && e.k == k_layout) {
      *out = e.map;
      return true;
    }
  auto fn = encode_fn_d();
  if (!fn || rows == 0 || rows > 0xFFFFFFFFull || (reinterpret_cast<uintptr_t>(base) & 15)) return false;
  cuuint64_t dims[2] = {(cuuint64_t)kKvWidth, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)kKvWidth * 4};
  cuuint32_t box[2] = {k_layout ? 32u : (cuuint32_t)kHeadDim, (cuuint32_t)kChunk};
  cuuint32_t es[2] = {1, 1};
  Entry e{base, rows, k_layout, {}};
  if (fn(&e.map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, es,
         CU_TENSOR_MAP_INTERLEAVE_NONE, k_layout ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  if (cache.size() >= 64) cache.erase(cache.begin());
  cache.push_back(e);
  *out = e.map;
  return true;
}

}  // namespace

cudaError_t launch_decode_attention(const float* q, KvView kv, DecodeTokens tok, int max_len, float* ctx,
                                    float* scratch, unsigned* counters, cudaStream_t s, bool pdl,
                                    const void* prefetch, size_t prefetch_bytes, int max_ctas) {
  const int max_chunks = (max_len + kChunk - 1) / kChunk;
  const int sms = device_sm_count();
  {
    cudaError_t e = ensure_smem_attr((const void*)decode_attn_kernel, kDecodeAttnSmem);
    if (e == cudaSuccess)
      e = ensure_smem_attr((const void*)decode_attn_merge_kernel,
                           (4 * kGroups * (kMaxSeq / kChunk) + kGroups) * sizeof(float));
    if (e != cudaSuccess) return e;
  }
  (void)counters;  // kept for the interface; the merge runs as its own kernel
  if (tok.nt <= 0 || max_chunks <= 0 || max_chunks > kMaxSeq / kChunk || (reinterpret_cast<uintptr_t>(q) & 15))
    return cudaErrorInvalidValue;
  CUtensorMap kmap, vmap;
  if (kv.page_table == nullptr) {
    if (!kv_map(&kmap, kv.k, (uint64_t)max_len, true) || !kv_map(&vmap, kv.v, (uint64_t)max_len, false))
      return cudaErrorInvalidValue;
  } else {
    const uint64_t rows = (uint64_t)kv.pool_pages * kLayers * 2 * kPage;
    if (kv.pool_pages <= 0 || !kv_map(&kmap, kv.k, rows, true) || !kv_map(&vmap, kv.k, rows, false))
      return cudaErrorInvalidValue;
  }
  // launches of at most kMaxTokens tokens each; every launch spreads its work items over up to one CTA per SM
  for (int t0 = 0; t0 < tok.nt; t0 += kMaxTokens) {
    DecodeTokens sub = tok;
    sub.pos += t0;
    sub.seq += t0;
    sub.nt = std::min(kMaxTokens, tok.nt - t0);
    const long long items = (long long)sub.nt * kKvHeads * max_chunks;
    int grid = (int)std::min<long long>(items, sms);
    if (max_ctas > 0) grid = std::min(grid, max_ctas);
    float* part = scratch + (size_t)t0 * kKvHeads * max_chunks * kGroups * kPartStride;
    cudaError_t e = launch_k(decode_attn_kernel, dim3(grid), dim3(kAttnThreads), kDecodeAttnSmem, s, pdl && t0 == 0,
                             kmap, vmap, q + (size_t)t0 * kHidden, kv, sub, max_chunks, ctx + (size_t)t0 * kHidden,
                             part, static_cast<const uint8_t*>(prefetch), prefetch_bytes);
    if (e != cudaSuccess) return e;
    if (max_chunks > 1) {
      e = launch_k(decode_attn_merge_kernel, dim3(sub.nt, kKvHeads), dim3(kMergeThreads),
                   (size_t)(4 * kGroups * max_chunks + kGroups) * sizeof(float), s, true, sub, max_chunks,
                   ctx + (size_t)t0 * kHidden, static_cast<const float*>(part));
      if (e != cudaSuccess) return e;
    }
  }
  return cudaSuccess;
}

unsigned decode_attn_kernel_error(bool reset) {
  unsigned v = 0;
  if (cudaMemcpyFromSymbol(&v, g_kernel_error, sizeof(v)) != cudaSuccess) return 0xFFFFFFFFu;
  if (reset && v) {
    const unsigned z = 0;
    cudaMemcpyToSymbol(g_kernel_error, &z, sizeof(z));
  }
  return v;
}

cudaError_t launch_prefill_attention(const float* q, const float* k_cache, const float* v_cache, int S, float* ctx,
                                     cudaStream_t s, int qoff) {
  const size_t smem = sizeof(PrefillSmem);
  if (cudaError_t e = ensure_smem_attr((const void*)prefill_attn_kernel, smem)) return e;
  return launch_k(prefill_attn_kernel, dim3((S + kPQ - 1) / kPQ, kKvHeads), dim3(256), smem, s, true, q, k_cache,
                  v_cache, S, qoff, ctx, static_cast<const int*>(nullptr));
}

cudaError_t launch_prefill_attention_gated(const float* q, const float* k_cache, const float* v_cache, int S,
                                           float* ctx, const int* only_if, cudaStream_t s, int qoff) {
  const size_t smem = sizeof(PrefillSmem);
  if (cudaError_t e = ensure_smem_attr((const void*)prefill_attn_kernel, smem)) return e;
  return launch_k(prefill_attn_kernel, dim3((S + kPQ - 1) / kPQ, kKvHeads), dim3(256), smem, s, true, q, k_cache,
                  v_cache, S, qoff, ctx, only_if);
}

}  // namespace qb
