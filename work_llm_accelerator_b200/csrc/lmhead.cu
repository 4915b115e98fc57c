// Final RMSNorm + tied fp16 LM head + greedy argmax on the tensor cores, for 1..128 tokens.
//
// Caller-side model head of the reference flow (verification/real_host_top_backend.py:138-146), defined in
// oracle/qwen_oracle.c as oracle_lm_head_argmax: y = decode-style RMSNorm(x) (double accumulation), logit[v]
// = sum_d f16(E[v][d]) * y[d] in fp32, next token = argmax (lowest index on ties).
//
// Here y is written exactly enough as two fp16 planes, y = hi + lo (hi = f16(y), lo = f16(y - hi), 22
// significant bits), and the fp16 table is the A operand of tcgen05.mma kind::f16 (M = 128 vocabulary rows,
// N = 2 x tokens, K = 16 per instruction, fp32 accumulation; fp16 x fp16 products are exact in fp32):
// logit = acc(hi) + acc(lo). The 467 MB table is streamed once per call whatever the token count: a
// persistent CTA per SM walks vocabulary tiles with a TMA ring, two TMEM accumulators let the epilogue of
// one tile overlap the MMAs of the next, and each tile's per-token argmax is merged into a 64-bit
// (orderable value, inverted index) word with atomicMax, so the result does not depend on tile order.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "lmhead.h"
#include "umma_sm100.cuh"

namespace qb {
namespace {

using namespace umma;

constexpr int kLmTiles = kVocab / kTileM;    // 1187
static_assert(kLmTiles * kTileM == kVocab, "vocabulary is a whole number of 128-row tiles");
constexpr int kLmKB = kHidden * 2 / kKBlock;  // 24 blocks of 64 fp16
constexpr int kLmThreads = 192;
constexpr int kLmEpi = 128;
constexpr int kLmBar = 1;

template <int NP>
struct LmCfg {
  static constexpr int kN = 2 * NP;                       // B rows: hi plane tokens, then lo plane
  static constexpr bool kResident = NP <= 16;             // whole B (24 blocks) kept in shared memory
  static constexpr int kBBlock = kN * kKBlock;            // bytes of one B block
  static constexpr int kStage = kUnitBytes + (kResident ? 0 : kBBlock);
  static constexpr int kResBytes = kResident ? kLmKB * kBBlock : 0;
  static constexpr int kStages = (196 * 1024 - kResBytes) / kStage > 8 ? 8 : (196 * 1024 - kResBytes) / kStage;
  static constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(kN >> 3) << 17) | ((uint32_t)(kTileM >> 4) << 24);
  static_assert(kN % 16 == 0 && kN <= 256, "MMA N");
  static_assert(2 * kN <= 512, "two accumulators in TMEM");
};

struct LmCtrl {
  uint64_t full[8], empty[8], acc_full[2], acc_empty[2], b_full;
  uint32_t tmem_base;
  int last;
  float wv[4][256];   // per warp: best value per token (epilogue argmax merge)
  int wi[4][256];
};

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

template <uint32_t IDESC>
__device__ __forceinline__ void mma_f16(uint32_t d, uint64_t a, uint64_t b, uint32_t acc) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\ntcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(d),
      "l"(a), "l"(b), "r"(IDESC), "r"(acc)
      : "memory");
}

// order-preserving 32-bit key of a float (larger float -> larger key)
__device__ __forceinline__ uint32_t orderable(float v) {
  const uint32_t b = __float_as_uint(v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

template <int NP>
__global__ void __launch_bounds__(kLmThreads, 1)
    lm_head_kernel(const __grid_constant__ CUtensorMap emap, const __grid_constant__ CUtensorMap pmap, LmArgs a) {
  using C = LmCfg<NP>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = align_smem_1024(smem_raw);
  uint8_t* bres = base;                              // resident B blocks (small token counts)
  uint8_t* ring = base + C::kResBytes;               // stages
  LmCtrl& cs = *reinterpret_cast<LmCtrl*>(ring + (size_t)C::kStages * C::kStage);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&cs.full[s], 1);
      mbar_init(&cs.empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&cs.acc_full[b], 1);
      mbar_init(&cs.acc_empty[b], kLmEpi);
    }
    mbar_init(&cs.b_full, 1);
    mbar_fence_init();
  }
  if (warp == 1) tmem_alloc(&cs.tmem_base, 512);
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = cs.tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(&emap) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(&pmap) : "memory");
      bool ok = true;
      if constexpr (C::kResident) {
        mbar_arrive_expect_tx(&cs.b_full, C::kResBytes);
        for (int kb = 0; kb < kLmKB; ++kb) tma_load_2d(bres + kb * C::kBBlock, &pmap, kb * 64, 0, &cs.b_full);
      }
      int s = 0;
      unsigned ph = 0;
      for (int tile = blockIdx.x; tile < kLmTiles && ok; tile += gridDim.x) {
        for (int kb = 0; kb < kLmKB && ok; ++kb) {
          if (!(ok = mbar_wait(&cs.empty[s], ph ^ 1))) break;
          mbar_arrive_expect_tx(&cs.full[s], C::kStage);
          uint8_t* st = ring + (size_t)s * C::kStage;
          tma_load_2d(st, &emap, kb * 64, tile * kTileM, &cs.full[s]);
          if constexpr (!C::kResident) tma_load_2d(st + kUnitBytes, &pmap, kb * 64, 0, &cs.full[s]);
          if (++s == C::kStages) {
            s = 0;
            ph ^= 1;
          }
        }
      }
      for (int i = 0; i < C::kStages && ok; ++i) {  // no copy in flight at exit
        ok = mbar_wait(&cs.empty[s], ph ^ 1);
        if (++s == C::kStages) {
          s = 0;
          ph ^= 1;
        }
      }
      if constexpr (C::kResident) mbar_wait(&cs.b_full, 0);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      bool ok = true;
      if constexpr (C::kResident) ok = mbar_wait(&cs.b_full, 0);
      int s = 0;
      unsigned ph = 0, item = 0;
      for (int tile = blockIdx.x; tile < kLmTiles; tile += gridDim.x, ++item) {
        const unsigned b = item & 1;
        ok = ok && mbar_wait(&cs.acc_empty[b], ((item >> 1) & 1) ^ 1);
        fence_after();
        const uint32_t d = tmem + b * C::kN;
        for (int kb = 0; kb < kLmKB; ++kb) {
          ok = ok && mbar_wait(&cs.full[s], ph);
          fence_after();
          if (ok) {
            const uint32_t sa = smem_u32(ring + (size_t)s * C::kStage);
            const uint32_t sb = C::kResident ? smem_u32(bres + kb * C::kBBlock) : sa + kUnitBytes;
            const uint64_t ad = sw128_desc(sa), bd = sw128_desc(sb);
#pragma unroll
            for (int j = 0; j < kKBlock / 32; ++j)
              mma_f16<C::kIdesc>(d, ad + 2 * j, bd + 2 * j, (kb > 0 || j > 0) ? 1u : 0u);
          }
          mma_commit(&cs.empty[s]);
          if (++s == C::kStages) {
            s = 0;
            ph ^= 1;
          }
        }
        mma_commit(&cs.acc_full[b]);
      }
    }
  } else {
    // ---- epilogue: thread = vocabulary row of the tile; per token: logit, argmax over the tile
    const int q = warp & 3, r = q * 32 + lane, ew = warp - 2;
    unsigned item = 0;
    for (int tile = blockIdx.x; tile < kLmTiles; tile += gridDim.x, ++item) {
      const unsigned b = item & 1;
      const bool ok = mbar_wait(&cs.acc_full[b], (item >> 1) & 1);
      __syncwarp();
      fence_after();
      const int row = tile * kTileM + r;
      const uint32_t lb = tmem + b * C::kN + ((uint32_t)(q * 32) << 16);
      for (int t0 = 0; t0 < NP; t0 += 16) {
        int hi[16], lo[16];
        if (ok) {
          tmem_ld16(lb + t0, hi);
          tmem_ld16(lb + NP + t0, lo);
        } else {
#pragma unroll
          for (int c = 0; c < 16; ++c) hi[c] = lo[c] = 0;
        }
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const int t = t0 + c;
          if (NP >= 16 || t < NP) {
            const float lg = __fadd_rn(__int_as_float(hi[c]), __int_as_float(lo[c]));
            if (t < a.n && a.logits != nullptr) a.logits[(size_t)t * kVocab + row] = lg;
            // argmax within the warp: larger value, then smaller row
            float bv = lg;
            int bi = row;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
              const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
              const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
              if (ov > bv || (ov == bv && oi < bi)) {
                bv = ov;
                bi = oi;
              }
            }
            if (lane == 0) {
              cs.wv[ew][t] = bv;
              cs.wi[ew][t] = bi;
            }
          }
        }
      }
      fence_before();
      mbar_arrive(&cs.acc_empty[b]);
      named_sync(kLmBar, kLmEpi);
      // merge the four warps per token and publish one 64-bit candidate per token
      for (int t = threadIdx.x - 64; t < a.n; t += kLmEpi) {
        float bv = cs.wv[0][t];
        int bi = cs.wi[0][t];
        for (int w = 1; w < 4; ++w) {
          const float ov = cs.wv[w][t];
          const int oi = cs.wi[w][t];
          if (ov > bv || (ov == bv && oi < bi)) {
            bv = ov;
            bi = oi;
          }
        }
        const unsigned long long key = ((unsigned long long)orderable(bv) << 32) | (0xFFFFFFFFu - (unsigned)bi);
        atomicMax(&a.packed[t], key);
      }
      named_sync(kLmBar, kLmEpi);
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    tmem_dealloc(tmem, 512);
  }
  if (threadIdx.x == 0) {
    __threadfence();
    cs.last = atomicAdd(a.counter, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (cs.last) {  // every CTA's candidates are in: unpack the winners and clear for the next call
    __threadfence();
    for (int t = threadIdx.x; t < a.n; t += blockDim.x) {
      const unsigned long long key = atomicExch(&a.packed[t], 0ull);
      a.next[t] = (int)(0xFFFFFFFFu - (unsigned)(key & 0xFFFFFFFFull));
    }
    if (threadIdx.x == 0) *a.counter = 0u;
  }
}

// Final RMSNorm (decode form, identical element order to the decode kernels) and the two fp16 planes;
// token rows n.. NP-1 are zero.
__global__ void __launch_bounds__(128) lm_prep_kernel(const float* __restrict__ x, const float* __restrict__ w, int n,
                                                      int np, __half* __restrict__ planes) {
  __shared__ double red[4];
  const int t = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  __half* hi = planes + (size_t)t * kHidden;
  __half* lo = planes + ((size_t)np + t) * kHidden;
  if (t >= n) {
    for (int k = tid; k < kHidden; k += 128) hi[k] = lo[k] = __float2half_rn(0.0f);
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
  const double inv = 1.0 / sqrt((red[0] + red[1] + red[2] + red[3]) / (double)kHidden + (double)kEps);
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const float4 wv = *reinterpret_cast<const float4*>(w + 512 * j + 4 * tid);
    const float wf[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float y = (float)((double)v[j][e] * inv * (double)wf[e]);
      const __half h = __float2half_rn(y);
      const int k = 512 * j + 4 * tid + e;
      hi[k] = h;
      lo[k] = __float2half_rn(y - __half2float(h));
    }
  }
}

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

bool make_map_u16(CUtensorMap* m, const void* base, uint64_t rows, uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)kHidden, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)kHidden * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t es[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int NP>
cudaError_t run_lm(const uint16_t* embed, const LmScratch& sc, LmArgs a, int ctas, cudaStream_t s) {
  using C = LmCfg<NP>;
  CUtensorMap emap, pmap;
  if (!make_map_u16(&emap, embed, kVocab, kTileM) || !make_map_u16(&pmap, sc.planes, 2 * NP, 2 * NP))
    return cudaErrorInvalidValue;
  auto kern = lm_head_kernel<NP>;
  const size_t smem = 1024 + (size_t)C::kResBytes + (size_t)C::kStages * C::kStage + sizeof(LmCtrl);
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
  kern<<<ctas, kLmThreads, smem, s>>>(emap, pmap, a);
  return cudaGetLastError();
}

}  // namespace

size_t lm_scratch_bytes() { return (size_t)2 * 128 * kHidden * 2 + 128 * 8 + 16; }

cudaError_t lm_head_tc(const uint16_t* embed, const float* norm_w, const float* x, int n, float* logits, int* next,
                       const LmScratch& sc, cudaStream_t s) {
  if (n < 1 || n > 128) return cudaErrorInvalidValue;
  const int np = n <= 8 ? 8 : n <= 64 ? 64 : 128;
  lm_prep_kernel<<<np, 128, 0, s>>>(x, norm_w, n, np, sc.planes);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  int sms = 148, dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  LmArgs a{};
  a.n = n;
  a.logits = logits;
  a.next = next;
  a.packed = sc.packed;
  a.counter = sc.counter;
  const int ctas = sms < kLmTiles ? sms : kLmTiles;
  if (np == 8) return run_lm<8>(embed, sc, a, ctas, s);
  if (np == 64) return run_lm<64>(embed, sc, a, ctas, s);
  return run_lm<128>(embed, sc, a, ctas, s);
}

unsigned lm_head_kernel_error(bool reset) {
  unsigned v = 0;
  if (cudaMemcpyFromSymbol(&v, g_kernel_error, sizeof(v)) != cudaSuccess) return 0xFFFFFFFFu;
  if (reset && v) {
    const unsigned z = 0;
    cudaMemcpyToSymbol(g_kernel_error, &z, sizeof(z));
  }
  return v;
}

}  // namespace qb
