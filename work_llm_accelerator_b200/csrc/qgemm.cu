// Integer tensor-core projections (tcgen05.mma kind::i8) for the W8 track.
//
// Reference computation: y[o] = bias[o] + sum_i x[i] * (code(o,i) * scale[o]) in fp32
// (hls/decode_only/qwen_decode_attention_kernel.cpp:62-98, hls/decode_only/qwen_decode_mlp_kernel.cpp:44-77).
// Here each token's fp32 activation row x is written exactly as an integer multiple of a per-token step,
// x ~= s_x * X with |X| <= 8355711 (24-bit, relative error 2^-24 of max|x|), and X is split into three
// balanced int8 digits X = d0 + 256 d1 + 65536 d2. The tensor cores compute the three integer dot products
// sum_i code(o,i) * d_k(i) with int32 accumulators, which are exact (|acc| <= 8960 * 128 * 128 < 2^31), so
// y = s_w[o] * s_x * (acc0 + 256 acc1 + 65536 acc2) differs from the reference by the 24-bit quantisation
// of x only (relative ~1e-7, the size of fp32 summation noise).
//
// One CTA computes a 128-row tile of the weight matrix (TMEM lanes) against N = 16 activation-digit rows
// (digit d of token t in row 4d + t; up to 4 tokens) over a contiguous range of 128-byte K blocks:
//   warp 0      TMA producer: 128x128-byte weight tiles, 128-byte swizzle, into a ring of stages
//   warp 1      allocates TMEM (32 columns); one lane issues 4 MMAs (K = 32 bytes each) per K block
//   warps 2-5   build the digit operand in shared memory (RMSNorm, per-token step, digits), fused here
//               so decode needs no extra kernel; then read the accumulator from TMEM and run the epilogue
// Small matrices split K across CTAs: partial accumulators are added with integer atomics (exact and
// order-independent) and the last CTA of a tile runs the epilogue.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include <mutex>

#include "qwen_kernels.cuh"
#include "qgemm.h"
#include "umma_sm100.cuh"

namespace qb {
namespace {

using umma::kDigitRange;
using umma::kKBlock;
using umma::kTileM;
using umma::kTileN;
using umma::fence_after;
using umma::fence_before;
using umma::mma_commit;
using umma::mma_i8;
using umma::sw128_desc;
using umma::tmem_ld16;

constexpr int kStages = 4;
constexpr int kThreads = 192;    // 6 warps
constexpr int kEpiThreads = 128; // warps 2..5
constexpr int kBarEpi = 1;       // named barrier among the epilogue warps
constexpr int kTmemCols = 32;

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------------------------------------------
// kernel
// ---------------------------------------------------------------------------------------------------
struct Smem {
  uint8_t a[kStages][kTileM * kKBlock];  // 16 KB per stage, 1024-byte aligned (first member)
  uint64_t full[kStages], empty[kStages];
  uint64_t b_ready, acc_ready;
  uint32_t tmem_base;
  int last;
  float sx[4];
  double red[kEpiThreads / 32][4];
  float y[kTileM][4];
};

enum XMode { kQPlain = 0, kQNorm = 1, kQEmbedNorm = 2 };

struct QArgs {
  int K;            // input length (elements = bytes of a weight row)
  int nkb;          // 128-byte K blocks in a row
  int split;        // K splits (CTAs per tile)
  int nt;           // tokens (1..4)
  int mtiles;
  int box_rows;     // rows per TMA box (128, or 64 for the gate|up pairing)
  int second_row0;  // gate|up: first row of the second box (8960); else 0
  const float* x;   // [nt][K] activations (plain / norm modes)
  const uint16_t* embed;
  const int* tokens;
  const float* norm_w;
  int* acc_g;       // [rows][16] split-K accumulators (zero between uses)
  unsigned* cnt;    // [mtiles] split-K arrival counters (zero between uses)
};

__device__ __forceinline__ float load_x(const QArgs& a, int mode, int t, int k) {
  if (mode == kQEmbedNorm) return __half2float(reinterpret_cast<const __half*>(a.embed)[(size_t)a.tokens[t] * kHidden + k]);
  return a.x[(size_t)t * a.K + k];
}

// Digit operand for K blocks [kb0, kb1) in the 128-byte-swizzled K-major layout the MMA reads:
// row n (0..15), byte k of block j lives at j*2048 + (n/8)*1024 + (n%8)*128 + ((k/16) ^ (n%8))*16 + k%16.
template <int MODE>
__device__ void build_digits(const QArgs& a, Smem& sm, uint8_t* bsm, int kb0, int kb1) {
  const int tid = threadIdx.x - 64;  // 0..127
  const int warp = tid / 32, lane = tid % 32;
  // per-token statistics over the whole row
  for (int t = 0; t < 4; ++t) {
    if (t >= a.nt) break;
    double inv = 1.0;
    if (MODE != kQPlain) {
      // thread tid sums elements 512 j + 4 tid + e (j < K / 512, e < 4) in that order: the same partial
      // sums as the persistent decode kernel, so both paths produce bit-identical results
      double ss = 0.0;
      for (int j = 0; j < a.K / 512; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const double v = load_x(a, MODE, t, 512 * j + 4 * tid + e);
          ss += v * v;
        }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if (lane == 0) sm.red[warp][t] = ss;
      named_sync(kBarEpi, kEpiThreads);
      const double tot = sm.red[0][t] + sm.red[1][t] + sm.red[2][t] + sm.red[3][t];
      inv = 1.0 / sqrt(tot / (double)kHidden + (double)kEps);
      named_sync(kBarEpi, kEpiThreads);
    }
    float m = 0.0f;
    for (int k = tid; k < a.K; k += kEpiThreads) {
      float v = load_x(a, MODE, t, k);
      if (MODE != kQPlain) v = (float)((double)v * inv * (double)a.norm_w[k]);
      m = fmaxf(m, fabsf(v));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) sm.red[warp][t] = (double)m;
    named_sync(kBarEpi, kEpiThreads);
    const float mx = (float)fmax(fmax(sm.red[0][t], sm.red[1][t]), fmax(sm.red[2][t], sm.red[3][t]));
    const float step = mx > 0.0f ? mx / kDigitRange : 1.0f;
    if (tid == 0) sm.sx[t] = step;
    named_sync(kBarEpi, kEpiThreads);
    // digits of this CTA's K range: one 16-byte chunk per thread iteration
    const double rstep = umma::digit_recip(step);
    const int nchunks = (kb1 - kb0) * 8;
    for (int c = tid; c < nchunks; c += kEpiThreads) {
      const int j = c >> 3, c16 = c & 7;
      const int k0 = (kb0 + j) * kKBlock + c16 * 16;
      uint32_t w0[4], w1[4], w2[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) w0[q] = w1[q] = w2[q] = 0u;
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const int k = k0 + e;
        float v = 0.0f;
        if (k < a.K) {
          v = load_x(a, MODE, t, k);
          if (MODE != kQPlain) v = (float)((double)v * inv * (double)a.norm_w[k]);
        }
        const int X = umma::digit_quotient(v, rstep);
        int d0, d1, d2;
        umma::split_digits(X, d0, d1, d2);
        w0[e >> 2] |= (uint32_t)(d0 & 255) << (8 * (e & 3));
        w1[e >> 2] |= (uint32_t)(d1 & 255) << (8 * (e & 3));
        w2[e >> 2] |= (uint32_t)(d2 & 255) << (8 * (e & 3));
      }
      const uint32_t* ws[3] = {w0, w1, w2};
#pragma unroll
      for (int d = 0; d < 3; ++d) {
        const int n = 4 * d + t;
        uint4* dst = reinterpret_cast<uint4*>(bsm + (size_t)j * 2048 + (n >> 3) * 1024 + (n & 7) * 128 +
                                              ((c16 ^ (n & 7)) * 16));
        *dst = make_uint4(ws[d][0], ws[d][1], ws[d][2], ws[d][3]);
      }
    }
  }
  // zero rows: tokens beyond nt and rows 12..15
  const int nzc = (kb1 - kb0) * kTileN * 8;
  for (int c = tid; c < nzc; c += kEpiThreads) {
    const int j = c / (kTileN * 8), rem = c % (kTileN * 8);
    const int n = rem >> 3, c16 = rem & 7;
    const int t = n & 3, d = n >> 2;
    if (d < 3 && t < a.nt) continue;
    uint4* dst = reinterpret_cast<uint4*>(bsm + (size_t)j * 2048 + (n >> 3) * 1024 + (n & 7) * 128 + ((c16 ^ (n & 7)) * 16));
    *dst = make_uint4(0u, 0u, 0u, 0u);
  }
}

template <int MODE, class Epi>
__global__ void __launch_bounds__(kThreads, 1) qgemm_kernel(const __grid_constant__ CUtensorMap tmap, QArgs a, Epi epi) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 128-byte-swizzled tiles need 1024-byte-aligned shared addresses: align both regions explicitly
  uint8_t* base = align_smem_1024(smem_raw);
  Smem& sm = *reinterpret_cast<Smem*>(base);
  uint8_t* bsm = base + sizeof(Smem);
  bsm = align_smem_1024(bsm);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int mtile = blockIdx.x / a.split, ks = blockIdx.x % a.split;
  const int kper = (a.nkb + a.split - 1) / a.split;
  const int kb0 = ks * kper, kb1 = min(a.nkb, kb0 + kper);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    mbar_init(&sm.b_ready, kEpiThreads);
    mbar_init(&sm.acc_ready, 1);
    mbar_fence_init();
  }
  if (warp == 1) {
    umma::tmem_alloc(&sm.tmem_base, kTmemCols);
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == 0) {
    // ---- TMA producer (weights do not depend on the preceding kernel)
    if (lane == 0 && kb1 > kb0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap) : "memory");
      int s = 0;
      unsigned ph = 0;
      bool ok = true;
      const int row0 = epi.tile_row0(mtile);
      for (int kb = kb0; kb < kb1 && ok; ++kb) {
        if (!(ok = mbar_wait(&sm.empty[s], ph ^ 1))) break;
        mbar_arrive_expect_tx(&sm.full[s], kTileM * kKBlock);
        if (a.box_rows == kTileM) {
          tma_load_2d(sm.a[s], &tmap, kb * kKBlock, row0, &sm.full[s]);
        } else {
          tma_load_2d(sm.a[s], &tmap, kb * kKBlock, row0, &sm.full[s]);
          tma_load_2d(sm.a[s] + a.box_rows * kKBlock, &tmap, kb * kKBlock, row0 + a.second_row0, &sm.full[s]);
        }
        if (++s == kStages) {
          s = 0;
          ph ^= 1;
        }
      }
      // all issued stages consumed by the MMAs before leaving (no copy in flight at exit)
      for (int i = 0; i < kStages && ok; ++i) {
        ok = mbar_wait(&sm.empty[s], ph ^ 1);
        if (++s == kStages) {
          s = 0;
          ph ^= 1;
        }
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer
    if (lane == 0) {
      bool ok = mbar_wait(&sm.b_ready, 0);
      fence_after();
      int s = 0;
      unsigned ph = 0;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (ok) ok = mbar_wait(&sm.full[s], ph);
        fence_after();
        if (ok) {
          const uint32_t abase = smem_u32(sm.a[s]);
          const uint32_t bbase = smem_u32(bsm + (size_t)(kb - kb0) * 2048);
#pragma unroll
          for (int j = 0; j < kKBlock / 32; ++j)
            mma_i8(tmem, sw128_desc(abase + 32 * j), sw128_desc(bbase + 32 * j), (kb > kb0 || j > 0) ? 1u : 0u);
        }
        mma_commit(&sm.empty[s]);  // stage free once these MMAs have read it
        if (++s == kStages) {
          s = 0;
          ph ^= 1;
        }
      }
      mma_commit(&sm.acc_ready);
    }
  } else {
    // ---- activation digits, then the epilogue
    griddep_wait();
    build_digits<MODE>(a, sm, bsm, kb0, kb1);
    umma::fence_async_smem();  // generic writes -> tensor-core reads
    mbar_arrive(&sm.b_ready);
    if (threadIdx.x == 64) griddep_launch();
    const bool ok = mbar_wait(&sm.acc_ready, 0);
    fence_after();
    const int quarter = warp & 3;          // TMEM lanes this warp may read
    const int r = quarter * 32 + lane;     // tile row
    int v[16];
    if (ok && kb1 > kb0) {
      tmem_ld16(tmem + ((uint32_t)(quarter * 32) << 16), v);
    } else {
#pragma unroll
      for (int c = 0; c < 16; ++c) v[c] = 0;
    }
    bool run = true;
    if (a.split > 1) {
      int* g = a.acc_g + ((size_t)mtile * kTileM + r) * 16;
#pragma unroll
      for (int c = 0; c < 12; ++c)
        if ((c & 3) < a.nt) atomicAdd(&g[c], v[c]);
      __threadfence();
      named_sync(kBarEpi, kEpiThreads);
      if (threadIdx.x == 64) sm.last = atomicAdd(&a.cnt[mtile], 1u) == (unsigned)(a.split - 1);
      named_sync(kBarEpi, kEpiThreads);
      run = sm.last != 0;
      if (run) {
        __threadfence();
#pragma unroll
        for (int c = 0; c < 12; ++c) {
          if ((c & 3) < a.nt) {
            v[c] = __ldcg(&g[c]);
            g[c] = 0;
          }
        }
        if (threadIdx.x == 64) a.cnt[mtile] = 0u;
      }
    }
    if (run) {
      if constexpr (Epi::kRaw) {
        epi.raw(mtile, r, v, sm.sx, a.nt);
      } else {
        float yv[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const long long tot = (long long)v[t] + 256ll * (long long)v[4 + t] + 65536ll * (long long)v[8 + t];
          yv[t] = (float)((double)tot * (double)sm.sx[t]);
        }
        epi.finish(mtile, r, yv, a.nt, sm.y);
      }
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    umma::tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------------------------------
// epilogues: finish(tile, r, yv, nt, ystage) runs on the 128 epilogue threads (r = tile row); yv[t] is
// s_x[t] * sum(code * X) for token t, before the weight scale.
// ---------------------------------------------------------------------------------------------------
// q|k|v: tile = one head (rows h*128 .. +127), rotate-half pairs (r, r+64) exchanged through shared memory.
struct QEpiQkv {
  static constexpr bool kRaw = false;
  __device__ void raw(int, int, const int (&)[16], const float*, int) const {}
  const float* bias;
  const float* scale;
  const float* cosv;
  const float* sinv;
  float* q_out;
  KvView kv;
  DecodeTokens tok;
  __device__ int tile_row0(int tile) const { return tile * kTileM; }
  __device__ void finish(int tile, int r, const float (&yv)[4], int nt, float (*ys)[4]) const {
    const int row = tile * kTileM + r;
    const float b = bias[row], s = scale[row];
#pragma unroll
    for (int t = 0; t < 4; ++t) ys[r][t] = __fmaf_rn(s, yv[t], b);
    named_sync(kBarEpi, kEpiThreads);
    const int h = tile;
    for (int t = 0; t < nt; ++t) {
      const float mine = ys[r][t], other = ys[r ^ 64][t];
      float y = mine;
      const int pos = tok.pos[t];
      if (h < kHeads + kKvHeads) {
        const int p = r & 63;
        const float c = cosv[(size_t)pos * 64 + p], sn = sinv[(size_t)pos * 64 + p];
        y = r < 64 ? __fsub_rn(__fmul_rn(mine, c), __fmul_rn(other, sn))
                   : __fadd_rn(__fmul_rn(mine, c), __fmul_rn(other, sn));
      }
      if (h < kHeads) {
        q_out[(size_t)t * kHidden + row] = y;
      } else {
        const int which = h < kHeads + kKvHeads ? 0 : 1;
        kv_row(kv, tok.seq[t], pos, which)[row - kHidden - which * kKvWidth] = y;
      }
    }
  }
};

// o_proj: y = scale * acc
struct QEpiScale {
  static constexpr bool kRaw = false;
  __device__ void raw(int, int, const int (&)[16], const float*, int) const {}
  const float* scale;
  float* out;
  __device__ int tile_row0(int tile) const { return tile * kTileM; }
  __device__ void finish(int tile, int r, const float (&yv)[4], int nt, float (*)[4]) const {
    const int row = tile * kTileM + r;
    const float s = scale[row];
    for (int t = 0; t < nt; ++t) out[(size_t)t * kHidden + row] = s * yv[t];
  }
};

// gate|up: tile j = gate rows 64j..64j+63 (tile rows 0..63) and up rows 8960+64j.. (tile rows 64..127)
struct QEpiGateUp {
  static constexpr bool kRaw = false;
  __device__ void raw(int, int, const int (&)[16], const float*, int) const {}
  const float* scale;
  float* h;
  __device__ int tile_row0(int tile) const { return tile * 64; }
  __device__ void finish(int tile, int r, const float (&yv)[4], int nt, float (*ys)[4]) const {
    const int row = r < 64 ? tile * 64 + r : kInter + tile * 64 + (r - 64);
    const float s = scale[row];
#pragma unroll
    for (int t = 0; t < 4; ++t) ys[r][t] = s * yv[t];
    named_sync(kBarEpi, kEpiThreads);
    if (r < 64) {
      for (int t = 0; t < nt; ++t) {
        const float gv = ys[r][t], uv = ys[r + 64][t];
        const float silu = __fdiv_rn(gv, __fadd_rn(1.0f, expf(-gv)));
        h[(size_t)t * kInter + tile * 64 + r] = __fmul_rn(silu, uv);
      }
    }
  }
};

// down: out = a + scale * acc (+ bf16 rounding for the next layer)
struct QEpiDown {
  static constexpr bool kRaw = false;
  __device__ void raw(int, int, const int (&)[16], const float*, int) const {}
  const float* scale;
  const float* resid;
  float* out;
  bool round_out;
  __device__ int tile_row0(int tile) const { return tile * kTileM; }
  __device__ void finish(int tile, int r, const float (&yv)[4], int nt, float (*)[4]) const {
    const int row = tile * kTileM + r;
    const float s = scale[row];
    for (int t = 0; t < nt; ++t) {
      float y = __fadd_rn(resid[(size_t)t * kHidden + row], s * yv[t]);
      if (round_out) y = round_bf16(y);
      out[(size_t)t * kHidden + row] = y;
    }
  }
};

// raw integer accumulators and the per-token steps (tests of the integer product)
struct QEpiRaw {
  static constexpr bool kRaw = true;
  int* acc_out;
  float* step_out;
  __device__ int tile_row0(int tile) const { return tile * kTileM; }
  __device__ void raw(int tile, int r, const int (&v)[16], const float* sx, int nt) const {
    const int row = tile * kTileM + r;
#pragma unroll
    for (int c = 0; c < 12; ++c) acc_out[(size_t)row * 12 + c] = (c & 3) < nt ? v[c] : 0;
    if (tile == 0 && r < nt) step_out[r] = sx[r];
  }
  __device__ void finish(int, int, const float (&)[4], int, float (*)[4]) const {}
};

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

template <int MODE, class Epi>
cudaError_t run_qgemm(const CUtensorMap& map, const QArgs& a, const Epi& e, cudaStream_t s, bool pdl) {
  auto kern = qgemm_kernel<MODE, Epi>;
  const int kbs = (a.nkb + a.split - 1) / a.split;
  const size_t smem = sizeof(Smem) + 2048 + (size_t)kbs * 2048;
  if (cudaError_t err = ensure_smem_attr((const void*)kern, smem)) return err;
  return launch_k(kern, dim3(a.mtiles * a.split), dim3(kThreads), smem, s, pdl, map, a, e);
}

}  // namespace

bool qgemm_make_map(QgemmMap* m, const uint8_t* w, int rows, int k_bytes, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  static_assert(sizeof(QgemmMap) >= sizeof(CUtensorMap), "map storage");
  cuuint64_t dims[2] = {(cuuint64_t)k_bytes, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)k_bytes};
  cuuint32_t box[2] = {(cuuint32_t)kKBlock, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  const CUresult r = fn(reinterpret_cast<CUtensorMap*>(m->bytes), CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
                        const_cast<uint8_t*>(w), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool qgemm_make_layer_maps(QgemmLayerMaps* m, const LayerDev& L) {
  return qgemm_make_map(&m->qkv, L.qkv_w, kQkvRows, kHidden, kTileM) &&
         qgemm_make_map(&m->o, L.o_w, kHidden, kHidden, kTileM) &&
         qgemm_make_map(&m->gu, L.gu_w, 2 * kInter, kHidden, 64) &&
         qgemm_make_map(&m->down, L.down_w, kHidden, kInter, kTileM);
}

size_t qgemm_acc_ints() { return (size_t)kQkvRows * 16; }
size_t qgemm_counter_count() { return (size_t)kQkvRows / kTileM; }

static QArgs base_args(int K, int nt, int mtiles, int split, const QgemmScratch& sc) {
  QArgs a{};
  a.K = K;
  a.nkb = K / kKBlock;
  if (K % kKBlock) a.nkb += 1;
  a.split = split;
  a.nt = nt;
  a.mtiles = mtiles;
  a.box_rows = kTileM;
  a.acc_g = sc.acc;
  a.cnt = sc.cnt;
  return a;
}

cudaError_t qgemm_qkv(const QgemmLayerMaps& m, const LayerDev& L, XSource src, DecodeTokens tok, const float* rope_cos,
                      const float* rope_sin, float* q_out, KvView kv, const QgemmScratch& sc, cudaStream_t s,
                      bool pdl) {
  QArgs a = base_args(kHidden, tok.nt, kQkvRows / kTileM, 6, sc);
  a.x = src.x;
  a.embed = src.embed;
  a.tokens = src.tokens;
  a.norm_w = L.input_ln;
  QEpiQkv e{L.qkv_b, L.qkv_s, rope_cos, rope_sin, q_out, kv, tok};
  const CUtensorMap& map = *reinterpret_cast<const CUtensorMap*>(m.qkv.bytes);
  if (src.x == nullptr) return run_qgemm<kQEmbedNorm>(map, a, e, s, pdl);
  return run_qgemm<kQNorm>(map, a, e, s, pdl);
}

cudaError_t qgemm_o(const QgemmLayerMaps& m, const LayerDev& L, const float* ctx, int nt, float* out,
                    const QgemmScratch& sc, cudaStream_t s, bool pdl) {
  QArgs a = base_args(kHidden, nt, kHidden / kTileM, 12, sc);
  a.x = ctx;
  QEpiScale e{L.o_s, out};
  return run_qgemm<kQPlain>(*reinterpret_cast<const CUtensorMap*>(m.o.bytes), a, e, s, pdl);
}

cudaError_t qgemm_gateup(const QgemmLayerMaps& m, const LayerDev& L, const float* x, int nt, float* h,
                         const QgemmScratch& sc, cudaStream_t s, bool pdl) {
  QArgs a = base_args(kHidden, nt, kInter / 64, 1, sc);
  a.box_rows = 64;
  a.second_row0 = kInter;
  a.x = x;
  a.norm_w = L.post_ln;
  QEpiGateUp e{L.gu_s, h};
  return run_qgemm<kQNorm>(*reinterpret_cast<const CUtensorMap*>(m.gu.bytes), a, e, s, pdl);
}

cudaError_t qgemm_down(const QgemmLayerMaps& m, const LayerDev& L, const float* h, const float* resid, int nt,
                       float* out, bool round_out, const QgemmScratch& sc, cudaStream_t s, bool pdl) {
  QArgs a = base_args(kInter, nt, kHidden / kTileM, 12, sc);
  a.x = h;
  QEpiDown e{L.down_s, resid, out, round_out};
  return run_qgemm<kQPlain>(*reinterpret_cast<const CUtensorMap*>(m.down.bytes), a, e, s, pdl);
}

cudaError_t qgemm_raw(const QgemmMap& m, int rows, int K, const float* x, int nt, int* acc_out, float* step_out,
                      const QgemmScratch& sc, cudaStream_t s) {
  if (rows % kTileM || K % kKBlock || nt < 1 || nt > 4) return cudaErrorInvalidValue;
  const int nkb = K / kKBlock;
  // split-K only where the shared scratch covers the rows; the single-CTA-per-tile form needs no scratch
  const int split = (nkb % 4 == 0 && rows <= kQkvRows) ? 4 : 1;
  if ((size_t)nkb / split * 2048 + sizeof(Smem) + 2048 > 227 * 1024) return cudaErrorInvalidValue;
  QArgs a = base_args(K, nt, rows / kTileM, split, sc);
  a.x = x;
  QEpiRaw e{acc_out, step_out};
  return run_qgemm<kQPlain>(*reinterpret_cast<const CUtensorMap*>(m.bytes), a, e, s, false);
}

unsigned qgemm_kernel_error(bool reset) {
  unsigned v = 0;
  if (cudaMemcpyFromSymbol(&v, g_kernel_error, sizeof(v)) != cudaSuccess) return 0xFFFFFFFFu;
  if (reset && v) {
    const unsigned z = 0;
    cudaMemcpyToSymbol(g_kernel_error, &z, sizeof(z));
  }
  return v;
}

}  // namespace qb
