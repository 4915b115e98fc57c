// Prefill (sequence) kernels on the CUDA cores: the exact prefill RMSNorm, the RoPE table, and the four
// projection GEMMs with their fused epilogues.
//
// RMSNorm (hls/prefill_only/qwen_prefill_attention_kernel.cpp:112-126, qwen_prefill_mlp_kernel.cpp:201-215):
// one thread per token sums x^2 serially in fp32 in the reference's order, so the normalised rows are
// bit-identical to the reference.
//
// Projections (`project_tiled_token`, qwen_prefill_attention_kernel.cpp:163-202; `project_tiled`,
// qwen_prefill_mlp_kernel.cpp:217-254): Y[t][o] = bias[o] + scale[o] * sum_i X[t][i] * code(o, i), fp32
// FMA over 64x64 output tiles with K-steps of 32. Epilogues: bias + RoPE (approx table) + K/V cache
// write for q|k|v; SiLU(approx_exp) * up for gate|up; `+ a` (optional bf16 rounding) for down.
#include "qwen_kernels.cuh"

namespace qb {
namespace {

// ---- RMSNorm -------------------------------------------------------------------------------------
// CTA = 8 tokens. The reference's sum of squares is one serial fp32 chain per token (kept bit for bit):
// all 128 threads stage the 8 rows in shared memory with asynchronous 16-byte copies, every one in flight
// at once, lanes 0..7 of warp 0 run the 8 chains (rows padded by four floats: 16-byte aligned, and the
// lanes read different banks), then all threads write the normalised rows from shared memory.
constexpr int kNormTok = 8, kNormPad = kHidden + 4;
constexpr size_t kNormSmem = (size_t)kNormTok * kNormPad * 4 + kNormTok * 4;

__global__ void __launch_bounds__(128) prefill_rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                              int S, float* __restrict__ xn) {
  griddep_wait();  // inputs come from the preceding kernel (programmatic dependent launch)
  griddep_launch();
  extern __shared__ float nsm[];
  float* rows = nsm;                          // [kNormTok][kNormPad]
  float* inv_s = nsm + kNormTok * kNormPad;   // [kNormTok]
  const int t0 = blockIdx.x * kNormTok, tid = threadIdx.x;
  const int n = min(kNormTok, S - t0);
  for (int i = tid; i < n * (kHidden / 4); i += 128) {
    const int r = i / (kHidden / 4), f = i % (kHidden / 4);
    const unsigned dst = (unsigned)__cvta_generic_to_shared(rows + r * kNormPad + 4 * f);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(x + (size_t)(t0 + r) * kHidden + 4 * f)
                 : "memory");
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();
  if (tid < n) {
    const float* row = rows + tid * kNormPad;
    float ms = 0.0f;
#pragma unroll 16
    for (int d = 0; d < kHidden; ++d) ms = __fadd_rn(ms, __fmul_rn(row[d], row[d]));
    ms = __fdiv_rn(ms, (float)kHidden);
    inv_s[tid] = __fdiv_rn(1.0f, approx_sqrt(__fadd_rn(ms, kEps)));
  }
  __syncthreads();
  for (int i = tid; i < n * kHidden; i += 128) {
    const int r = i / kHidden, d = i % kHidden;
    xn[(size_t)(t0 + r) * kHidden + d] = __fmul_rn(__fmul_rn(rows[r * kNormPad + d], inv_s[r]), __ldg(w + d));
  }
}

// ---- RoPE table (qwen_prefill_attention_kernel.cpp:128-143) ---------------------------------------
__global__ void prefill_rope_table_kernel(int npos, float* __restrict__ cos_out, float* __restrict__ sin_out) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= npos * 64) return;
  const int pos = idx / 64, pair = idx % 64;
  float inv_freq = 1.0f;
  for (int p = 0; p < pair; ++p) inv_freq = __fmul_rn(inv_freq, kRopeFreqStep);
  const float angle = __fmul_rn((float)pos, inv_freq);
  float s, c;
  approx_sincos(angle, &s, &c);
  cos_out[idx] = c;
  sin_out[idx] = s;
}

// ---- GEMM ----------------------------------------------------------------------------------------
constexpr int BM = 64, BN = 64, BK = 32;

enum Epi { kEpiQkv = 0, kEpiScale = 1, kEpiGateUp = 2, kEpiDown = 3 };

struct GemmArgs {
  const float* x;       // [S][K]
  const uint8_t* w;     // codes, row-major [N][K]
  const float* scale;
  const float* bias;    // q|k|v only
  int S, K, wbits;
  // epilogue outputs
  float* out;           // q (Qkv), y (Scale, Down), h (GateUp)
  float* k_cache;
  float* v_cache;
  const float* cosv;
  const float* sinv;
  const float* resid;   // down: a
  bool round_out;
};

// row of the weight matrix for local tile column nl of column tile `tn`
template <int EPI>
__device__ __forceinline__ int tile_row(int tn, int nl) {
  if constexpr (EPI == kEpiQkv) {
    // tile = (head, pair block): columns 0..31 -> pairs, 32..63 -> their partners 64 apart
    const int h = tn >> 1, pb = tn & 1;
    return h * kHeadDim + pb * 32 + (nl & 31) + (nl >> 5) * 64;
  } else if constexpr (EPI == kEpiGateUp) {
    return tn * 32 + (nl & 31) + (nl >> 5) * kInter;
  } else {
    return tn * BN + nl;
  }
}

__device__ __forceinline__ float code_at(const uint8_t* row, int k, int wbits) {
  if (wbits == 8) return (float)(int8_t)row[k];
  const uint8_t b = row[k >> 1];
  const int nib = (k & 1) ? (b >> 4) : (b & 0xF);
  return (float)(nib >= 8 ? nib - 16 : nib);
}

template <int EPI>
__global__ void __launch_bounds__(256) prefill_gemm_kernel(GemmArgs a) {
  __shared__ float As[BK][BM + 4];
  __shared__ float Bs[BK][BN + 4];
  const int tm = blockIdx.y, tn = blockIdx.x;
  const int tid = threadIdx.x, tx = tid % 16, ty = tid / 16;
  const size_t row_bytes = (size_t)a.K * a.wbits / 8;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;

  for (int k0 = 0; k0 < a.K; k0 += BK) {
    // A tile: 64 tokens x 32 k
    for (int i = tid; i < BM * BK; i += 256) {
      const int m = i / BK, kk = i % BK;
      const int t = tm * BM + m;
      As[kk][m] = t < a.S ? a.x[(size_t)t * a.K + k0 + kk] : 0.0f;
    }
    // B tile: 64 rows x 32 k (codes as floats)
    for (int i = tid; i < BN * BK; i += 256) {
      const int nl = i / BK, kk = i % BK;
      const int r = tile_row<EPI>(tn, nl);
      Bs[kk][nl] = code_at(a.w + (size_t)r * row_bytes, k0 + kk, a.wbits);
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < BK; ++kk) {
      float av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) av[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) bv[j] = Bs[kk][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }

#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int t = tm * BM + ty * 4 + i;
    if (t >= a.S) continue;
    if constexpr (EPI == kEpiQkv) {
#pragma unroll
      for (int jp = 0; jp < 2; ++jp) {
        const int ne = tx + 16 * jp, no = ne + 32;
        const int re = tile_row<EPI>(tn, ne), ro = tile_row<EPI>(tn, no);
        float ye = a.bias[re] + a.scale[re] * acc[i][jp];
        float yo = a.bias[ro] + a.scale[ro] * acc[i][jp + 2];
        const int h = re / kHeadDim, p = re % kHeadDim;
        if (h < kHeads + kKvHeads) {
          const float c = a.cosv[(size_t)t * 64 + p], s = a.sinv[(size_t)t * 64 + p];
          const float e2 = __fsub_rn(__fmul_rn(ye, c), __fmul_rn(yo, s));
          const float o2 = __fadd_rn(__fmul_rn(yo, c), __fmul_rn(ye, s));
          ye = e2;
          yo = o2;
        }
        if (h < kHeads) {
          a.out[(size_t)t * kHidden + re] = ye;
          a.out[(size_t)t * kHidden + ro] = yo;
        } else if (h < kHeads + kKvHeads) {
          a.k_cache[(size_t)t * kKvWidth + re - kHidden] = ye;
          a.k_cache[(size_t)t * kKvWidth + ro - kHidden] = yo;
        } else {
          a.v_cache[(size_t)t * kKvWidth + re - kHidden - kKvWidth] = ye;
          a.v_cache[(size_t)t * kKvWidth + ro - kHidden - kKvWidth] = yo;
        }
      }
    } else if constexpr (EPI == kEpiGateUp) {
#pragma unroll
      for (int jp = 0; jp < 2; ++jp) {
        const int j = tile_row<EPI>(tn, tx + 16 * jp);
        const float gv = a.scale[j] * acc[i][jp];
        const float uv = a.scale[kInter + j] * acc[i][jp + 2];
        const float silu = __fdiv_rn(gv, __fadd_rn(1.0f, approx_exp_fast(-gv)));
        a.out[(size_t)t * kInter + j] = __fmul_rn(silu, uv);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int r = tile_row<EPI>(tn, tx + 16 * j);
        float y = a.scale[r] * acc[i][j];
        if constexpr (EPI == kEpiDown) {
          y = __fadd_rn(a.resid[(size_t)t * kHidden + r], y);
          if (a.round_out) y = round_bf16(y);
        }
        a.out[(size_t)t * kHidden + r] = y;
      }
    }
  }
}

template <int EPI>
cudaError_t run_gemm(const GemmArgs& a, int n_tiles, cudaStream_t s) {
  prefill_gemm_kernel<EPI><<<dim3(n_tiles, (a.S + BM - 1) / BM), 256, 0, s>>>(a);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_prefill_rmsnorm(const float* x, const float* w, int S, float* xn, cudaStream_t s) {
  if (reinterpret_cast<uintptr_t>(x) & 15) return cudaErrorInvalidValue;  // 16-byte asynchronous row copies
  const cudaError_t e =
      cudaFuncSetAttribute(prefill_rmsnorm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kNormSmem);
  if (e != cudaSuccess) return e;
  return launch_k(prefill_rmsnorm_kernel, dim3((S + kNormTok - 1) / kNormTok), dim3(128), kNormSmem, s, true, x, w, S,
                  xn);
}

cudaError_t launch_prefill_rope_table(int npos, float* cos_out, float* sin_out, cudaStream_t s) {
  const int n = npos * 64;
  prefill_rope_table_kernel<<<(n + 255) / 256, 256, 0, s>>>(npos, cos_out, sin_out);
  return cudaGetLastError();
}

cudaError_t launch_prefill_qkv(int wbits, const LayerDev& L, const float* xn, int S, const float* rope_cos,
                               const float* rope_sin, float* q_out, float* k_cache, float* v_cache, cudaStream_t s) {
  GemmArgs a{};
  a.x = xn;
  a.w = L.qkv_w;
  a.scale = L.qkv_s;
  a.bias = L.qkv_b;
  a.S = S;
  a.K = kHidden;
  a.wbits = wbits;
  a.out = q_out;
  a.k_cache = k_cache;
  a.v_cache = v_cache;
  a.cosv = rope_cos;
  a.sinv = rope_sin;
  return run_gemm<kEpiQkv>(a, kQkvRows / BN, s);
}

cudaError_t launch_prefill_o(int wbits, const LayerDev& L, const float* ctx, int S, float* out, cudaStream_t s) {
  GemmArgs a{};
  a.x = ctx;
  a.w = L.o_w;
  a.scale = L.o_s;
  a.S = S;
  a.K = kHidden;
  a.wbits = wbits;
  a.out = out;
  return run_gemm<kEpiScale>(a, kHidden / BN, s);
}

cudaError_t launch_prefill_gateup(int wbits, const LayerDev& L, const float* xn, int S, float* h, cudaStream_t s) {
  GemmArgs a{};
  a.x = xn;
  a.w = L.gu_w;
  a.scale = L.gu_s;
  a.S = S;
  a.K = kHidden;
  a.wbits = wbits;
  a.out = h;
  return run_gemm<kEpiGateUp>(a, kInter / 32, s);
}

cudaError_t launch_prefill_down(int wbits, const LayerDev& L, const float* h, const float* resid, int S, float* out,
                                bool round_out, cudaStream_t s) {
  GemmArgs a{};
  a.x = h;
  a.w = L.down_w;
  a.scale = L.down_s;
  a.S = S;
  a.K = kInter;
  a.wbits = wbits;
  a.out = out;
  a.resid = resid;
  a.round_out = round_out;
  return run_gemm<kEpiDown>(a, kHidden / BN, s);
}

}  // namespace qb
