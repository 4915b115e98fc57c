// Decode (batch 1..4) projections as HBM-streaming GEMV kernels on the CUDA cores.
//
// Reference computation (`project_tiled`, hls/decode_only/qwen_decode_attention_kernel.cpp:62-98 and
// hls/decode_only/qwen_decode_mlp_kernel.cpp:44-77): y[o] = bias[o] + sum_i x[i] * (code(o,i) * scale[o]),
// accumulated serially in fp32. Here the per-channel scale is applied once in the epilogue,
// y[o] = bias[o] + scale[o] * sum_i x[i] * code(o,i), and the sum is split across lanes and warps
// (fp32 FMA). The reorder changes results by rounding only (relative ~1e-7).
//
// Layout of the work: a warp owns R weight rows ("row group") and walks them in 16-byte chunks, lane l
// taking chunks l, l+32, ... (128-bit, L1-bypassing loads; the next chunk is loaded before the current
// one is consumed). KSPLIT warps may share one row group, each taking a contiguous slice of chunks, and
// reduce through shared memory. Activations for all NT tokens are staged once per CTA in shared memory,
// swizzled so that the per-lane float4 reads of a chunk are bank-conflict free; RMSNorm (decode form:
// double-precision sum of squares, hls/decode_only/qwen_decode_attention_kernel.cpp:13-27) and the
// embedding gather are fused into that staging step. Integer codes become floats with the 2^23
// magic-number trick (byte permute + one FADD), exact for int8 and int4.
#include <cuda_fp16.h>

#include "qwen_kernels.cuh"

namespace qb {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// float4 index swizzle inside one token's activation row in shared memory.
__device__ __forceinline__ int swz(int f) { return f ^ ((f >> 3) & 7); }

__device__ __forceinline__ float comp(const float4& v, int i) {
  return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}

// code byte k (0..3) of an offset-binary word -> 2^23 + code + 128
__device__ __forceinline__ float byte_magic(uint32_t w, int k) {
  return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540u | k));
}

// Multiply-accumulate one 16-byte chunk of one row into acc[t] (and acc_hi[t] for high int4 nibbles,
// which carry a factor 16 removed after the reduction). xs points at this chunk's float4s for token 0;
// tokens are `tstride` float4 apart.
template <int WBITS, int NT>
__device__ __forceinline__ void chunk_fma(const uint4 w, const float4* xs, int f0, int tstride, float (&acc)[NT],
                                          float (&acc_hi)[NT]) {
  const uint32_t words[4] = {w.x, w.y, w.z, w.w};
  if constexpr (WBITS == 8) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t ob = words[q] ^ 0x80808080u;
      float4 xv[NT];
#pragma unroll
      for (int t = 0; t < NT; ++t) xv[t] = xs[t * tstride + swz(f0 + q)];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float wv = byte_magic(ob, k) - 8388736.0f;
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[t] = fmaf(comp(xv[t], k), wv, acc[t]);
      }
    }
  } else if constexpr (WBITS == 4) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t ob = words[q] ^ 0x88888888u;
      float4 xa[NT], xb[NT];
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        xa[t] = xs[t * tstride + swz(f0 + 2 * q)];
        xb[t] = xs[t * tstride + swz(f0 + 2 * q + 1)];
      }
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const uint32_t m = __byte_perm(ob, 0x4B000000u, 0x7540u | b);
        const float lo = __uint_as_float(m & 0x4B00000Fu) - 8388616.0f;
        const float hi = __uint_as_float(m & 0x4B0000F0u) - 8388736.0f;
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          const float4& xv = b < 2 ? xa[t] : xb[t];
          const int c = (b & 1) * 2;
          acc[t] = fmaf(comp(xv, c), lo, acc[t]);
          acc_hi[t] = fmaf(comp(xv, c + 1), hi, acc_hi[t]);
        }
      }
    }
  } else {  // 16: fp16 weights (LM head)
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 wf = __half22float2(*reinterpret_cast<const __half2*>(&words[q]));
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        const float4 xv = xs[t * tstride + swz(f0 + (q >> 1))];
        const int c = (q & 1) * 2;
        acc[t] = fmaf(comp(xv, c), wf.x, acc[t]);
        acc[t] = fmaf(comp(xv, c + 1), wf.y, acc[t]);
      }
    }
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

enum XMode { kXPlain = 0, kXNorm = 1, kXEmbedNorm = 2 };

struct GemvArgs {
  const uint8_t* w;   // row-major codes (rows * K * WBITS / 8 bytes)
  int K;              // input length (1536 or 8960)
  int ngroups;        // row groups
  int nt;             // tokens actually present (<= NT)
  const float* x;     // [nt][K] (kXPlain, kXNorm)
  const uint16_t* embed;
  const int* tokens;
  const float* norm_w;
};

// Stage the activations of nt tokens into shared memory (swizzled), applying the decode RMSNorm when
// asked: out = float((double)x * inv * (double)w), inv = 1 / sqrt(sum(double x^2) / 1536 + eps).
template <int NT, int MODE>
__device__ __forceinline__ void stage_x(const GemvArgs& a, float4* xs, double* red) {
  const int K4 = a.K / 4;
  const int tid = threadIdx.x;
  double ss[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    ss[t] = 0.0;
    if (t < a.nt) {
      for (int i = tid; i < K4; i += kThreads) {
        float4 v;
        if constexpr (MODE == kXEmbedNorm) {
          const uint2 h = *reinterpret_cast<const uint2*>(a.embed + (size_t)a.tokens[t] * kHidden + i * 4);
          const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&h.x));
          const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&h.y));
          v = make_float4(lo.x, lo.y, hi.x, hi.y);
        } else {
          v = reinterpret_cast<const float4*>(a.x + (size_t)t * a.K)[i];
        }
        xs[t * K4 + swz(i)] = v;
        if constexpr (MODE != kXPlain) {
          ss[t] += (double)v.x * v.x + (double)v.y * v.y + (double)v.z * v.z + (double)v.w * v.w;
        }
      }
    } else {
      for (int i = tid; i < K4; i += kThreads) xs[t * K4 + swz(i)] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  if constexpr (MODE != kXPlain) {
    const int warp = tid / 32, lane = tid % 32;
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const double v = warp_sum_d(ss[t]);
      if (lane == 0) red[t * kWarps + warp] = v;
    }
    __syncthreads();
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      double tot = 0.0;
      for (int w = 0; w < kWarps; ++w) tot += red[t * kWarps + w];
      const double inv = 1.0 / sqrt(tot / (double)kHidden + (double)kEps);
      if (t < a.nt) {
        for (int i = tid; i < K4; i += kThreads) {
          float4 v = xs[t * K4 + swz(i)];
          const float4 w = reinterpret_cast<const float4*>(a.norm_w)[i];
          v.x = (float)((double)v.x * inv * (double)w.x);
          v.y = (float)((double)v.y * inv * (double)w.y);
          v.z = (float)((double)v.z * inv * (double)w.z);
          v.w = (float)((double)v.w * inv * (double)w.w);
          xs[t * K4 + swz(i)] = v;
        }
      }
    }
  }
}

template <int WBITS, int NT, int R, int KSPLIT, int MODE, class Epi>
__global__ void __launch_bounds__(kThreads) gemv_kernel(GemvArgs a, Epi epi) {
  extern __shared__ float4 smem[];
  float4* xs = smem;
  float* red = reinterpret_cast<float*>(xs + (size_t)NT * (a.K / 4));
  __shared__ double nred[NT * kWarps];

  griddep_wait();
  stage_x<NT, MODE>(a, xs, nred);
  __syncthreads();
  griddep_launch();

  constexpr int kGroupsPerCta = kWarps / KSPLIT;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int gslot = warp / KSPLIT, part = warp % KSPLIT;
  const int K4 = a.K / 4;
  const size_t row_bytes = (size_t)a.K * WBITS / 8;
  const int nchunks = (int)(row_bytes / 16);
  const int cpp = (nchunks + KSPLIT - 1) / KSPLIT;
  const int c0 = part * cpp;
  const int c1 = min(nchunks, c0 + cpp);
  constexpr int kF4PerChunk = WBITS == 8 ? 4 : (WBITS == 4 ? 8 : 2);

  for (int gbase = blockIdx.x * kGroupsPerCta; gbase < a.ngroups; gbase += gridDim.x * kGroupsPerCta) {
    const int g = gbase + gslot;
    float acc[R][NT], acch[R][NT];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int t = 0; t < NT; ++t) acc[r][t] = acch[r][t] = 0.0f;

    if (g < a.ngroups) {
      const uint8_t* rowp[R];
#pragma unroll
      for (int r = 0; r < R; ++r) rowp[r] = a.w + (size_t)epi.row(g, r) * row_bytes;
      int c = c0 + lane;
      uint4 cur[R];
      if (c < c1) {
#pragma unroll
        for (int r = 0; r < R; ++r) cur[r] = ldg_stream(rowp[r] + (size_t)c * 16);
      }
      for (; c < c1; c += 32) {
        uint4 nxt[R];
        const int cn = c + 32;
        if (cn < c1) {
#pragma unroll
          for (int r = 0; r < R; ++r) nxt[r] = ldg_stream(rowp[r] + (size_t)cn * 16);
        }
#pragma unroll
        for (int r = 0; r < R; ++r) chunk_fma<WBITS, NT>(cur[r], xs, c * kF4PerChunk, K4, acc[r], acch[r]);
#pragma unroll
        for (int r = 0; r < R; ++r) cur[r] = nxt[r];
      }
    }

    float v[R][NT];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        const float s = WBITS == 4 ? fmaf(acch[r][t], 0.0625f, acc[r][t]) : acc[r][t];
        v[r][t] = warp_sum(s);
      }

    if constexpr (KSPLIT == 1) {
      if (g < a.ngroups && lane == 0) epi.finish(g, v, a.nt);
    } else {
      float* slot = red + ((size_t)gslot * KSPLIT + part) * (R * NT);
      if (lane == 0) {
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
          for (int t = 0; t < NT; ++t) slot[r * NT + t] = v[r][t];
      }
      __syncthreads();
      if (part == 0 && lane == 0 && g < a.ngroups) {
        const float* base = red + (size_t)gslot * KSPLIT * (R * NT);
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            float s = 0.0f;
            for (int p = 0; p < KSPLIT; ++p) s += base[p * R * NT + r * NT + t];
            v[r][t] = s;
          }
        epi.finish(g, v, a.nt);
      }
      __syncthreads();
    }
  }
  epi.cta_end(a.nt);
}

// ------------------------------------------------------------------------------------------------
// epilogues
// ------------------------------------------------------------------------------------------------
struct EpiBase {
  __device__ void cta_end(int) {}
};

// q | k | v rows with bias; RoPE on q and k heads (rotate-half pairs p, p+64); K and V rows go to the
// cache at the token's position (qwen_decode_attention_kernel.cpp:100-111, 202-213). Row group g = one
// (head, pair) with rows {h*128 + p, h*128 + p + 64}.
struct EpiQkv : EpiBase {
  const float* bias;
  const float* scale;
  const float* cosv;  // [pos][64]
  const float* sinv;
  float* q_out;
  KvView kv;
  DecodeTokens tok;
  __device__ int row(int g, int r) const { return (g >> 6) * kHeadDim + (g & 63) + r * 64; }
  template <int NT>
  __device__ void finish(int g, const float (&v)[2][NT], int nt) const {
    const int h = g >> 6, p = g & 63;
    const int re = h * kHeadDim + p, ro = re + 64;
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      if (t >= nt) break;
      float ye = bias[re] + scale[re] * v[0][t];
      float yo = bias[ro] + scale[ro] * v[1][t];
      const int pos = tok.pos[t];
      if (h < kHeads + kKvHeads) {
        const float c = cosv[(size_t)pos * 64 + p], s = sinv[(size_t)pos * 64 + p];
        const float ne = __fsub_rn(__fmul_rn(ye, c), __fmul_rn(yo, s));
        const float no = __fadd_rn(__fmul_rn(yo, c), __fmul_rn(ye, s));
        ye = ne;
        yo = no;
      }
      if (h < kHeads) {
        q_out[(size_t)t * kHidden + re] = ye;
        q_out[(size_t)t * kHidden + ro] = yo;
      } else {
        const int which = h < kHeads + kKvHeads ? 0 : 1;
        float* dst = kv_row(kv, tok.seq[t], pos, which);
        const int base = re - kHidden - which * kKvWidth;
        dst[base] = ye;
        dst[base + 64] = yo;
      }
    }
  }
};

// y = scale * acc (o_proj: no bias, no residual, qwen_decode_attention_kernel.cpp:215).
template <int R>
struct EpiScale : EpiBase {
  const float* scale;
  float* out;
  int n;  // output row length
  __device__ int row(int g, int r) const { return g * R + r; }
  template <int NT>
  __device__ void finish(int g, const float (&v)[R][NT], int nt) const {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int o = g * R + r;
#pragma unroll
      for (int t = 0; t < NT; ++t)
        if (t < nt) out[(size_t)t * n + o] = scale[o] * v[r][t];
    }
  }
};

// h[j] = silu(gate[j]) * up[j] with silu(v) = v / (1 + expf(-v)) (qwen_decode_mlp_kernel.cpp:79-81,
// 113-115). Row group g covers j = 2g, 2g+1: rows {j, 8960 + j, j + 1, 8960 + j + 1}.
struct EpiGateUp : EpiBase {
  const float* scale;  // gate | up scales
  float* h;
  __device__ int row(int g, int r) const { return 2 * g + (r >> 1) + (r & 1) * kInter; }
  template <int NT>
  __device__ void finish(int g, const float (&v)[4][NT], int nt) const {
#pragma unroll
    for (int jj = 0; jj < 2; ++jj) {
      const int j = 2 * g + jj;
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        if (t >= nt) break;
        const float gv = scale[j] * v[2 * jj][t];
        const float uv = scale[kInter + j] * v[2 * jj + 1][t];
        const float silu = __fdiv_rn(gv, __fadd_rn(1.0f, expf(-gv)));
        h[(size_t)t * kInter + j] = __fmul_rn(silu, uv);
      }
    }
  }
};

// out = a + scale * acc (qwen_decode_mlp_kernel.cpp:116-119), optionally rounded to bf16 for the next
// layer (the caller's rounding, verification/real_host_top_backend.py:334).
template <int R>
struct EpiDown : EpiBase {
  const float* scale;
  const float* a;
  float* out;
  bool round_out;
  __device__ int row(int g, int r) const { return g * R + r; }
  template <int NT>
  __device__ void finish(int g, const float (&v)[R][NT], int nt) const {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int o = g * R + r;
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        if (t >= nt) break;
        float y = __fadd_rn(a[(size_t)t * kHidden + o], scale[o] * v[r][t]);
        if (round_out) y = round_bf16(y);
        out[(size_t)t * kHidden + o] = y;
      }
    }
  }
};

// Greedy LM head: logits[v] = E[v] . y, argmax with the lowest index winning ties. Each warp keeps its
// best per token; the CTA reduces them into `partial`, and the last CTA to finish reduces all CTAs.
template <int R, int NT>
struct EpiLm {
  float* logits;  // optional
  float* partial; // [gridDim][NT][2]
  unsigned* counter;
  int* next_token;
  // per-lane-0 running best (lives in registers of the calling thread)
  mutable float best_v[NT];
  mutable int best_i[NT];
  __device__ int row(int g, int r) const { return g * R + r; }
  __device__ void init() const {
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      best_v[t] = -INFINITY;
      best_i[t] = 0x7fffffff;
    }
  }
  template <int NT2>
  __device__ void finish(int g, const float (&v)[R][NT2], int nt) const {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int o = g * R + r;
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        if (t >= nt) break;
        if (logits) logits[(size_t)t * kVocab + o] = v[r][t];
        if (v[r][t] > best_v[t] || (v[r][t] == best_v[t] && o < best_i[t])) {
          best_v[t] = v[r][t];
          best_i[t] = o;
        }
      }
    }
  }
  __device__ void cta_end(int nt) const {
    __shared__ float sv[kWarps][NT];
    __shared__ int si[kWarps][NT];
    __shared__ bool last;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    if (lane == 0) {
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        sv[warp][t] = best_v[t];
        si[warp][t] = best_i[t];
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int t = 0; t < nt; ++t) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int w = 0; w < kWarps; ++w)
          if (sv[w][t] > bv || (sv[w][t] == bv && si[w][t] < bi)) {
            bv = sv[w][t];
            bi = si[w][t];
          }
        partial[((size_t)blockIdx.x * NT + t) * 2] = bv;
        partial[((size_t)blockIdx.x * NT + t) * 2 + 1] = __int_as_float(bi);
      }
      __threadfence();
      const unsigned prev = atomicAdd(counter, 1u);
      last = (prev == gridDim.x - 1);
    }
    __syncthreads();
    if (last && threadIdx.x == 0) {
      __threadfence();
      for (int t = 0; t < nt; ++t) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (unsigned b = 0; b < gridDim.x; ++b) {
          const float pv = __ldcg(&partial[((size_t)b * NT + t) * 2]);
          const int pi = __float_as_int(__ldcg(&partial[((size_t)b * NT + t) * 2 + 1]));
          if (pv > bv || (pv == bv && pi < bi)) {
            bv = pv;
            bi = pi;
          }
        }
        next_token[t] = bi;
      }
      *counter = 0u;
    }
  }
};

template <int WBITS, int NT, int R, int KSPLIT, int MODE, class Epi>
cudaError_t run_gemv(const GemvArgs& a, const Epi& epi, int grid, cudaStream_t s, bool pdl) {
  const size_t smem = (size_t)NT * a.K * sizeof(float) + (KSPLIT > 1 ? (size_t)kWarps * R * NT * sizeof(float) : 0);
  auto kern = gemv_kernel<WBITS, NT, R, KSPLIT, MODE, Epi>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  return launch_k(kern, dim3(grid), dim3(kThreads), smem, s, pdl, a, epi);
}

int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

int grid_for(int ngroups, int groups_per_cta, int max_ctas) {
  const int need = (ngroups + groups_per_cta - 1) / groups_per_cta;
  return need < max_ctas ? need : max_ctas;
}

// Dispatch on (wbits, nt) to compiled instances.
template <int R, int KSPLIT, int MODE, class Epi, int NT>
cudaError_t dispatch_wbits(int wbits, const GemvArgs& a, const Epi& e, int grid, cudaStream_t s, bool pdl) {
  if (wbits == 8) return run_gemv<8, NT, R, KSPLIT, MODE>(a, e, grid, s, pdl);
  if (wbits == 4) return run_gemv<4, NT, R, KSPLIT, MODE>(a, e, grid, s, pdl);
  return cudaErrorInvalidValue;
}

template <int R, int KSPLIT, int MODE, class Epi>
cudaError_t dispatch(int wbits, const GemvArgs& a, const Epi& e, int grid, cudaStream_t s, bool pdl) {
  switch (a.nt) {
    case 1: return dispatch_wbits<R, KSPLIT, MODE, Epi, 1>(wbits, a, e, grid, s, pdl);
    case 2: return dispatch_wbits<R, KSPLIT, MODE, Epi, 2>(wbits, a, e, grid, s, pdl);
    case 3:
    case 4: return dispatch_wbits<R, KSPLIT, MODE, Epi, 4>(wbits, a, e, grid, s, pdl);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

cudaError_t launch_decode_qkv(int wbits, const LayerDev& L, XSource src, DecodeTokens tok, const float* rope_cos,
                              const float* rope_sin, float* q_out, KvView kv, cudaStream_t s, bool pdl) {
  GemvArgs a{};
  a.w = L.qkv_w;
  a.K = kHidden;
  a.ngroups = kQkvRows / 2;  // (head, pair) groups
  a.nt = tok.nt;
  a.x = src.x;
  a.embed = src.embed;
  a.tokens = src.tokens;
  a.norm_w = L.input_ln;
  EpiQkv e;
  e.bias = L.qkv_b;
  e.scale = L.qkv_s;
  e.cosv = rope_cos;
  e.sinv = rope_sin;
  e.q_out = q_out;
  e.kv = kv;
  e.tok = tok;
  const int grid = grid_for(a.ngroups, kWarps, 4 * num_sms());
  if (src.x == nullptr) return dispatch<2, 1, kXEmbedNorm>(wbits, a, e, grid, s, pdl);
  return dispatch<2, 1, kXNorm>(wbits, a, e, grid, s, pdl);
}

cudaError_t launch_decode_o(int wbits, const LayerDev& L, const float* ctx, int nt, float* out, cudaStream_t s,
                            bool pdl) {
  GemvArgs a{};
  a.w = L.o_w;
  a.K = kHidden;
  a.ngroups = kHidden / 2;
  a.nt = nt;
  a.x = ctx;
  EpiScale<2> e;
  e.scale = L.o_s;
  e.out = out;
  e.n = kHidden;
  const int grid = grid_for(a.ngroups, kWarps / 2, 4 * num_sms());
  return dispatch<2, 2, kXPlain>(wbits, a, e, grid, s, pdl);
}

cudaError_t launch_decode_gateup(int wbits, const LayerDev& L, const float* x, int nt, float* h, cudaStream_t s,
                                 bool pdl) {
  GemvArgs a{};
  a.w = L.gu_w;
  a.K = kHidden;
  a.ngroups = kInter / 2;
  a.nt = nt;
  a.x = x;
  a.norm_w = L.post_ln;
  EpiGateUp e;
  e.scale = L.gu_s;
  e.h = h;
  const int grid = grid_for(a.ngroups, kWarps, 4 * num_sms());
  return dispatch<4, 1, kXNorm>(wbits, a, e, grid, s, pdl);
}

cudaError_t launch_decode_down(int wbits, const LayerDev& L, const float* h, const float* a_res, int nt, float* out,
                               bool round_out, cudaStream_t s, bool pdl) {
  GemvArgs a{};
  a.w = L.down_w;
  a.K = kInter;
  a.ngroups = kHidden / 4;
  a.nt = nt;
  a.x = h;
  EpiDown<4> e;
  e.scale = L.down_s;
  e.a = a_res;
  e.out = out;
  e.round_out = round_out;
  const int grid = grid_for(a.ngroups, 1, 4 * num_sms());
  return dispatch<4, 8, kXPlain>(wbits, a, e, grid, s, pdl);
}

namespace {
constexpr int kLmR = 4;
constexpr int kLmGrid = 4 * 148;
template <int NT>
__global__ void __launch_bounds__(kThreads) lm_head_kernel(GemvArgs a, EpiLm<kLmR, NT> epi) {
  epi.init();
  // Reuse the generic body through a thin wrapper: identical to gemv_kernel<16, NT, kLmR, 1, kXNorm>.
  extern __shared__ float4 smem[];
  float4* xs = smem;
  __shared__ double nred[NT * kWarps];
  griddep_wait();
  stage_x<NT, kXNorm>(a, xs, nred);
  __syncthreads();
  griddep_launch();
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int K4 = a.K / 4;
  const size_t row_bytes = (size_t)a.K * 2;
  const int nchunks = (int)(row_bytes / 16);
  for (int gbase = blockIdx.x * kWarps; gbase < a.ngroups; gbase += gridDim.x * kWarps) {
    const int g = gbase + warp;
    float acc[kLmR][NT], acch[kLmR][NT];
#pragma unroll
    for (int r = 0; r < kLmR; ++r)
#pragma unroll
      for (int t = 0; t < NT; ++t) acc[r][t] = acch[r][t] = 0.0f;
    if (g < a.ngroups) {
      const uint8_t* rowp[kLmR];
#pragma unroll
      for (int r = 0; r < kLmR; ++r) rowp[r] = a.w + (size_t)(g * kLmR + r) * row_bytes;
      int c = lane;
      uint4 cur[kLmR];
#pragma unroll
      for (int r = 0; r < kLmR; ++r) cur[r] = ldg_stream(rowp[r] + (size_t)c * 16);
      for (; c < nchunks; c += 32) {
        uint4 nxt[kLmR];
        if (c + 32 < nchunks) {
#pragma unroll
          for (int r = 0; r < kLmR; ++r) nxt[r] = ldg_stream(rowp[r] + (size_t)(c + 32) * 16);
        }
#pragma unroll
        for (int r = 0; r < kLmR; ++r) chunk_fma<16, NT>(cur[r], xs, c * 2, K4, acc[r], acch[r]);
#pragma unroll
        for (int r = 0; r < kLmR; ++r) cur[r] = nxt[r];
      }
    }
    float v[kLmR][NT];
#pragma unroll
    for (int r = 0; r < kLmR; ++r)
#pragma unroll
      for (int t = 0; t < NT; ++t) v[r][t] = warp_sum(acc[r][t]);
    if (g < a.ngroups && lane == 0) epi.finish(g, v, a.nt);
  }
  epi.cta_end(a.nt);
}

template <int NT>
cudaError_t run_lm(const GemvArgs& a, const EpiLm<kLmR, NT>& e, cudaStream_t s, bool pdl) {
  const size_t smem = (size_t)NT * a.K * sizeof(float);
  return launch_k(lm_head_kernel<NT>, dim3(kLmGrid), dim3(kThreads), smem, s, pdl, a, e);
}
}  // namespace

int lm_head_partial_floats() { return kLmGrid * kGemvMaxTokens * 2; }

cudaError_t launch_lm_head_argmax(const uint16_t* embed, const float* norm_w, const float* x, int nt, float* logits,
                                  float* partial, unsigned* counter, int* next_token, cudaStream_t s, bool pdl) {
  GemvArgs a{};
  a.w = reinterpret_cast<const uint8_t*>(embed);
  a.K = kHidden;
  a.ngroups = kVocab / kLmR;
  a.nt = nt;
  a.x = x;
  a.norm_w = norm_w;
  switch (nt) {
    case 1: {
      EpiLm<kLmR, 1> e{logits, partial, counter, next_token};
      return run_lm<1>(a, e, s, pdl);
    }
    case 2: {
      EpiLm<kLmR, 2> e{logits, partial, counter, next_token};
      return run_lm<2>(a, e, s, pdl);
    }
    case 3:
    case 4: {
      EpiLm<kLmR, 4> e{logits, partial, counter, next_token};
      return run_lm<4>(a, e, s, pdl);
    }
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace qb
