// Decode (batch 1..4) projections as HBM-streaming GEMV kernels on the CUDA cores.
//
// Reference computation (`project_tiled`, hls/decode_only/qwen_decode_attention_kernel.cpp:62-98 and
// hls/decode_only/qwen_decode_mlp_kernel.cpp:44-77): y[o] = bias[o] + sum_i x[i] * (code(o,i) * scale[o]),
// accumulated serially in fp32. Here the per-channel scale is applied once in the epilogue,
// y[o] = bias[o] + scale[o] * sum_i x[i] * code(o,i), and the sum is split across lanes (fp32 FMA). The
// reorder changes results by rounding only (relative ~1e-7).
//
// Structure (one persistent CTA per SM): a producer warp streams the weight rows of 8-row work units into
// a ring of shared-memory stages with cp.async.bulk copies completing on mbarriers, starting before the
// kernel waits for its predecessor (weights do not depend on it), so HBM is busy from the first cycle.
// Eight consumer warps take one row each: lane l multiplies 16-byte chunks l, l+32, ... of its row slice
// with the activations (staged once per CTA in shared memory, swizzled for conflict-free float4 reads;
// RMSNorm in the decode form -- double sum of squares, hls/decode_only/qwen_decode_attention_kernel.cpp:13-27
// -- and the embedding gather are fused into that staging), then reduces with warp shuffles. Row results
// meet in shared memory for the pairwise epilogues (RoPE pairs p/p+64, SiLU(gate) * up). Integer codes
// become floats with the 2^23 magic-number trick (byte permute + one FADD), exact for int8 and int4.
#include <cuda_fp16.h>

#include "qwen_kernels.cuh"
#include "sm100_async.cuh"

namespace qb {
namespace {

constexpr int kRows = 8;                   // rows per work unit = consumer warps
constexpr int kConsumers = kRows * 32;     // consumer threads
constexpr int kThreads = kConsumers + 32;  // + one producer warp
constexpr int kBarConsumers = 1;           // named barrier id among consumer warps
constexpr int kSmemTarget = 110 * 1024;    // stay below half an SM so the next kernel's CTA fits beside

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
// which carry a factor 16 removed after the reduction). f0 is the chunk's first float4 index in the
// activation row; tokens are `tstride` float4 apart.
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
  int nunits;         // 8-row work units
  int nt;             // tokens actually present (<= NT)
  const float* x;     // [nt][K] (kXPlain, kXNorm)
  const uint16_t* embed;
  const int* tokens;
  const float* norm_w;
  const uint8_t* pf;  // optional L2 prefetch hint (next kernels' weights)
  size_t pf_bytes;
  int kb_bytes;       // bytes of one row per stage (a column block)
  int nkb;            // column blocks per row
  int nstages;        // ring depth
};

// Stage the activations of nt tokens into shared memory (swizzled), applying the decode RMSNorm when
// asked: out = float((double)x * inv * (double)w), inv = 1 / sqrt(sum(double x^2) / 1536 + eps).
// Run by the consumer warps only.
template <int NT, int MODE>
__device__ __forceinline__ void stage_x(const GemvArgs& a, float4* xs, double* red) {
  const int K4 = a.K / 4;
  const int tid = threadIdx.x;
  double ss[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    ss[t] = 0.0;
    if (t < a.nt) {
      for (int i = tid; i < K4; i += kConsumers) {
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
      for (int i = tid; i < K4; i += kConsumers) xs[t * K4 + swz(i)] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  if constexpr (MODE != kXPlain) {
    const int warp = tid / 32, lane = tid % 32;
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const double v = warp_sum_d(ss[t]);
      if (lane == 0) red[t * kRows + warp] = v;
    }
    named_sync(kBarConsumers, kConsumers);
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      double tot = 0.0;
      for (int w = 0; w < kRows; ++w) tot += red[t * kRows + w];
      const double inv = 1.0 / sqrt(tot / (double)kHidden + (double)kEps);
      if (t < a.nt) {
        for (int i = tid; i < K4; i += kConsumers) {
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

template <int WBITS, int NT, int MODE, class Epi>
__global__ void __launch_bounds__(kThreads, 1) gemv_kernel(GemvArgs a, Epi epi) {
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + a.nstages;
  float4* xs = reinterpret_cast<float4*>(smem + 256);
  const int K4 = a.K / 4;
  uint8_t* stages = reinterpret_cast<uint8_t*>(xs + (size_t)NT * K4);
  float* red = reinterpret_cast<float*>(stages + (size_t)a.nstages * kRows * a.kb_bytes);
  __shared__ double nred[NT * kRows];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const size_t row_bytes = (size_t)a.K * WBITS / 8;

  if (threadIdx.x == 0) {
    for (int s = 0; s < a.nstages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kRows);
    }
    mbar_fence_init();
  }
  __syncthreads();

  if (warp == kRows) {
    // ---- producer warp: weights are independent of the preceding kernel, so no grid-dependency wait.
    if (a.pf != nullptr && a.pf_bytes != 0) {
      const size_t per = ((a.pf_bytes + gridDim.x - 1) / gridDim.x + 15) & ~size_t(15);
      const size_t b0 = (size_t)blockIdx.x * per, b1 = min(a.pf_bytes, b0 + per);
      for (size_t off = b0 + (size_t)lane * 32768; off < b1; off += 32 * 32768)
        prefetch_l2(a.pf + off, (unsigned)min((size_t)32768, b1 - off));
    }
    if (lane == 0) {
      int s = 0;
      unsigned ph = 0;
      const unsigned stage_tx = (unsigned)(kRows * a.kb_bytes);
      bool ok = true;
      for (int u = blockIdx.x; u < a.nunits && ok; u += gridDim.x) {
        for (int kb = 0; kb < a.nkb; ++kb) {
          if (!(ok = mbar_wait(&empty[s], ph ^ 1))) break;
          mbar_arrive_expect_tx(&full[s], stage_tx);
          uint8_t* dst = stages + (size_t)s * kRows * a.kb_bytes;
#pragma unroll
          for (int r = 0; r < kRows; ++r)
            bulk_g2s(dst + (size_t)r * a.kb_bytes, a.w + (size_t)epi.row(u, r) * row_bytes + (size_t)kb * a.kb_bytes,
                     (unsigned)a.kb_bytes, &full[s]);
          if (++s == a.nstages) {
            s = 0;
            ph ^= 1;
          }
        }
      }
      // every stage released by the consumers => no copy is still in flight when the CTA exits
      for (int i = 0; i < a.nstages && ok; ++i) {
        ok = mbar_wait(&empty[s], ph ^ 1);
        if (++s == a.nstages) {
          s = 0;
          ph ^= 1;
        }
      }
    }
    return;
  }

  // ---- consumer warps
  griddep_wait();
  stage_x<NT, MODE>(a, xs, nred);
  named_sync(kBarConsumers, kConsumers);
  if (threadIdx.x == 0) griddep_launch();

  const int kb_chunks = a.kb_bytes / 16;
  constexpr int kF4PerChunk = WBITS == 8 ? 4 : (WBITS == 4 ? 8 : 2);
  int s = 0;
  unsigned ph = 0;
  int slot = 0;
  bool dead = false;  // a bounded wait gave up: keep the barrier schedule, skip the work
  for (int u = blockIdx.x; u < a.nunits; u += gridDim.x) {
    const int row = epi.row(u, warp);
    const typename Epi::Pre pre = epi.preload(row, lane);
    float acc[NT], acch[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[t] = acch[t] = 0.0f;
    for (int kb = 0; kb < a.nkb; ++kb) {
      if (!dead && !mbar_wait(&full[s], ph)) dead = true;
      if (!dead) {
        const uint4* srow = reinterpret_cast<const uint4*>(stages + ((size_t)s * kRows + warp) * a.kb_bytes);
        const int fbase = kb * kb_chunks * kF4PerChunk;
        for (int c = lane; c < kb_chunks; c += 32)
          chunk_fma<WBITS, NT>(srow[c], xs, fbase + c * kF4PerChunk, K4, acc, acch);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      if (++s == a.nstages) {
        s = 0;
        ph ^= 1;
      }
    }
    float v[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) v[t] = warp_sum(WBITS == 4 ? fmaf(acch[t], 0.0625f, acc[t]) : acc[t]);
    float* rs = red + (size_t)slot * kRows * NT;
    epi.row_done(u, warp, lane, row, pre, v, rs, a.nt);
    if (Epi::kPairs) {
      named_sync(kBarConsumers, kConsumers);
      epi.pair_done(u, warp, lane, row, rs, a.nt);
    }
    slot ^= 1;
  }
  epi.cta_end(a.nt);
}

// ------------------------------------------------------------------------------------------------
// epilogues: row(u, w) maps work unit u and consumer warp w to a weight row; row_done() runs in every
// consumer warp (lanes < nt, one token each) once its row is reduced; pair_done() runs after all eight
// rows of the unit are in shared memory (Epi::kPairs).
// ------------------------------------------------------------------------------------------------
struct NoPre {};

struct EpiBase {
  __device__ void cta_end(int) const {}
};

// q | k | v rows with bias; RoPE on q and k heads (rotate-half pairs p, p+64); K and V rows go to the
// cache at the token's position (qwen_decode_attention_kernel.cpp:100-111, 202-213). Unit u = 4 pairs of
// one head: warp w holds row h*128 + p0 + (w >> 1) + 64 * (w & 1).
struct EpiQkv : EpiBase {
  static constexpr bool kPairs = true;
  struct Pre {
    float bias, scale;
  };
  const float* bias;
  const float* scale;
  const float* cosv;  // [pos][64]
  const float* sinv;
  float* q_out;
  KvView kv;
  DecodeTokens tok;
  __device__ int row(int u, int w) const { return (u >> 4) * kHeadDim + (u & 15) * 4 + (w >> 1) + (w & 1) * 64; }
  __device__ Pre preload(int r, int lane) const { return lane < kGemvMaxTokens ? Pre{bias[r], scale[r]} : Pre{0.f, 0.f}; }
  template <int NT>
  __device__ void row_done(int, int w, int lane, int, const Pre& p, const float (&v)[NT], float* rs, int nt) const {
#pragma unroll
    for (int t = 0; t < NT; ++t)
      if (lane == t && t < nt) rs[w * NT + t] = p.bias + p.scale * v[t];
  }
  __device__ void pair_done(int u, int w, int lane, int r, const float* rs, int nt) const {
    if (lane >= nt) return;
    constexpr int NTS = kGemvMaxTokens;
    (void)NTS;
    const int t = lane;
    const int h = r / kHeadDim;
    const int ntok = nt;
    (void)ntok;
    const float mine = rs[w * stride_ + t];
    const float other = rs[(w ^ 1) * stride_ + t];
    float y = mine;
    const int pos = tok.pos[t];
    if (h < kHeads + kKvHeads) {
      const int p = r % kHeadDim - (w & 1) * 64;
      const float c = cosv[(size_t)pos * 64 + p], s = sinv[(size_t)pos * 64 + p];
      y = (w & 1) == 0 ? __fsub_rn(__fmul_rn(mine, c), __fmul_rn(other, s))
                       : __fadd_rn(__fmul_rn(mine, c), __fmul_rn(other, s));
    }
    if (h < kHeads) {
      q_out[(size_t)t * kHidden + r] = y;
    } else {
      const int which = h < kHeads + kKvHeads ? 0 : 1;
      kv_row(kv, tok.seq[t], pos, which)[r - kHidden - which * kKvWidth] = y;
    }
    (void)u;
  }
  int stride_;  // tokens per row in the shared row buffer (= NT of the instantiation)
};

// y = scale * acc (o_proj: no bias, no residual, qwen_decode_attention_kernel.cpp:215).
struct EpiScale : EpiBase {
  static constexpr bool kPairs = false;
  struct Pre {
    float scale;
  };
  const float* scale;
  float* out;
  int n;  // output row length
  __device__ int row(int u, int w) const { return u * kRows + w; }
  __device__ Pre preload(int r, int lane) const { return lane < kGemvMaxTokens ? Pre{scale[r]} : Pre{0.f}; }
  template <int NT>
  __device__ void row_done(int, int, int lane, int r, const Pre& p, const float (&v)[NT], float*, int nt) const {
#pragma unroll
    for (int t = 0; t < NT; ++t)
      if (lane == t && t < nt) out[(size_t)t * n + r] = p.scale * v[t];
  }
  __device__ void pair_done(int, int, int, int, const float*, int) const {}
};

// h[j] = silu(gate[j]) * up[j] with silu(v) = v / (1 + expf(-v)) (qwen_decode_mlp_kernel.cpp:79-81,
// 113-115). Unit u covers j = 4u .. 4u+3: warp w holds gate row (w even) or up row (w odd) of j = 4u + w/2.
struct EpiGateUp : EpiBase {
  static constexpr bool kPairs = true;
  struct Pre {
    float scale;
  };
  const float* scale;  // gate | up scales
  float* h;
  int stride_;
  __device__ int row(int u, int w) const { return 4 * u + (w >> 1) + (w & 1) * kInter; }
  __device__ Pre preload(int r, int lane) const { return lane < kGemvMaxTokens ? Pre{scale[r]} : Pre{0.f}; }
  template <int NT>
  __device__ void row_done(int, int w, int lane, int, const Pre& p, const float (&v)[NT], float* rs, int nt) const {
#pragma unroll
    for (int t = 0; t < NT; ++t)
      if (lane == t && t < nt) rs[w * NT + t] = p.scale * v[t];
  }
  __device__ void pair_done(int u, int w, int lane, int, const float* rs, int nt) const {
    if ((w & 1) || lane >= nt) return;
    const int t = lane;
    const float gv = rs[w * stride_ + t];
    const float uv = rs[(w + 1) * stride_ + t];
    const float silu = __fdiv_rn(gv, __fadd_rn(1.0f, expf(-gv)));
    h[(size_t)t * kInter + 4 * u + (w >> 1)] = __fmul_rn(silu, uv);
  }
};

// out = a + scale * acc (qwen_decode_mlp_kernel.cpp:116-119), optionally rounded to bf16 for the next
// layer (the caller's rounding, verification/real_host_top_backend.py:334).
struct EpiDown : EpiBase {
  static constexpr bool kPairs = false;
  struct Pre {
    float scale, resid[kGemvMaxTokens];
  };
  const float* scale;
  const float* a;
  float* out;
  bool round_out;
  int nt_;
  __device__ int row(int u, int w) const { return u * kRows + w; }
  __device__ Pre preload(int r, int lane) const {
    Pre p{};
    if (lane < nt_) {
      p.scale = scale[r];
      p.resid[0] = a[(size_t)lane * kHidden + r];
    }
    return p;
  }
  template <int NT>
  __device__ void row_done(int, int, int lane, int r, const Pre& p, const float (&v)[NT], float*, int nt) const {
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      if (lane == t && t < nt) {
        float y = __fadd_rn(p.resid[0], p.scale * v[t]);
        if (round_out) y = round_bf16(y);
        out[(size_t)t * kHidden + r] = y;
      }
    }
  }
  __device__ void pair_done(int, int, int, int, const float*, int) const {}
};

// Greedy LM head: logits[v] = E[v] . y, argmax with the lowest index winning ties. Lane t of each warp keeps
// token t's best over the warp's rows; the CTA reduces them into `partial`, and the last CTA to finish
// reduces all CTAs.
struct EpiLm {
  static constexpr bool kPairs = false;
  struct Pre {};
  float* logits;  // optional
  float* partial; // [gridDim][kGemvMaxTokens][2]
  unsigned* counter;
  int* next_token;
  mutable float best_v;
  mutable int best_i;
  __device__ int row(int u, int w) const { return u * kRows + w; }
  __device__ Pre preload(int, int) const { return Pre{}; }
  template <int NT>
  __device__ void row_done(int, int, int lane, int r, const Pre&, const float (&v)[NT], float*, int nt) const {
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      if (lane == t && t < nt) {
        if (logits) logits[(size_t)t * kVocab + r] = v[t];
        if (v[t] > best_v || (v[t] == best_v && r < best_i)) {
          best_v = v[t];
          best_i = r;
        }
      }
    }
  }
  __device__ void pair_done(int, int, int, int, const float*, int) const {}
  __device__ void cta_end(int nt) const {
    __shared__ float sv[kRows][kGemvMaxTokens];
    __shared__ int si[kRows][kGemvMaxTokens];
    __shared__ bool last;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    if (lane < kGemvMaxTokens) {
      sv[warp][lane] = best_v;
      si[warp][lane] = best_i;
    }
    named_sync(kBarConsumers, kConsumers);
    if (threadIdx.x == 0) {
      for (int t = 0; t < nt; ++t) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int w = 0; w < kRows; ++w)
          if (sv[w][t] > bv || (sv[w][t] == bv && si[w][t] < bi)) {
            bv = sv[w][t];
            bi = si[w][t];
          }
        partial[((size_t)blockIdx.x * kGemvMaxTokens + t) * 2] = bv;
        partial[((size_t)blockIdx.x * kGemvMaxTokens + t) * 2 + 1] = __int_as_float(bi);
      }
      __threadfence();
      const unsigned prev = atomicAdd(counter, 1u);
      last = (prev == gridDim.x - 1);
    }
    named_sync(kBarConsumers, kConsumers);
    if (last && threadIdx.x == 0) {
      __threadfence();
      for (int t = 0; t < nt; ++t) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (unsigned b = 0; b < gridDim.x; ++b) {
          const float pv = __ldcg(&partial[((size_t)b * kGemvMaxTokens + t) * 2]);
          const int pi = __float_as_int(__ldcg(&partial[((size_t)b * kGemvMaxTokens + t) * 2 + 1]));
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

int num_sms() { return device_sm_count(); }

// Stage geometry: a row is split into column blocks of at most 4 KB so that a stage (8 rows) stays small;
// ring depth fills the shared-memory target (at least 2 stages).
void plan_stages(GemvArgs& a, int wbits, int nt_alloc) {
  const int row_bytes = a.K * wbits / 8;
  int nkb = 1;
  while (row_bytes / nkb > 4096 || (row_bytes % nkb) != 0 || ((row_bytes / nkb) % 16) != 0) ++nkb;
  a.nkb = nkb;
  a.kb_bytes = row_bytes / nkb;
  const int x_bytes = nt_alloc * a.K * 4;
  const int stage = kRows * a.kb_bytes;
  int ns = (kSmemTarget - 256 - x_bytes - 2 * kRows * nt_alloc * 4) / stage;
  if (ns < 2) ns = 2;
  if (ns > 8) ns = 8;
  a.nstages = ns;
}

template <int WBITS, int NT, int MODE, class Epi>
cudaError_t run_gemv(GemvArgs a, const Epi& epi, cudaStream_t s, bool pdl) {
  plan_stages(a, WBITS, NT);
  const size_t smem = 256 + (size_t)NT * a.K * 4 + (size_t)a.nstages * kRows * a.kb_bytes + 2 * kRows * NT * 4;
  auto kern = gemv_kernel<WBITS, NT, MODE, Epi>;
  if (cudaError_t e = ensure_smem_attr((const void*)kern, smem)) return e;
  const int grid = a.nunits < num_sms() ? a.nunits : num_sms();
  return launch_k(kern, dim3(grid), dim3(kThreads), smem, s, pdl, a, epi);
}

template <int MODE, class Epi, int NT>
cudaError_t dispatch_wbits(int wbits, const GemvArgs& a, Epi e, cudaStream_t s, bool pdl) {
  if (wbits == 8) return run_gemv<8, NT, MODE>(a, e, s, pdl);
  if (wbits == 4) return run_gemv<4, NT, MODE>(a, e, s, pdl);
  return cudaErrorInvalidValue;
}

template <int MODE, class Epi>
cudaError_t dispatch(int wbits, const GemvArgs& a, Epi e, cudaStream_t s, bool pdl) {
  switch (a.nt) {
    case 1: return dispatch_wbits<MODE, Epi, 1>(wbits, a, e, s, pdl);
    case 2: return dispatch_wbits<MODE, Epi, 2>(wbits, a, e, s, pdl);
    case 3:
    case 4: return dispatch_wbits<MODE, Epi, 4>(wbits, a, e, s, pdl);
    default: return cudaErrorInvalidValue;
  }
}

int nt_alloc(int nt) { return nt <= 2 ? nt : 4; }

}  // namespace

cudaError_t launch_decode_qkv(int wbits, const LayerDev& L, XSource src, DecodeTokens tok, const float* rope_cos,
                              const float* rope_sin, float* q_out, KvView kv, cudaStream_t s, bool pdl,
                              const void* pf, size_t pf_bytes) {
  GemvArgs a{};
  a.pf = static_cast<const uint8_t*>(pf);
  a.pf_bytes = pf_bytes;
  a.w = L.qkv_w;
  a.K = kHidden;
  a.nunits = kQkvRows / kRows;
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
  e.stride_ = nt_alloc(tok.nt);
  if (src.x == nullptr) return dispatch<kXEmbedNorm>(wbits, a, e, s, pdl);
  return dispatch<kXNorm>(wbits, a, e, s, pdl);
}

cudaError_t launch_decode_o(int wbits, const LayerDev& L, const float* ctx, int nt, float* out, cudaStream_t s,
                            bool pdl, const void* pf, size_t pf_bytes) {
  GemvArgs a{};
  a.pf = static_cast<const uint8_t*>(pf);
  a.pf_bytes = pf_bytes;
  a.w = L.o_w;
  a.K = kHidden;
  a.nunits = kHidden / kRows;
  a.nt = nt;
  a.x = ctx;
  EpiScale e;
  e.scale = L.o_s;
  e.out = out;
  e.n = kHidden;
  return dispatch<kXPlain>(wbits, a, e, s, pdl);
}

cudaError_t launch_decode_gateup(int wbits, const LayerDev& L, const float* x, int nt, float* h, cudaStream_t s,
                                 bool pdl, const void* pf, size_t pf_bytes) {
  GemvArgs a{};
  a.pf = static_cast<const uint8_t*>(pf);
  a.pf_bytes = pf_bytes;
  a.w = L.gu_w;
  a.K = kHidden;
  a.nunits = 2 * kInter / kRows;
  a.nt = nt;
  a.x = x;
  a.norm_w = L.post_ln;
  EpiGateUp e;
  e.scale = L.gu_s;
  e.h = h;
  e.stride_ = nt_alloc(nt);
  return dispatch<kXNorm>(wbits, a, e, s, pdl);
}

cudaError_t launch_decode_down(int wbits, const LayerDev& L, const float* h, const float* a_res, int nt, float* out,
                               bool round_out, cudaStream_t s, bool pdl, const void* pf, size_t pf_bytes) {
  GemvArgs a{};
  a.pf = static_cast<const uint8_t*>(pf);
  a.pf_bytes = pf_bytes;
  a.w = L.down_w;
  a.K = kInter;
  a.nunits = kHidden / kRows;
  a.nt = nt;
  a.x = h;
  EpiDown e;
  e.scale = L.down_s;
  e.a = a_res;
  e.out = out;
  e.round_out = round_out;
  e.nt_ = nt;
  return dispatch<kXPlain>(wbits, a, e, s, pdl);
}

namespace {
template <int NT>
cudaError_t run_lm(const GemvArgs& a, EpiLm e, cudaStream_t s, bool pdl) {
  e.best_v = -INFINITY;
  e.best_i = 0x7fffffff;
  return run_gemv<16, NT, kXNorm>(a, e, s, pdl);
}
}  // namespace

int lm_head_partial_floats() { return 1024 * kGemvMaxTokens * 2; }

cudaError_t launch_lm_head_argmax(const uint16_t* embed, const float* norm_w, const float* x, int nt, float* logits,
                                  float* partial, unsigned* counter, int* next_token, cudaStream_t s, bool pdl) {
  GemvArgs a{};
  a.w = reinterpret_cast<const uint8_t*>(embed);
  a.K = kHidden;
  a.nunits = kVocab / kRows;
  a.nt = nt;
  a.x = x;
  a.norm_w = norm_w;
  EpiLm e{logits, partial, counter, next_token, -INFINITY, 0x7fffffff};
  switch (nt) {
    case 1: return run_lm<1>(a, e, s, pdl);
    case 2: return run_lm<2>(a, e, s, pdl);
    case 3:
    case 4: return run_lm<4>(a, e, s, pdl);
    default: return cudaErrorInvalidValue;
  }
}

unsigned gemv_kernel_error(bool reset) {
  unsigned v = 0;
  if (cudaMemcpyFromSymbol(&v, g_kernel_error, sizeof(v)) != cudaSuccess) return 0xFFFFFFFFu;
  if (reset && v) {
    const unsigned z = 0;
    cudaMemcpyToSymbol(g_kernel_error, &z, sizeof(z));
  }
  return v;
}

}  // namespace qb
