// Reference-order ("exact") kernels: see exact.h. One thread per output, serial sums in the reference's
// order, every product and sum rounded on its own (explicit _rn intrinsics, so nvcc cannot contract them).
#include "exact.h"

#include <cuda_fp16.h>

#include "exact_expf.cuh"

namespace qb {
namespace exact {
namespace {

// ------------------------------------------------------------------------------------------------
// kernels
// ------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) rmsnorm_dec_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                          float* __restrict__ out) {
  __shared__ float xs[kHidden];
  __shared__ double inv_s;
  const float* xr = x + (size_t)blockIdx.x * kHidden;
  for (int d = threadIdx.x; d < kHidden; d += blockDim.x) xs[d] = xr[d];
  __syncthreads();
  if (threadIdx.x == 0) {
    double ms = 0.0;
    for (int d = 0; d < kHidden; ++d) {
      const double v = (double)xs[d];
      ms = __dadd_rn(ms, __dmul_rn(v, v));
    }
    ms = __ddiv_rn(ms, (double)kHidden);
    inv_s = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(ms, (double)kEps)));
  }
  __syncthreads();
  const double inv = inv_s;
  for (int d = threadIdx.x; d < kHidden; d += blockDim.x)
    out[(size_t)blockIdx.x * kHidden + d] = __double2float_rn(__dmul_rn(__dmul_rn((double)xs[d], inv), (double)w[d]));
}

template <int WBITS>
__device__ __forceinline__ int code_of(const uint32_t (&words)[4], int j) {
  if (WBITS == 8) return (int)(int8_t)((words[j >> 2] >> (8 * (j & 3))) & 0xffu);
  const int nib = (int)((words[j >> 3] >> (4 * (j & 7))) & 0xfu);  // even flat index = low nibble
  return nib >= 8 ? nib - 16 : nib;
}

// grid (ceil(rows / 128), n), 128 threads, k floats of dynamic shared memory (the token's input row)
template <int WBITS>
__global__ void __launch_bounds__(128) project_kernel(const float* __restrict__ x, int k, const uint8_t* __restrict__ w,
                                                      const float* __restrict__ bias, const float* __restrict__ scale,
                                                      int rows, float* __restrict__ y, const float* __restrict__ resid,
                                                      int round_out) {
  extern __shared__ float xs[];
  const int t = blockIdx.y;
  for (int i = threadIdx.x; i < k; i += blockDim.x) xs[i] = x[(size_t)t * k + i];
  __syncthreads();
  const int o = blockIdx.x * blockDim.x + threadIdx.x;
  if (o >= rows) return;
  const float sc = scale[o];
  float acc = bias ? bias[o] : 0.0f;
  constexpr int kPer = 128 / WBITS;  // codes per 16-byte chunk
  const uint4* wr = reinterpret_cast<const uint4*>(w + (size_t)o * ((size_t)k * WBITS / 8));
  const int chunks = k / kPer;
  for (int c = 0; c < chunks; ++c) {
    const uint4 v = __ldg(wr + c);
    const uint32_t words[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const float wv = __fmul_rn((float)code_of<WBITS>(words, j), sc);
      acc = __fadd_rn(acc, __fmul_rn(xs[c * kPer + j], wv));
    }
  }
  float out = acc;
  if (resid) out = __fadd_rn(resid[(size_t)t * rows + o], acc);
  if (round_out) out = round_bf16(out);
  y[(size_t)t * rows + o] = out;
}

// grid n, 256 threads
__global__ void __launch_bounds__(256) rope_store_kernel(const float* __restrict__ qkv, const int* __restrict__ pos,
                                                         int pos_base, const float* __restrict__ cos_tab,
                                                         const float* __restrict__ sin_tab, float* __restrict__ q_out,
                                                         KvView kv, const int* __restrict__ seq, int seq_const) {
  const int t = blockIdx.x;
  const int p = pos ? pos[t] : pos_base + t;
  const int slot = seq ? seq[t] : seq_const;
  const float* row = qkv + (size_t)t * kQkvRows;
  float* krow = kv_row(kv, slot, p, 0);
  float* vrow = kv_row(kv, slot, p, 1);
  for (int i = threadIdx.x; i < (kHeads + kKvHeads) * 64; i += blockDim.x) {
    const int head = i >> 6, pair = i & 63;
    const float c = cos_tab[(size_t)p * 64 + pair], sn = sin_tab[(size_t)p * 64 + pair];
    const float even = row[head * kHeadDim + pair], odd = row[head * kHeadDim + pair + 64];
    const float re = __fsub_rn(__fmul_rn(even, c), __fmul_rn(odd, sn));
    const float ro = __fadd_rn(__fmul_rn(odd, c), __fmul_rn(even, sn));
    if (head < kHeads) {
      q_out[(size_t)t * kHidden + head * kHeadDim + pair] = re;
      q_out[(size_t)t * kHidden + head * kHeadDim + pair + 64] = ro;
    } else {
      const int kh = head - kHeads;
      krow[kh * kHeadDim + pair] = re;
      krow[kh * kHeadDim + pair + 64] = ro;
    }
  }
  for (int i = threadIdx.x; i < kKvWidth; i += blockDim.x) vrow[i] = row[kHidden + kKvWidth + i];
}

// Two-pass attention of one (query token, head), 256 threads: pass 1 max of score * scaling over the keys
// (threads own keys, max is exact in any order), pass 2 over blocks of 256 keys: the threads form the
// weights of one block in parallel, then thread d < 128 adds e_j * v_j[d] and thread 128 adds e_j in key
// order.
constexpr int kAttnThreads = 256;

template <bool kPrefill>
__device__ __forceinline__ void attention_one(const float* __restrict__ qh, const KvView& kv, int slot, int total,
                                              float scaling, float* __restrict__ ctx_out, int kvh) {
  __shared__ float qs[kHeadDim];
  __shared__ float es[kAttnThreads];
  __shared__ float red[kAttnThreads / 32];
  __shared__ float inv_s;
  const int tid = threadIdx.x;
  if (tid < kHeadDim) qs[tid] = qh[tid];
  __syncthreads();
  auto score = [&](int j) {
    const float* kr = kv_row(kv, slot, j, 0) + kvh * kHeadDim;
    float s = 0.0f;
    for (int d = 0; d < kHeadDim; ++d) s = __fadd_rn(s, __fmul_rn(qs[d], kr[d]));
    return __fmul_rn(s, scaling);
  };
  float m = -1.0e30f;
  for (int j = tid; j < total; j += kAttnThreads) {
    const float ss = score(j);
    m = (m < ss) ? ss : m;
  }
  for (int off = 16; off > 0; off >>= 1) {
    const float o = __shfl_xor_sync(0xffffffffu, m, off);
    m = (m < o) ? o : m;
  }
  if ((tid & 31) == 0) red[tid >> 5] = m;
  __syncthreads();
  m = red[0];
  for (int i = 1; i < kAttnThreads / 32; ++i) m = (m < red[i]) ? red[i] : m;
  float acc = 0.0f, denom = 0.0f;
  for (int base = 0; base < total; base += kAttnThreads) {
    __syncthreads();  // es of the previous block consumed
    const int j = base + tid;
    if (j < total) {
      const float arg = __fsub_rn(score(j), m);
      es[tid] = kPrefill ? approx_exp(arg) : exact_expf(arg);
    }
    __syncthreads();
    const int cnt = min(kAttnThreads, total - base);
    if (tid < kHeadDim) {
      for (int jj = 0; jj < cnt; ++jj) {
        const float* vr = kv_row(kv, slot, base + jj, 1) + kvh * kHeadDim;
        acc = __fadd_rn(acc, __fmul_rn(es[jj], vr[tid]));
      }
    } else if (tid == kHeadDim) {
      for (int jj = 0; jj < cnt; ++jj) denom = __fadd_rn(denom, es[jj]);
    }
  }
  if (tid == kHeadDim) inv_s = denom > 0.0f ? __fdiv_rn(1.0f, denom) : 0.0f;
  __syncthreads();
  if (tid < kHeadDim) ctx_out[tid] = __fmul_rn(acc, inv_s);
}

// grid (n, 12)
__global__ void __launch_bounds__(kAttnThreads) attn_dec_kernel(const float* __restrict__ q, KvView kv,
                                                                const int* __restrict__ pos,
                                                                const int* __restrict__ seq, float scaling,
                                                                float* __restrict__ ctx) {
  const int t = blockIdx.x, h = blockIdx.y;
  attention_one<false>(q + (size_t)t * kHidden + h * kHeadDim, kv, seq[t], pos[t] + 1, scaling,
                       ctx + (size_t)t * kHidden + h * kHeadDim, h / kGroups);
}

// grid (S, 12): query t at position q0 + t over keys 0 .. q0 + t
__global__ void __launch_bounds__(kAttnThreads) attn_pre_kernel(const float* __restrict__ q, KvView kv, int q0,
                                                                float* __restrict__ ctx) {
  const int t = blockIdx.x, h = blockIdx.y;
  attention_one<true>(q + (size_t)t * kHidden + h * kHeadDim, kv, 0, q0 + t + 1, kAttentionScaling,
                      ctx + (size_t)t * kHidden + h * kHeadDim, h / kGroups);
}

__global__ void silu_mul_kernel(const float* __restrict__ gu, int n, int prefill, float* __restrict__ h) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (size_t)n * kInter) return;
  const size_t t = i / kInter, c = i % kInter;
  const float g = gu[t * 2 * kInter + c], u = gu[t * 2 * kInter + kInter + c];
  const float e = prefill ? approx_exp(-g) : exact_expf(-g);
  h[i] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, e)), u);
}

// grid (ceil(vocab / 128), n), 128 threads
__global__ void __launch_bounds__(128) logits_kernel(const uint16_t* __restrict__ embed, const float* __restrict__ y,
                                                     float* __restrict__ logits) {
  __shared__ float ys[kHidden];
  const int t = blockIdx.y;
  for (int d = threadIdx.x; d < kHidden; d += blockDim.x) ys[d] = y[(size_t)t * kHidden + d];
  __syncthreads();
  const int v = blockIdx.x * blockDim.x + threadIdx.x;
  if (v >= kVocab) return;
  const uint4* row = reinterpret_cast<const uint4*>(embed + (size_t)v * kHidden);
  float acc = 0.0f;
  for (int c = 0; c < kHidden / 8; ++c) {
    const uint4 u = __ldg(row + c);
    const uint32_t words[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const __half hv = __ushort_as_half((unsigned short)((words[j >> 1] >> (16 * (j & 1))) & 0xffffu));
      acc = __fadd_rn(acc, __fmul_rn(__half2float(hv), ys[c * 8 + j]));
    }
  }
  logits[(size_t)t * kVocab + v] = acc;
}

// grid n, 1024 threads: first index of the largest logit
__global__ void __launch_bounds__(1024) argmax_kernel(const float* __restrict__ logits, int* __restrict__ next) {
  __shared__ float bv[32];
  __shared__ int bi[32];
  const float* lg = logits + (size_t)blockIdx.x * kVocab;
  float best = -__int_as_float(0x7f800000);
  int idx = 0x7fffffff;
  for (int v = threadIdx.x; v < kVocab; v += blockDim.x) {
    const float x = lg[v];
    if (x > best) {  // strict: the first (lowest) index of this thread's maximum is kept
      best = x;
      idx = v;
    }
  }
  auto better = [](float a, int ia, float b, int ib) { return b > a || (b == a && ib < ia); };
  for (int off = 16; off > 0; off >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, off);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, off);
    if (better(best, idx, ob, oi)) {
      best = ob;
      idx = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    bv[threadIdx.x >> 5] = best;
    bi[threadIdx.x >> 5] = idx;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < 32; ++w)
      if (better(best, idx, bv[w], bi[w])) {
        best = bv[w];
        idx = bi[w];
      }
    next[blockIdx.x] = idx == 0x7fffffff ? 0 : idx;
  }
}

__global__ void expf_kernel(const float* __restrict__ x, float* __restrict__ y, long long n) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    y[i] = exact_expf(x[i]);
}

}  // namespace

cudaError_t launch_rmsnorm_dec(const float* x, const float* w, int n, float* out, cudaStream_t s) {
  rmsnorm_dec_kernel<<<n, 256, 0, s>>>(x, w, out);
  return cudaGetLastError();
}

cudaError_t launch_project(int wbits, const float* x, int n, int k, const uint8_t* w, const float* bias,
                           const float* scale, int rows, float* y, const float* resid, bool round_out,
                           cudaStream_t s) {
  if ((wbits != 4 && wbits != 8) || n <= 0 || k % 32 != 0 || (reinterpret_cast<uintptr_t>(w) & 15) != 0)
    return cudaErrorInvalidValue;
  const dim3 grid((rows + 127) / 128, n);
  const size_t smem = (size_t)k * 4;  // at most 8960 floats: within the default 48 KB
  if (wbits == 8) {
    project_kernel<8><<<grid, 128, smem, s>>>(x, k, w, bias, scale, rows, y, resid, round_out ? 1 : 0);
  } else {
    project_kernel<4><<<grid, 128, smem, s>>>(x, k, w, bias, scale, rows, y, resid, round_out ? 1 : 0);
  }
  return cudaGetLastError();
}

cudaError_t launch_rope_store(const float* qkv, int n, const int* pos, int pos_base, const float* cos_tab,
                              const float* sin_tab, float* q_out, KvView kv, const int* seq, int seq_const,
                              cudaStream_t s) {
  rope_store_kernel<<<n, 256, 0, s>>>(qkv, pos, pos_base, cos_tab, sin_tab, q_out, kv, seq, seq_const);
  return cudaGetLastError();
}

cudaError_t launch_attention_dec(const float* q, KvView kv, const int* pos, const int* seq, int n, float scaling,
                                 float* ctx, cudaStream_t s) {
  attn_dec_kernel<<<dim3(n, kHeads), kAttnThreads, 0, s>>>(q, kv, pos, seq, scaling, ctx);
  return cudaGetLastError();
}

cudaError_t launch_attention_pre(const float* q, const float* k, const float* v, int S, float* ctx,
                                 cudaStream_t s, int q0) {
  KvView kv{};
  kv.k = const_cast<float*>(k);
  kv.v = const_cast<float*>(v);
  kv.page_table = nullptr;
  attn_pre_kernel<<<dim3(S, kHeads), kAttnThreads, 0, s>>>(q, kv, q0, ctx);
  return cudaGetLastError();
}

cudaError_t launch_silu_mul(const float* gu, int n, bool prefill, float* h, cudaStream_t s) {
  const size_t total = (size_t)n * kInter;
  silu_mul_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(gu, n, prefill ? 1 : 0, h);
  return cudaGetLastError();
}

cudaError_t launch_lm_head(const uint16_t* embed, const float* norm_w, const float* x, int n, float* y,
                           float* logits, int* next, cudaStream_t s) {
  rmsnorm_dec_kernel<<<n, 256, 0, s>>>(x, norm_w, y);
  logits_kernel<<<dim3((kVocab + 127) / 128, n), 128, 0, s>>>(embed, y, logits);
  argmax_kernel<<<n, 1024, 0, s>>>(logits, next);
  return cudaGetLastError();
}

cudaError_t launch_expf(const float* x, float* y, long long n, cudaStream_t s) {
  expf_kernel<<<148 * 8, 256, 0, s>>>(x, y, n);
  return cudaGetLastError();
}

}  // namespace exact
}  // namespace qb
