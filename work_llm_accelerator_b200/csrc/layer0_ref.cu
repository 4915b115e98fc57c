// Kernels of the fp32-weight "layer0 reference" layers (see layer0_ref.h). Each output is one thread's serial
// sum in the reference's order; every operation is an explicit _rn intrinsic, so nothing is contracted into an
// FMA (the reference's x86-64 -O2 build has none).
#include "layer0_ref.h"

#include <cmath>

#include "exact_expf.cuh"
#include "qwen_common.cuh"

namespace qb {
namespace l0 {
namespace {

__global__ void __launch_bounds__(256) rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w, float eps,
                                                      int decode_form, float* __restrict__ out) {
  __shared__ float xs[kHidden];
  __shared__ double inv_d;
  __shared__ float inv_f;
  const float* xr = x + (size_t)blockIdx.x * kHidden;
  for (int d = threadIdx.x; d < kHidden; d += blockDim.x) xs[d] = xr[d];
  __syncthreads();
  if (threadIdx.x == 0) {
    if (decode_form) {  // qwen_decode_layer0_reference_wrapper.cpp:25-36
      double ms = 0.0;
      for (int d = 0; d < kHidden; ++d) ms = __dadd_rn(ms, __dmul_rn((double)xs[d], (double)xs[d]));
      ms = __ddiv_rn(ms, (double)kHidden);
      inv_d = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(ms, (double)eps)));
    } else {  // qwen_prefill_layer0_reference_wrapper.cpp:25-37
      float ms = 0.0f;
      for (int d = 0; d < kHidden; ++d) ms = __fadd_rn(ms, __fmul_rn(xs[d], xs[d]));
      ms = __fdiv_rn(ms, (float)kHidden);
      inv_f = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, eps)));
    }
  }
  __syncthreads();
  for (int d = threadIdx.x; d < kHidden; d += blockDim.x) {
    float o;
    if (decode_form) {
      o = round_bf16(__double2float_rn(__dmul_rn(__dmul_rn((double)xs[d], inv_d), (double)w[d])));
    } else {
      const float nb = round_bf16(__fmul_rn(xs[d], inv_f));
      o = round_bf16(__fmul_rn(nb, w[d]));
    }
    out[(size_t)blockIdx.x * kHidden + d] = o;
  }
}

// grid (ceil(rows / 128), n), 128 threads, k floats of dynamic shared memory
__global__ void __launch_bounds__(128) linear_kernel(const float* __restrict__ x, int k, const float* __restrict__ w,
                                                     const float* __restrict__ bias, int rows, float* __restrict__ y) {
  extern __shared__ float xs[];
  const int t = blockIdx.y;
  for (int i = threadIdx.x; i < k; i += blockDim.x) xs[i] = x[(size_t)t * k + i];
  __syncthreads();
  const int o = blockIdx.x * blockDim.x + threadIdx.x;
  if (o >= rows) return;
  double acc = bias ? (double)bias[o] : 0.0;
  const float4* wr = reinterpret_cast<const float4*>(w + (size_t)o * k);
  for (int c = 0; c < k / 4; ++c) {
    const float4 v = __ldg(wr + c);
    acc = __dadd_rn(acc, __dmul_rn((double)xs[4 * c], (double)v.x));
    acc = __dadd_rn(acc, __dmul_rn((double)xs[4 * c + 1], (double)v.y));
    acc = __dadd_rn(acc, __dmul_rn((double)xs[4 * c + 2], (double)v.z));
    acc = __dadd_rn(acc, __dmul_rn((double)xs[4 * c + 3], (double)v.w));
  }
  y[(size_t)t * rows + o] = round_bf16(__double2float_rn(acc));
}

// grid n, 256 threads: 12 query heads and 2 key heads x 64 pairs
__global__ void rope_kernel(float* __restrict__ q, float* __restrict__ k, int pos0, const float* __restrict__ cos_tab,
                            const float* __restrict__ sin_tab, int prefill_form) {
  const int t = blockIdx.x, p = pos0 + t;
  for (int i = threadIdx.x; i < (kHeads + kKvHeads) * 64; i += blockDim.x) {
    const int head = i >> 6, pair = i & 63;
    float* hd = head < kHeads ? q + (size_t)t * kHidden + head * kHeadDim
                              : k + (size_t)t * kKvWidth + (head - kHeads) * kHeadDim;
    float c = cos_tab[(size_t)p * 64 + pair], sn = sin_tab[(size_t)p * 64 + pair];
    const float even = hd[pair], odd = hd[pair + 64];
    if (prefill_form) {  // qwen_prefill_layer0_reference_wrapper.cpp:124-139
      c = round_bf16(c);
      sn = round_bf16(sn);
      const float ec = round_bf16(__fmul_rn(even, c)), os = round_bf16(__fmul_rn(odd, sn));
      const float oc = round_bf16(__fmul_rn(odd, c)), es = round_bf16(__fmul_rn(even, sn));
      hd[pair] = round_bf16(__fsub_rn(ec, os));
      hd[pair + 64] = round_bf16(__fadd_rn(oc, es));
    } else {  // qwen_decode_layer0_reference_wrapper.cpp:59-72
      hd[pair] = __fsub_rn(__fmul_rn(even, c), __fmul_rn(odd, sn));
      hd[pair + 64] = __fadd_rn(__fmul_rn(odd, c), __fmul_rn(even, sn));
    }
  }
}

constexpr int kAttnThreads = 128;

// grid (n, 12), 128 threads. Three passes over the keys in blocks of 128 (scores recomputed in each): the max,
// the serial sum of exp(score - max), and the serial context sums with weights probs / sum.
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(const float* __restrict__ q, int q0,
                                                                 const float* __restrict__ kb,
                                                                 const float* __restrict__ vb, long long head_stride,
                                                                 long long row_stride, double scaling,
                                                                 float* __restrict__ ctx) {
  __shared__ float qs[kHeadDim];
  __shared__ double ps[kAttnThreads];
  __shared__ double red[kAttnThreads / 32];
  __shared__ double sum_s;
  const int t = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
  const int kvh = h / kGroups;
  const int total = q0 + t + 1;
  const float* kh = kb + (size_t)kvh * head_stride;
  const float* vh = vb + (size_t)kvh * head_stride;
  qs[tid] = q[(size_t)t * kHidden + h * kHeadDim + tid];
  __syncthreads();
  auto score = [&](int j) {
    const float* kr = kh + (size_t)j * row_stride;
    double dot = 0.0;
    for (int d = 0; d < kHeadDim; ++d) dot = __dadd_rn(dot, __dmul_rn((double)qs[d], (double)kr[d]));
    return __dmul_rn(dot, scaling);
  };
  double m = -1.0e300;
  for (int j = tid; j < total; j += kAttnThreads) {
    const double s = score(j);
    m = (m < s) ? s : m;
  }
  for (int off = 16; off > 0; off >>= 1) {
    const double o = __shfl_xor_sync(0xffffffffu, m, off);
    m = (m < o) ? o : m;
  }
  if ((tid & 31) == 0) red[tid >> 5] = m;
  __syncthreads();
  m = red[0];
  for (int i = 1; i < kAttnThreads / 32; ++i) m = (m < red[i]) ? red[i] : m;
  // pass 2: sum of the probabilities in key order
  double sum = 0.0;
  for (int base = 0; base < total; base += kAttnThreads) {
    __syncthreads();
    if (base + tid < total) ps[tid] = exp(__dsub_rn(score(base + tid), m));
    __syncthreads();
    if (tid == 0) {
      const int cnt = min(kAttnThreads, total - base);
      for (int jj = 0; jj < cnt; ++jj) sum = __dadd_rn(sum, ps[jj]);
    }
  }
  if (tid == 0) sum_s = sum;
  __syncthreads();
  sum = sum_s;
  // pass 3: context, thread = dim
  double acc = 0.0;
  for (int base = 0; base < total; base += kAttnThreads) {
    __syncthreads();
    if (base + tid < total) ps[tid] = __ddiv_rn(exp(__dsub_rn(score(base + tid), m)), sum);
    __syncthreads();
    const int cnt = min(kAttnThreads, total - base);
    for (int jj = 0; jj < cnt; ++jj)
      acc = __dadd_rn(acc, __dmul_rn(ps[jj], (double)vh[(size_t)(base + jj) * row_stride + tid]));
  }
  ctx[(size_t)t * kHidden + h * kHeadDim + tid] = __double2float_rn(acc);
}

__global__ void add_kernel(const float* __restrict__ a, const float* __restrict__ b, long long n, float* __restrict__ y) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) y[i] = __fadd_rn(a[i], b[i]);
}

__global__ void silu_mul_kernel(const float* __restrict__ g, const float* __restrict__ u, long long n,
                                float* __restrict__ h) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) h[i] = __fmul_rn(__fdiv_rn(g[i], __fadd_rn(1.0f, exact_expf(-g[i]))), u[i]);
}

__global__ void head_major_kernel(const float* __restrict__ src, int n, int round, float* __restrict__ dst) {
  const int j = blockIdx.x;
  for (int i = threadIdx.x; i < kKvWidth; i += blockDim.x) {
    const int hh = i >> 7, d = i & 127;
    const float v = src[(size_t)j * kKvWidth + i];
    dst[((size_t)hh * n + j) * kHeadDim + d] = round ? round_bf16(v) : v;
  }
}

}  // namespace

cudaError_t rmsnorm(const float* x, const float* w, int n, float eps, bool decode_form, float* out, cudaStream_t s) {
  rmsnorm_kernel<<<n, 256, 0, s>>>(x, w, eps, decode_form ? 1 : 0, out);
  return cudaGetLastError();
}

cudaError_t linear(const float* x, int n, int k, const float* w, const float* bias, int rows, float* y,
                   cudaStream_t s) {
  if (k % 4 != 0 || (reinterpret_cast<uintptr_t>(w) & 15) != 0) return cudaErrorInvalidValue;
  linear_kernel<<<dim3((rows + 127) / 128, n), 128, (size_t)k * 4, s>>>(x, k, w, bias, rows, y);
  return cudaGetLastError();
}

cudaError_t rope(float* q, float* k, int n, int pos0, const float* cos_tab, const float* sin_tab, bool prefill_form,
                 cudaStream_t s) {
  rope_kernel<<<n, 256, 0, s>>>(q, k, pos0, cos_tab, sin_tab, prefill_form ? 1 : 0);
  return cudaGetLastError();
}

cudaError_t attention(const float* q, int n, int q0, const float* k, const float* v, long long head_stride,
                      long long row_stride, float* ctx, cudaStream_t s) {
  const double scaling = (double)(float)(1.0 / std::sqrt((double)kHeadDim));
  attention_kernel<<<dim3(n, kHeads), kAttnThreads, 0, s>>>(q, q0, k, v, head_stride, row_stride, scaling, ctx);
  return cudaGetLastError();
}

cudaError_t add(const float* a, const float* b, long long n, float* y, cudaStream_t s) {
  add_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(a, b, n, y);
  return cudaGetLastError();
}

cudaError_t silu_mul(const float* g, const float* u, long long n, float* h, cudaStream_t s) {
  silu_mul_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(g, u, n, h);
  return cudaGetLastError();
}

cudaError_t to_head_major(const float* src, int n, bool round, float* dst, cudaStream_t s) {
  head_major_kernel<<<n, 256, 0, s>>>(src, n, round ? 1 : 0, dst);
  return cudaGetLastError();
}

}  // namespace l0
}  // namespace qb
