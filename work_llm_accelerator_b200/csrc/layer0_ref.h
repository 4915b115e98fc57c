// Kernels of the fp32-weight "layer0 reference" layers (layer0_ref.cu): the reference's golden decoder layer
// with unquantised weights, double accumulation and bf16 rounding after every linear and norm
// (hls/decode_only/qwen_decode_layer0_reference_wrapper.cpp:75-209,
// hls/prefill_only/qwen_prefill_layer0_reference_wrapper.cpp:60-255). Internal to libqwen_b200.so.
#pragma once

#include <cuda_runtime.h>

namespace qb {
namespace l0 {

// out[t] = RMSNorm of x[t], bf16-rounded. decode_form: double sums, out = bf16(float(x * inv * w));
// otherwise (prefill): fp32 serial sums, inv = 1 / sqrtf(ms / 1536 + eps), out = bf16(bf16(x * inv) * w).
cudaError_t rmsnorm(const float* x, const float* w, int n, float eps, bool decode_form, float* out, cudaStream_t s);

// y[t][o] = bf16(float(bias[o] + sum_i double(x[t][i]) * double(w[o][i]))), the sum serial over i; bias optional.
// x [n][k], w [rows][k] fp32, y [n][rows].
cudaError_t linear(const float* x, int n, int k, const float* w, const float* bias, int rows, float* y,
                   cudaStream_t s);

// Rotate-half RoPE of q [n][1536] and k [n][256] in place at positions pos0 + t, with the table
// cos/sin[pos][64] = float(cos/sin(pos * 1e6^(-2 i / 128))) (double angle). prefill_form rounds the table
// values, each product and each result to bf16.
cudaError_t rope(float* q, float* k, int n, int pos0, const float* cos_tab, const float* sin_tab, bool prefill_form,
                 cudaStream_t s);

// Causal attention in double: query t (global position q0 + t) over keys 0 .. q0 + t; scores = double dot *
// scaling, probs = exp(score - max), context = sum_j (probs_j / sum) * v_j (each sum serial in key order),
// stored as float. Key j, dim d of KV head h at base + h * head_stride + j * row_stride + d (K and V alike).
cudaError_t attention(const float* q, int n, int q0, const float* k, const float* v, long long head_stride,
                      long long row_stride, float* ctx, cudaStream_t s);

// y = a + b elementwise (fp32), n floats.
cudaError_t add(const float* a, const float* b, long long n, float* y, cudaStream_t s);

// h = silu(g) * u with silu(v) = v / (1 + expf(-v)) (the host C library's expf), n floats.
cudaError_t silu_mul(const float* g, const float* u, long long n, float* h, cudaStream_t s);

// dst[h][j][d] = (round ? bf16 : identity)(src[j][h * 128 + d]) for j < n: token-major K/V rows to the
// head-major cache layout [2][n][128] of the layer0 entry points.
cudaError_t to_head_major(const float* src, int n, bool round, float* dst, cudaStream_t s);

}  // namespace l0
}  // namespace qb
