// Reference-order ("exact") kernels: the reference host code's arithmetic, operation for operation, for
// validating greedy-token identity with the reference host libraries. Internal to libqwen_b200.so.
//
// Every fp32 sum runs serially in the reference's order (one thread per output), products and sums are
// rounded separately (no FMA), the decode RMSNorm sums in double, and the decode softmax and SiLU use
// glibc's expf restated (exact_expf below). These kernels trade speed for bit-identity: they are the
// engine's "exact" option, not its throughput path.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "qwen_common.cuh"

namespace qb {
namespace exact {

// out[t] = decode RMSNorm of x[t] (qwen_decode_attention_kernel.cpp:13-27): serial double sum of squares,
// 1 / sqrt(ms / 1536 + eps) in double, out = float((x * inv) * w). x, out [n][1536].
cudaError_t launch_rmsnorm_dec(const float* x, const float* w, int n, float* out, cudaStream_t s);

// y[t][o] = resid[t][o] + ((bias ? bias[o] : 0) + sum_i x[t][i] * (float(code(o, i)) * scale[o])), the sum
// serial over i = 0..k-1 (qwen_decode_attention_kernel.cpp:62-98, qwen_prefill_attention_kernel.cpp:163-202);
// resid optional; round_out rounds the result to bf16 (RNE). w is [rows][k] codes of `wbits` (4: two per
// byte, low nibble first; 8: int8), 16-byte aligned rows. x [n][k], y and resid [n][rows].
cudaError_t launch_project(int wbits, const float* x, int n, int k, const uint8_t* w, const float* bias,
                           const float* scale, int rows, float* y, const float* resid, bool round_out,
                           cudaStream_t s);

// RoPE and cache write of n tokens from q|k|v rows [n][2048]: the 12 query heads and 2 key heads rotated
// (pairs (i, i + 64), products and sums rounded separately) with the table row of each token's position
// (pos[t], or pos_base + t when pos is null), q written to q_out [n][1536], the rotated K row and the V row
// stored at that position through kv (sequence seq[t], or seq_const when seq is null).
cudaError_t launch_rope_store(const float* qkv, int n, const int* pos, int pos_base, const float* cos_tab,
                              const float* sin_tab, float* q_out, KvView kv, const int* seq, int seq_const,
                              cudaStream_t s);

// Decode attention context (qwen_decode_attention_kernel.cpp:113-162) of n tokens, token t over the
// pos[t] + 1 cached keys of sequence seq[t]: two passes, serial dot products, exact_expf, serial
// denominator and context sums, context = acc * (1 / denom). q, ctx [n][1536].
cudaError_t launch_attention_dec(const float* q, KvView kv, const int* pos, const int* seq, int n, float scaling,
                                 float* ctx, cudaStream_t s);

// Causal prefill attention context (qwen_prefill_attention_kernel.cpp:204-289) of S queries at positions
// q0 .. q0 + S - 1 over the flat K/V rows [q0 + S][256]: the same two passes with approx_exp. q, ctx [S][1536].
cudaError_t launch_attention_pre(const float* q, const float* k, const float* v, int S, float* ctx,
                                 cudaStream_t s, int q0 = 0);

// h[t][i] = silu(g) * u with g = gu[t][i], u = gu[t][8960 + i], silu(v) = v / (1 + exp(-v)): exact_expf
// (decode, qwen_decode_mlp_kernel.cpp:79-81) or approx_exp (prefill, qwen_prefill_mlp_kernel.cpp:256-258).
cudaError_t launch_silu_mul(const float* gu, int n, bool prefill, float* h, cudaStream_t s);

// Final decode RMSNorm of x [n][1536] into y, logits[t][v] = serial sum_d float(E[v][d]) * y[t][d], and
// next[t] = the first index of the largest logit (NaN logits never win). y [n][1536], logits [n][151936].
cudaError_t launch_lm_head(const uint16_t* embed, const float* norm_w, const float* x, int n, float* y,
                           float* logits, int* next, cudaStream_t s);

// y[i] = exact_expf(x[i]), exposed so that its identity with the host C library can be checked.
cudaError_t launch_expf(const float* x, float* y, long long n, cudaStream_t s);

}  // namespace exact
}  // namespace qb
