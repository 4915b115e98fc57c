/*
 * Device-pointer operator API of libqwen_b200.so: single hot-path kernels on buffers the caller already
 * holds in GPU memory, enqueued on the caller's stream (no host staging, no synchronisation).
 * Status codes: 0 ok, 1 invalid argument (message in qwen_b200_last_error()), 30 CUDA failure.
 */
#ifndef QWEN_B200_OPS_H
#define QWEN_B200_OPS_H

#ifdef __cplusplus
extern "C" {
#endif

/* Decode attention context for one token: 12 query heads over 2 KV heads, head_dim 128 (replaces the
 * reference's decode_attention_context, hls/decode_only/qwen_decode_attention_kernel.cpp:113-162).
 *   q        [1536] fp32, the token's post-RoPE query (device memory)
 *   k_cache  [seq_len][256] fp32 token-major keys (device memory), the token's own row included
 *   v_cache  [seq_len][256] fp32 token-major values (device memory)
 *   context  [1536] fp32 output (device memory)
 *   stream   cudaStream_t (NULL = legacy default stream)
 * The split-history scratch is allocated by the library on a device's first call and grown when a
 * longer history arrives; calls on one device share it, so calls that overlap on the GPU race. */
int qwen_b200_decode_attention(const float* q, const float* k_cache, const float* v_cache, int seq_len,
                               float* context, void* stream);

/* Same computation and arguments as qwen_b200_decode_attention, for callers that cannot allocate device
 * memory at the point where they run attention -- e.g. a serving runtime that reserves all GPU memory in
 * its own pool at start-up, or a latency-critical loop where cudaMalloc/cudaFree would synchronise the
 * device. No counterpart in the reference (its host library has no device memory at all). It allocates
 * nothing: its scratch is a fixed array compiled into the library (about 0.8 MB, held on every GPU that
 * loads the library until the process exits), so seq_len is limited to 8192 (status 1 above it). The
 * first call on a device looks up that array's address and should come before any stream capture. All
 * calls on a device share the array (each call clears the parts that must start at zero), so calls that
 * overlap on the GPU race. */
int qwen_b200_decode_attention_noalloc(const float* q, const float* k_cache, const float* v_cache, int seq_len,
                                       float* context, void* stream);

/* Integer core of the W8 projections on the int8 tensor cores, exposed so that its exactness can be
 * checked: the fp32 activations x[t] (t < n_tokens <= 4, length k) are written as step[t] * X with
 * step[t] = max|x[t]| / 8355710 (fp32 division; 1.0 for an all-zero row) and X = rint(x / step) split into
 * balanced int8 digits X = d0 + 256 d1 + 65536 d2, each in [-128, 127]; then
 *   acc[r][4 d + t] = sum_i codes[r][i] * d_d(t, i)     (int32, exact)
 * for every row r, and 0 in the columns of absent tokens. The W8 projections compute
 * y = scale[r] * step[t] * (acc0 + 256 acc1 + 65536 acc2) from the same sums, in place of the reference's
 * fp32 dot product (hls/decode_only/qwen_decode_attention_kernel.cpp:62-98).
 *   codes  [rows][k] int8 weight codes (device memory, 16-byte aligned), rows % 128 == 0, k % 128 == 0
 *   x      [n_tokens][k] fp32 (device memory)
 *   acc    [rows][12] int32 output (device memory);  step  [n_tokens] fp32 output (device memory) */
int qwen_b200_w8_digit_products(const signed char* codes, int rows, int k, const float* x, int n_tokens, int* acc,
                                float* step, void* stream);

/* Many-token form of the same integer core (the prefill and batched projections): x [n_tokens][k] fp32
 * (16-byte aligned) becomes three digit planes with the per-token step as above, and
 *   acc[d][t][r] = sum_i codes[r][i] * d_d(t, i)      (int32, exact), d < 3, t < n_tokens, r < rows
 * acc is [3][n_tokens][rows] int32, step [n_tokens] fp32 (device memory). Uses stream-ordered temporary
 * allocations for the planes. rows % 128 == 0, k % 128 == 0, 1 <= n_tokens <= 65536. */
int qwen_b200_w8_digit_planes(const signed char* codes, int rows, int k, const float* x, int n_tokens, int* acc,
                              float* step, void* stream);

/* Causal prefill attention context of seq_len tokens (replaces the reference's two-pass prefill context,
 * hls/prefill_only/qwen_prefill_attention_kernel.cpp:204-289): for every query t and head h,
 *   max = max_{j<=t} s_j,  e_j = approx_exp(s_j - max),  context = (sum_j e_j v_j) * (1 / sum_j e_j)
 * with s_j = (q_h . k_j) * 0.08838834764831845 and the reference's approx_exp.
 *   q        [seq_len][1536] fp32 post-RoPE queries (device memory, 16-byte aligned)
 *   k_cache  [seq_len][256] fp32 token-major keys (device memory, 16-byte aligned)
 *   v_cache  [seq_len][256] fp32 token-major values (device memory)
 *   context  [seq_len][1536] fp32 output (device memory, 16-byte aligned)
 *   mode     0: tensor cores (operands as fp16 hi + lo pairs, fp32 accumulation; inputs with |x| >= 32768
 *               or non-finite values are computed by the CUDA-core kernel instead), 1: CUDA cores (fp32)
 * Mode 0 uses stream-ordered temporary allocations (about 8 KB per token). */
int qwen_b200_prefill_attention(const float* q, const float* k_cache, const float* v_cache, int seq_len,
                                float* context, int mode, void* stream);

/* The prefill softmax exponential as the tensor-core attention evaluates it: y[i] = approx_exp(x[i])
 * (hls/prefill_only/qwen_prefill_attention_kernel.cpp:47-110, degree-6 Taylor series with halving and
 * squaring), evaluated without divisions or branches; exposed so that its bit-identity with the reference's
 * function can be checked.
 * x, y [n] fp32 device memory. */
int qwen_b200_prefill_approx_exp(const float* x, float* y, long long n, void* stream);

/* The decode softmax and SiLU exponential of the engine's "exact" option: y[i] = expf(x[i]) exactly as the
 * reference host library's expf computes it (hls/decode_only/qwen_decode_attention_kernel.cpp:149 and
 * qwen_decode_mlp_kernel.cpp:80 call std::exp on floats, which resolves to glibc's expf: a 32-entry 2^(i/32)
 * table and a degree-3 polynomial in double, restated with the fused multiply-adds of glibc's x86-64 FMA
 * build). Exposed so that its identity with the host C library can be checked.
 * x, y [n] fp32 device memory. */
int qwen_b200_exact_expf(const float* x, float* y, long long n, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* QWEN_B200_OPS_H */
