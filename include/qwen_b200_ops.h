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

#ifdef __cplusplus
}
#endif

#endif /* QWEN_B200_OPS_H */
