/*
 * Device-resident full-model engine (28 decoder layers + embedding + final RMSNorm + tied fp16 LM head
 * + greedy argmax) on one B200, built from the same kernels as the drop-in per-layer ABI.
 *
 * The reference has no engine: its caller (verification/real_host_top_backend.py:208-351) re-quantizes
 * and re-sends every layer's weights to the host .so on every call, rounds hidden states to bf16
 * between layers (:260, :334) and finishes with the Hugging Face final norm and LM head (:138-146).
 * This engine keeps the weights, the KV cache and the activations in HBM, applies the same bf16
 * rounding between layers, and exposes the prefill / decode-step pair that RealHostTopBackend
 * implements, with token ids in and next-token ids out. All functions return 0 on success, 1 for an
 * invalid argument, 30 for a CUDA failure (see qwen_b200_last_error()), 31 if no device is usable.
 *
 * Numerics: decode uses the reference's decode operators (double RMSNorm, exact RoPE, expf softmax and
 * SiLU); prefill uses the reference's prefill approximations (approx_sqrt/approx_sincos/approx_exp),
 * exactly as RealHostTopBackend mixes the two .so paths. The attention residual is dropped, as in the
 * reference's quantized layer (hls/decode_only/qwen_decode_attention_kernel.cpp:215).
 */
#ifndef QWEN_B200_ENGINE_H
#define QWEN_B200_ENGINE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct qwen_engine qwen_engine;

/* Create an engine on CUDA device `device` with weight codes of `wbits` (4: packed int4, the reference
 * format; 8: int8), room for `max_seqs` concurrent sequences of up to `max_len` tokens each. */
int qwen_engine_create(int device, int wbits, int max_seqs, int max_len, qwen_engine** out);
void qwen_engine_destroy(qwen_engine* e);

/* Fill every parameter with the deterministic seeded generator (weights N(0, weight_sigma) quantized per
 * output channel, biases N(0, 0.02), norm weights N(1, 0.02), fp16 embedding N(0, 0.02)). */
int qwen_engine_init_synthetic(qwen_engine* e, uint64_t seed, float weight_sigma);
/* Load one layer from DDR images in the layout of `wbits` (hls/common/llm_memory_layout.h:84-128). */
int qwen_engine_load_layer(qwen_engine* e, int layer, const uint8_t* weight_ddr, const float* scale_ddr);
/* Load the fp16 [151936][1536] embedding / LM head (as uint16 bits) and the final norm weight [1536]. */
int qwen_engine_load_embedding(qwen_engine* e, const uint16_t* embed_f16, const float* final_norm);

/* Prefill `n` tokens into sequence slot `slot` (which must be empty); writes the greedy next token. */
int qwen_engine_prefill(qwen_engine* e, int slot, const int32_t* tokens, int n, int32_t* next_token);
/* Chunked prefill: `n` more prompt tokens into `slot` after the tokens it already holds (an empty slot: the same
 * as qwen_engine_prefill). The chunk's tokens take the following positions and attend to the cached rows and to
 * each other causally; the result equals prefilling the whole prompt at once (the reference only prefills from
 * position 0, hls/prefill_only/qwen_prefill_attention_kernel.cpp:2232-2367). Writes the greedy next token. */
int qwen_engine_prefill_chunk(qwen_engine* e, int slot, const int32_t* tokens, int n, int32_t* next_token);
/* One greedy decode step for `n` sequences: tokens[i] is appended to slots[i]; next_tokens[i] receives
 * the argmax. Host buffers; the call returns after the next tokens are on the host. */
int qwen_engine_decode(qwen_engine* e, const int32_t* slots, const int32_t* tokens, int n, int32_t* next_tokens);

/* Write / read `n_tokens` KV rows of one layer of a slot in the reference's flat token-major layout
 * ([t][kv_head][128] fp32). write_kv also sets the slot length to n_tokens when layer == 27. */
int qwen_engine_write_kv(qwen_engine* e, int slot, int layer, const float* k, const float* v, int n_tokens);
int qwen_engine_read_kv(qwen_engine* e, int slot, int layer, float* k, float* v, int n_tokens);
/* The same rows in the Hugging Face cache layout the reference caller hands to and takes from its layers
 * (verification/real_host_top_backend.py:199-206): head-major [kv_head 2][t][128] fp32 for K and for V.
 * write_kv_hf also sets the slot length to n_tokens when layer == 27. */
int qwen_engine_read_kv_hf(qwen_engine* e, int slot, int layer, float* k, float* v, int n_tokens);
int qwen_engine_write_kv_hf(qwen_engine* e, int slot, int layer, const float* k, const float* v, int n_tokens);
int qwen_engine_set_seq_len(qwen_engine* e, int slot, int len);
int qwen_engine_seq_len(qwen_engine* e, int slot);
int qwen_engine_reset(qwen_engine* e, int slot);

/* Options: "graphs" (capture decode steps in CUDA graphs, default 1), "pdl" (programmatic dependent
 * launch, default 1), "dump_hidden" (keep every layer's output of the last call, default 0),
 * "logits" (keep the last call's logits, default 0), "prefetch" (stream the next kernels' weights into L2,
 * default 1), "stack" (W8: the whole decode step as one persistent kernel, default 1; 0 = five tensor-core
 * kernels per layer), "bs1" (W8, one sequence per step: the persistent kernel on the CUDA cores with
 * self-validating cross-CTA words, default 1; 0 = the tensor-core persistent kernel; same results),
 * "bs1_ctas" (CTAs of that kernel, 144 .. the SM count, default 144, which leaves SMs free for kernels on
 * other streams and measured fastest; results do not depend on it),
 * "bs1_poison" (test hook of the failure path: the next batch-1 launch finds its cross-CTA counts
 * impossible, gives up after its bounded waits (~1 s) and sets the kernel error flag; the launch after it is
 * clean), "qgemm" (W8 separate-kernel path on the int8 tensor cores, default 1; 0 = CUDA-core
 * GEMV), "trace" (record a per-CTA, per-layer timeline of the persistent kernel, default 0), "batched" (W8: steps
 * of more than 4 sequences as one many-token tensor-core step, default 1; 0 = groups of 4), "lm_tc" (LM head
 * on the tensor cores, default 1; 0 = CUDA-core GEMV), "stack_ring" (weight stages in flight per SM in the
 * persistent kernel, 2..9, default 9), "prefill_attn_tc" (prefill attention on the tensor cores, default 1;
 * 0 = CUDA-core kernel), "attn_ctas" (cap on the CTAs of the separate decode attention kernel, default 0 = one
 * per SM; results do not depend on it), "exact" (every layer and the LM head in the reference host code's
 * arithmetic order: serial fp32 sums per output without FMA, the double decode RMSNorm, the host C library's
 * expf restated for the decode softmax and SiLU, the prefill approximations; greedy tokens and every layer's
 * hidden state are then bit-identical to the reference host libraries. Default 0; slow: one thread per output). */
int qwen_engine_set_option(qwen_engine* e, const char* name, long long value);
/* Per-layer outputs of the last prefill/decode call: [28][rows][1536] floats (rows = tokens of that call). */
int qwen_engine_read_hidden(qwen_engine* e, float* out, long long n_floats);
/* Timeline of the last persistent-kernel decode step (option "trace"): [ctas][28][slots] global-timer
 * nanoseconds, 0 where a CTA had no work. Slot i (stage i: 0 q|k|v, 1 attention, 2 o_proj, 3 gate|up,
 * 4 down) = inputs ready, 5 + i = digits built, 10 + i = epilogues done; 16 + s / 20 + s (projection s:
 * 0 q|k|v, 1 o, 2 gate|up, 3 down) = first weight unit issued / last MMA committed. */
int qwen_engine_read_trace(qwen_engine* e, unsigned long long* out, long long n, int* ctas, int* slots);
/* Logits of the last call: [rows][151936] floats. */
int qwen_engine_read_logits(qwen_engine* e, float* out, long long n_floats);

/* Device-resident timing loop: `warmup` + `steps` greedy decode steps of the `n` sequences in `slots`,
 * each step feeding its argmax back as the next input on the device (no host round trip); the `steps`
 * are timed with CUDA events on the engine's stream. Writes the mean milliseconds per step. */
int qwen_engine_bench_decode(qwen_engine* e, const int32_t* slots, const int32_t* first_tokens, int n, int steps,
                             int warmup, float* ms_per_step);
/* One decode step with device-resident token buffers on the engine's stream, without a host round trip:
 * d_tokens[i] (device int32) is appended to slots[i]; d_next[i] (device int32) receives the argmax. The
 * call returns once the step is enqueued; positions advance on the host bookkeeping immediately. */
int qwen_engine_decode_device(qwen_engine* e, const int32_t* slots, const int32_t* d_tokens, int n,
                              int32_t* d_next);
/* Copy one layer's parameters back out in the DDR-image layout of the engine's width. */
int qwen_engine_read_layer(qwen_engine* e, int layer, uint8_t* weight_ddr, float* scale_ddr);
/* Time each decode kernel kind in isolation with CUDA events on the engine's stream (layers rotated so
 * that weights come from HBM, not L2) for `n` tokens at history `past`; ms_out[6] receives the mean
 * per-launch milliseconds of {qkv, attention, o, gate_up, down, lm_head}. */
int qwen_engine_profile_kernels(qwen_engine* e, int n, int past, int iters, float* ms_out);
/* Per-kernel device time of `steps` eager greedy decode steps of one sequence (device-resident tokens,
 * starting from first_token): ms_out[0] = mean milliseconds of the 28-layer part (the persistent W8 kernel,
 * or the five kernels per layer otherwise), ms_out[1] = the final norm + LM head + argmax kernel. */
int qwen_engine_profile_decode(qwen_engine* e, int slot, int first_token, int steps, float* ms_out);
/* Device time per kernel group of `steps` batched (W8, n > 4) greedy decode steps, eager launches, mean
 * milliseconds per step: ms_out[8] = {RMSNorm, digit planes, q|k|v GEMM, attention, o_proj GEMM, gate|up
 * GEMM, down GEMM, LM head}. */
int qwen_engine_profile_batched(qwen_engine* e, const int32_t* slots, const int32_t* first_tokens, int n, int steps,
                                float* ms_out);
/* Token exchange of a multi-GPU run: one process and one engine per GPU, independent sequences on each, and
 * the step's next-token ids all-gathered over NCCL (NVLink / NVSwitch) -- the only collective of the path.
 * The reference has no counterpart (its host libraries run one layer of one sequence per call).
 * NCCL is opened at run time (libnccl.so.2: the copy already loaded in the process, else the system one);
 * failures return 30 with NCCL's message in qwen_b200_last_error().
 *   qwen_engine_nccl_unique_id: a new communicator id (128 bytes), made on one rank and passed to the
 *     others by the caller's own bootstrap (a TCP store, MPI, a file).
 *   qwen_engine_nccl_init: join the communicator as `rank` of `nranks` (blocks until every rank joined).
 *   qwen_engine_gather_tokens: enqueue on the engine's stream the all-gather of n int32 ids per rank,
 *     d_local [n] -> d_all [nranks][n] (device memory), after the step that wrote them. */
int qwen_engine_nccl_unique_id(uint8_t* id_out);
int qwen_engine_nccl_init(qwen_engine* e, const uint8_t* id, int nranks, int rank);
int qwen_engine_gather_tokens(qwen_engine* e, const int32_t* d_local, int n, int32_t* d_all);
/* The same all-gather on a side stream of the engine, so that it runs beside the following decode steps:
 * it starts after the engine stream's work enqueued so far, and the engine stream's work enqueued after the
 * call waits for the previous asynchronous gather (at most two in flight: d_local may be rewritten from the
 * step after next on). qwen_engine_gather_join makes the engine stream wait for the last one (d_all is then
 * complete once the stream reaches that point). With option "bs1_ctas" below the SM count (the default) the
 * batch-1 decode kernel leaves SMs free for the NCCL kernel. */
int qwen_engine_gather_tokens_async(qwen_engine* e, const int32_t* d_local, int n, int32_t* d_all);
int qwen_engine_gather_join(qwen_engine* e);
/* The engine's CUDA stream (cudaStream_t) for callers that record their own events. */
void* qwen_engine_stream(qwen_engine* e);
/* Number of kernels one decode step of `n` sequences launches. */
int qwen_engine_kernels_per_decode_step(qwen_engine* e, int n);

#ifdef __cplusplus
}
#endif

#endif /* QWEN_B200_ENGINE_H */
