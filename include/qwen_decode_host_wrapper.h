/*
 * Drop-in C-ABI of libqwen_decode_stub.so, served on a B200 by libqwen_b200.so.
 *
 * Every entry point below takes exactly the arguments of the reference declaration cited beside it and
 * returns the reference's status codes (0 ok; 1 null or invalid argument; 10 invalid decode descriptor;
 * 11 null port), plus 30 when a CUDA call failed and 31 when no CUDA device is usable (the message is
 * in qwen_b200_last_error(), declared in qwen_b200_runtime.h). Buffers are host arrays (device
 * pointers are accepted as well); calls are synchronous. Weight codes are packed int4 (two per byte,
 * even flat index in the low nibble) unless the name ends in `_w8`.
 */
#ifndef QWEN_B200_DECODE_HOST_WRAPPER_H
#define QWEN_B200_DECODE_HOST_WRAPPER_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* replaces hls/decode_only/qwen_decode_host_wrapper.h:9-12 (zero-weight stub layer) */
int qwen_decode_stub_forward(const float* input_token, int past_seq_len, float* output_token);

/* replaces hls/decode_only/qwen_decode_host_wrapper.h:14-31 */
int qwen_decode_attention_smoke_forward(const float* input_token, int past_seq_len,
                                        const float* input_layernorm_weight, const uint8_t* q_packed_weights,
                                        const uint8_t* k_packed_weights, const uint8_t* v_packed_weights,
                                        const uint8_t* o_packed_weights, const float* q_bias, const float* k_bias,
                                        const float* v_bias, const float* q_scales, const float* k_scales,
                                        const float* v_scales, const float* o_scales, float* k_cache, float* v_cache,
                                        float* output_token);

/* replaces hls/decode_only/qwen_decode_host_wrapper.h:33-42 */
int qwen_decode_mlp_smoke_forward(const float* attention_residual_token, const float* post_attention_layernorm_weight,
                                  const uint8_t* gate_packed_weights, const uint8_t* up_packed_weights,
                                  const uint8_t* down_packed_weights, const float* gate_scales,
                                  const float* up_scales, const float* down_scales, float* output_token);

/* replaces hls/decode_only/qwen_decode_host_wrapper.h:44-61 (descriptor + DDR ports; the five SRAM
 * ports are only null-checked, as in the reference) */
int qwen_decode_top_smoke_forward(int layer_id, int past_seq_len, uint64_t input_token_addr,
                                  uint64_t output_token_addr, uint64_t layer_weights_base_addr,
                                  uint64_t layer_scales_base_addr, uint64_t k_cache_base_addr,
                                  uint64_t v_cache_base_addr, const uint8_t* weight_ddr, const float* scale_ddr,
                                  float* kv_cache_ddr, float* activation_ddr, uint8_t* weight_sram, float* kv_sram,
                                  int32_t* partial_sum_sram, float* softmax_sram, float* control_sram);

/* replaces hls/decode_only/qwen_decode_host_wrapper.h:63-87 */
int qwen_decode_layer_smoke_forward(const float* input_token, int past_seq_len, const float* input_layernorm_weight,
                                    const float* post_attention_layernorm_weight, const uint8_t* q_packed_weights,
                                    const uint8_t* k_packed_weights, const uint8_t* v_packed_weights,
                                    const uint8_t* o_packed_weights, const uint8_t* gate_packed_weights,
                                    const uint8_t* up_packed_weights, const uint8_t* down_packed_weights,
                                    const float* q_bias, const float* k_bias, const float* v_bias,
                                    const float* q_scales, const float* k_scales, const float* v_scales,
                                    const float* o_scales, const float* gate_scales, const float* up_scales,
                                    const float* down_scales, float* k_cache, float* v_cache, float* output_token);

/* Int8-weight variants (one code per byte; the DDR layout keeps the reference's field order with
 * 1-byte weights). No counterpart in the reference, whose weights are int4 only; they mirror
 * hls/decode_only/qwen_decode_host_wrapper.h:44-61 and :63-87 respectively. */
int qwen_decode_top_smoke_forward_w8(int layer_id, int past_seq_len, uint64_t input_token_addr,
                                     uint64_t output_token_addr, uint64_t layer_weights_base_addr,
                                     uint64_t layer_scales_base_addr, uint64_t k_cache_base_addr,
                                     uint64_t v_cache_base_addr, const uint8_t* weight_ddr, const float* scale_ddr,
                                     float* kv_cache_ddr, float* activation_ddr, uint8_t* weight_sram, float* kv_sram,
                                     int32_t* partial_sum_sram, float* softmax_sram, float* control_sram);
int qwen_decode_layer_smoke_forward_w8(const float* input_token, int past_seq_len,
                                       const float* input_layernorm_weight,
                                       const float* post_attention_layernorm_weight, const uint8_t* q_weights,
                                       const uint8_t* k_weights, const uint8_t* v_weights, const uint8_t* o_weights,
                                       const uint8_t* gate_weights, const uint8_t* up_weights,
                                       const uint8_t* down_weights, const float* q_bias, const float* k_bias,
                                       const float* v_bias, const float* q_scales, const float* k_scales,
                                       const float* v_scales, const float* o_scales, const float* gate_scales,
                                       const float* up_scales, const float* down_scales, float* k_cache,
                                       float* v_cache, float* output_token);

/* replaces hls/decode_only/qwen_decode_host_wrapper.h:89-113 (body: qwen_decode_layer0_reference_wrapper.cpp:75-209):
 * the fp32-weight golden decoder layer (double accumulation, bf16 rounding after every linear and norm, the
 * attention residual kept), one token at position past_seq_len. Weights are fp32 row-major [out][in]; biases
 * may be null. Caches are head-major: past [2][past_seq_len][128], next [2][past_seq_len + 1][128]. Status 1
 * when input, output or a next cache is null, past_seq_len < 0, a weight or norm vector is null, or a past
 * cache is null while past_seq_len > 0 (the reference reads it). */
int qwen_decode_layer0_reference_forward(const float* input_token, int past_seq_len, const float* past_k_cache,
                                         const float* past_v_cache, const float* input_layernorm_weight,
                                         const float* q_weight, const float* q_bias, const float* k_weight,
                                         const float* k_bias, const float* v_weight, const float* v_bias,
                                         const float* o_weight, const float* o_bias,
                                         const float* post_attention_layernorm_weight, const float* gate_weight,
                                         const float* gate_bias, const float* up_weight, const float* up_bias,
                                         const float* down_weight, const float* down_bias, float rms_eps,
                                         float* output_token, float* next_k_cache, float* next_v_cache);

#ifdef __cplusplus
}
#endif

#endif /* QWEN_B200_DECODE_HOST_WRAPPER_H */
