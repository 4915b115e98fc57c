/*
 * Drop-in C-ABI of libqwen_prefill_stub.so, served on a B200 by libqwen_b200.so.
 *
 * Arguments, validation order and status codes follow the reference declaration cited beside each entry
 * point: 0 ok; 1 null / invalid argument or tile; 2 capacity (sequence or tile above the compiled
 * capacity); 20 invalid prefill descriptor, sequence length or tile set; 21 null port; 22 memory window
 * (alignment, bounds or overlap); plus 30 (CUDA failure) and 31 (no usable CUDA device) with the message
 * in qwen_b200_last_error(). The tile arguments are validated exactly as the reference does but do not
 * change the arithmetic (they never did in the reference either: its partial sums carry across tiles).
 *
 * Sequence capacity: the reference compiles it in (kDefaultPrefillSeqTile = 128). Here it defaults to 128
 * as well and can be raised at run time with qwen_b200_set_prefill_seq_capacity() or the environment
 * variable QWEN_B200_PREFILL_SEQ_CAPACITY (up to 32768); the memory-window bounds scale with it exactly as
 * they do when the reference is rebuilt with a larger kDefaultPrefillSeqTile.
 */
#ifndef QWEN_B200_PREFILL_HOST_WRAPPER_H
#define QWEN_B200_PREFILL_HOST_WRAPPER_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* replaces hls/prefill_only/qwen_prefill_host_wrapper.h:9-23 (zero-weight stub layer) */
int qwen_prefill_stub_forward(const float* input_sequence, int seq_len, int attention_seq_tile,
                              int attention_query_tile, int attention_key_tile, int attention_hidden_proj_tile,
                              int attention_kv_proj_tile, int attention_head_dim_tile,
                              int attention_query_heads_parallel, int attention_kv_heads_parallel, int mlp_seq_tile,
                              int mlp_hidden_tile, int mlp_ff_tile, float* output_sequence);

/* replaces hls/prefill_only/qwen_prefill_host_wrapper.h:25-50 */
int qwen_prefill_attention_smoke_forward(const float* input_sequence, int seq_len, int attention_seq_tile,
                                         int attention_query_tile, int attention_key_tile,
                                         int attention_hidden_proj_tile, int attention_kv_proj_tile,
                                         int attention_head_dim_tile, int attention_query_heads_parallel,
                                         int attention_kv_heads_parallel, const float* input_layernorm_weight,
                                         const uint8_t* q_packed_weights, const uint8_t* k_packed_weights,
                                         const uint8_t* v_packed_weights, const uint8_t* o_packed_weights,
                                         const float* q_bias, const float* k_bias, const float* v_bias,
                                         const float* q_scales, const float* k_scales, const float* v_scales,
                                         const float* o_scales, float* k_cache, float* v_cache,
                                         float* output_sequence);

/* replaces hls/prefill_only/qwen_prefill_host_wrapper.h:52-65 */
int qwen_prefill_mlp_smoke_forward(const float* attention_residual_sequence, int seq_len, int mlp_seq_tile,
                                   int mlp_hidden_tile, int mlp_ff_tile,
                                   const float* post_attention_layernorm_weight,
                                   const uint8_t* gate_packed_weights, const uint8_t* up_packed_weights,
                                   const uint8_t* down_packed_weights, const float* gate_scales,
                                   const float* up_scales, const float* down_scales, float* output_sequence);

/* replaces hls/prefill_only/qwen_prefill_host_wrapper.h:67-102 */
int qwen_prefill_layer_smoke_forward(
    const float* input_sequence, int seq_len, int attention_seq_tile, int attention_query_tile,
    int attention_key_tile, int attention_hidden_proj_tile, int attention_kv_proj_tile, int attention_head_dim_tile,
    int attention_query_heads_parallel, int attention_kv_heads_parallel, int mlp_seq_tile, int mlp_hidden_tile,
    int mlp_ff_tile, const float* input_layernorm_weight, const float* post_attention_layernorm_weight,
    const uint8_t* q_packed_weights, const uint8_t* k_packed_weights, const uint8_t* v_packed_weights,
    const uint8_t* o_packed_weights, const uint8_t* gate_packed_weights, const uint8_t* up_packed_weights,
    const uint8_t* down_packed_weights, const float* q_bias, const float* k_bias, const float* v_bias,
    const float* q_scales, const float* k_scales, const float* v_scales, const float* o_scales,
    const float* gate_scales, const float* up_scales, const float* down_scales, float* k_cache, float* v_cache,
    float* output_sequence);

/* replaces hls/prefill_only/qwen_prefill_host_wrapper.h:104-139 (the reference streams the tensors
 * through its HLS glue top; numerically identical to the layer entry point, and accepted only with the
 * default tile set, else status 2) */
int qwen_prefill_glue_smoke_forward(
    const float* input_sequence, int seq_len, int attention_seq_tile, int attention_query_tile,
    int attention_key_tile, int attention_hidden_proj_tile, int attention_kv_proj_tile, int attention_head_dim_tile,
    int attention_query_heads_parallel, int attention_kv_heads_parallel, int mlp_seq_tile, int mlp_hidden_tile,
    int mlp_ff_tile, const float* input_layernorm_weight, const float* post_attention_layernorm_weight,
    const uint8_t* q_packed_weights, const uint8_t* k_packed_weights, const uint8_t* v_packed_weights,
    const uint8_t* o_packed_weights, const uint8_t* gate_packed_weights, const uint8_t* up_packed_weights,
    const uint8_t* down_packed_weights, const float* q_bias, const float* k_bias, const float* v_bias,
    const float* q_scales, const float* k_scales, const float* v_scales, const float* o_scales,
    const float* gate_scales, const float* up_scales, const float* down_scales, float* k_cache, float* v_cache,
    float* output_sequence);

/* replaces hls/prefill_only/qwen_prefill_host_wrapper.h:141-169 (descriptor + DDR ports; the attention
 * output is written to the scratch slot output_sequence_addr + seq_len * 1536 * 4, as the reference does) */
int qwen_prefill_top_smoke_forward(int layer_id, int seq_len, int attention_seq_tile, int attention_query_tile,
                                   int attention_key_tile, int attention_hidden_proj_tile, int attention_kv_proj_tile,
                                   int attention_head_dim_tile, int attention_query_heads_parallel,
                                   int attention_kv_heads_parallel, int mlp_seq_tile, int mlp_hidden_tile,
                                   int mlp_ff_tile, uint64_t input_sequence_addr, uint64_t output_sequence_addr,
                                   uint64_t layer_weights_base_addr, uint64_t layer_scales_base_addr,
                                   uint64_t k_cache_base_addr, uint64_t v_cache_base_addr, const uint8_t* weight_ddr,
                                   const float* scale_ddr, float* kv_cache_ddr, float* activation_ddr,
                                   uint8_t* weight_sram, float* kv_sram, int32_t* partial_sum_sram,
                                   float* softmax_sram, float* control_sram);

/* Int8-weight variants (one code per byte; DDR layout with 1-byte weights). No counterpart in the
 * reference, whose weights are int4 only; they mirror hls/prefill_only/qwen_prefill_host_wrapper.h:141-169
 * and :67-102 respectively. */
int qwen_prefill_top_smoke_forward_w8(int layer_id, int seq_len, int attention_seq_tile, int attention_query_tile,
                                      int attention_key_tile, int attention_hidden_proj_tile,
                                      int attention_kv_proj_tile, int attention_head_dim_tile,
                                      int attention_query_heads_parallel, int attention_kv_heads_parallel,
                                      int mlp_seq_tile, int mlp_hidden_tile, int mlp_ff_tile,
                                      uint64_t input_sequence_addr, uint64_t output_sequence_addr,
                                      uint64_t layer_weights_base_addr, uint64_t layer_scales_base_addr,
                                      uint64_t k_cache_base_addr, uint64_t v_cache_base_addr,
                                      const uint8_t* weight_ddr, const float* scale_ddr, float* kv_cache_ddr,
                                      float* activation_ddr, uint8_t* weight_sram, float* kv_sram,
                                      int32_t* partial_sum_sram, float* softmax_sram, float* control_sram);
int qwen_prefill_layer_smoke_forward_w8(
    const float* input_sequence, int seq_len, int attention_seq_tile, int attention_query_tile,
    int attention_key_tile, int attention_hidden_proj_tile, int attention_kv_proj_tile, int attention_head_dim_tile,
    int attention_query_heads_parallel, int attention_kv_heads_parallel, int mlp_seq_tile, int mlp_hidden_tile,
    int mlp_ff_tile, const float* input_layernorm_weight, const float* post_attention_layernorm_weight,
    const uint8_t* q_weights, const uint8_t* k_weights, const uint8_t* v_weights, const uint8_t* o_weights,
    const uint8_t* gate_weights, const uint8_t* up_weights, const uint8_t* down_weights, const float* q_bias,
    const float* k_bias, const float* v_bias, const float* q_scales, const float* k_scales, const float* v_scales,
    const float* o_scales, const float* gate_scales, const float* up_scales, const float* down_scales,
    float* k_cache, float* v_cache, float* output_sequence);

/* replaces hls/prefill_only/qwen_prefill_host_wrapper.h:171-191 (body: qwen_prefill_layer0_reference_wrapper.cpp:
 * 60-255, 257-300): the fp32-weight golden decoder layer over seq_len tokens from position 0 (fp32 RMSNorm,
 * double accumulation, bf16 rounding after every linear and norm, bf16 RoPE factors, the attention residual
 * kept). Status 1 when input or output is null, seq_len is outside 1..32768 or a weight or norm vector is null. */
int qwen_prefill_layer0_reference_forward(const float* input_sequence, int seq_len,
                                          const float* input_layernorm_weight, const float* q_weight,
                                          const float* q_bias, const float* k_weight, const float* k_bias,
                                          const float* v_weight, const float* v_bias, const float* o_weight,
                                          const float* o_bias, const float* post_attention_layernorm_weight,
                                          const float* gate_weight, const float* gate_bias, const float* up_weight,
                                          const float* up_bias, const float* down_weight, const float* down_bias,
                                          float rms_eps, float* output_sequence);
/* replaces hls/prefill_only/qwen_prefill_host_wrapper.h:193-215 (body: :302-347): the same layer, also writing
 * the bf16-rounded post-RoPE K and V head-major [2][seq_len][128] to k_cache / v_cache (both or neither:
 * status 1 when exactly one is null). */
int qwen_prefill_layer0_reference_forward_with_cache(
    const float* input_sequence, int seq_len, const float* input_layernorm_weight, const float* q_weight,
    const float* q_bias, const float* k_weight, const float* k_bias, const float* v_weight, const float* v_bias,
    const float* o_weight, const float* o_bias, const float* post_attention_layernorm_weight,
    const float* gate_weight, const float* gate_bias, const float* up_weight, const float* up_bias,
    const float* down_weight, const float* down_bias, float rms_eps, float* output_sequence, float* k_cache,
    float* v_cache);

#ifdef __cplusplus
}
#endif

#endif /* QWEN_B200_PREFILL_HOST_WRAPPER_H */
