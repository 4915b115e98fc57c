// Internal C++ interface of libqwen_b200.so used by the drop-in C-ABI libraries
// (libqwen_decode_stub.so, libqwen_prefill_stub.so). No CUDA types appear here, so the ABI files
// compile with a plain C++ compiler.
#pragma once

#include <cstdint>

namespace qb {

// One layer's tensors, as separate host arrays (device pointers are accepted too: every copy is
// cudaMemcpyDefault). Weight codes are packed int4 (wbits 4) or int8 (wbits 8), row-major.
struct LayerPtrs {
  const uint8_t *q_w, *k_w, *v_w, *o_w, *gate_w, *up_w, *down_w;
  const float *input_ln, *post_ln;
  const float *q_b, *k_b, *v_b;
  const float *q_s, *k_s, *v_s, *o_s, *gate_s, *up_s, *down_s;
};

// Layer pointers decoded from the reference's DDR images (hls/decode_only/qwen_decode_top_wrapper.cpp:40-75):
// weights at weight_ddr + base + offset, floats at scale_ddr + (base + offset) / 4.
LayerPtrs layer_ptrs_from_ddr(const uint8_t* weight_ddr, uint64_t weights_base, const float* scale_ddr,
                              uint64_t scales_base, int wbits);

// Decode one token through the attention half and/or the MLP half on the GPU.
//   attention: x [1536] -> attn [1536]; reads k/v rows [0, past) and writes row `past` of k_cache/v_cache.
//   mlp:       a [1536] (attention output, or `x` when attention == false) -> out [1536].
// `attn_out` receives the attention output when non-null. Returns a reference status code
// (0 ok, 30 CUDA failure with qwen_b200_last_error() set).
int run_decode(int wbits, const LayerPtrs& L, bool attention, bool mlp, const float* x, int past, float* k_cache,
               float* v_cache, float* attn_out, float* out);

// Prefill seq_len tokens through the attention half and/or the MLP half on the GPU.
//   attention: x [S][1536] -> attn [S][1536]; writes k/v rows [0, S).
//   mlp:       a [S][1536] -> out [S][1536].
int run_prefill(int wbits, const LayerPtrs& L, bool attention, bool mlp, const float* x, int seq_len, float* k_cache,
                float* v_cache, float* attn_out, float* out);

// fp32 weights of one "layer0 reference" layer (unquantised, row-major [out][in]); biases may be null.
struct Layer0Ptrs {
  const float *input_ln, *q_w, *q_b, *k_w, *k_b, *v_w, *v_b, *o_w, *o_b;
  const float *post_ln, *gate_w, *gate_b, *up_w, *up_b, *down_w, *down_b;
};

// The reference's fp32 golden decoder layer on the GPU, same arithmetic and roundings
// (hls/decode_only/qwen_decode_layer0_reference_wrapper.cpp:75-209): one decode token at position `past`,
// caches head-major ([2][past][128] in, [2][past + 1][128] out). Returns 0 or 30 / 31.
int run_layer0_decode(const Layer0Ptrs& W, const float* x, int past, const float* past_k, const float* past_v,
                      float eps, float* out, float* next_k, float* next_v);
// Prefill form (hls/prefill_only/qwen_prefill_layer0_reference_wrapper.cpp:60-255): S tokens from position 0;
// k_cache / v_cache (both or neither) receive the bf16-rounded post-RoPE K and V head-major [2][S][128].
int run_layer0_prefill(const Layer0Ptrs& W, const float* x, int S, float eps, float* out, float* k_cache,
                       float* v_cache);

// Zero-weight layer (all codes 0, scales 1, norm weights 1, biases 0) on the device, used by the
// reference's `*_stub_forward` entry points (hls/decode_only/qwen_decode_host_wrapper.cpp:12-71).
const LayerPtrs& zero_layer_device();

// Prefill sequence capacity: the reference's compile-time kDefaultPrefillSeqTile (128), settable at run
// time (environment QWEN_B200_PREFILL_SEQ_CAPACITY or qwen_b200_set_prefill_seq_capacity).
int prefill_seq_capacity();

void set_error(const char* fmt, ...);

}  // namespace qb
