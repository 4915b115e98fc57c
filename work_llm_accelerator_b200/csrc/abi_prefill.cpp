// Drop-in C-ABI of the reference's libqwen_prefill_stub.so (hls/prefill_only/qwen_prefill_host_wrapper.h:9-215),
// running on the GPU through libqwen_b200.so. Validation follows the reference, in its order:
//   attention kernel  : nulls / seq <= 0 / tile <= 0 / head_dim != 128 -> 1;
//                       seq or tile above capacity -> 2        (qwen_prefill_attention_kernel.cpp:2252-2268)
//   MLP kernel        : nulls / seq <= 0 / tile <= 0 / hidden > 256 / ff > 640 -> 1
//                                                              (qwen_prefill_mlp_kernel.cpp:277-283)
//   top wrapper       : seq <= 0 or > 32768 or > capacity -> 20 (qwen_prefill_top_wrapper.cpp:10-15)
//   top core          : layer id / tile set -> 20, null port -> 21, memory windows -> 22
//                                                              (qwen_prefill_top_core.cpp:42-98)
//   blocks            : null stage pointers -> 21               (qwen_prefill_attention_block.cpp:14)
// Side effects on error match the reference: an MLP-stage error is returned after the attention stage
// has written the K/V cache (and, for the top path, the scratch slot).
#include <cstdint>
#include <vector>

#include "../../include/qwen_prefill_host_wrapper.h"
#include "runtime.h"

namespace {

constexpr int kHidden = 1536;
constexpr int kInter = 8960;
constexpr int kKvWidth = 256;
constexpr int kLayers = 28;
constexpr int kMaxSeq = 32768;
constexpr int kHeads = 12;
constexpr int kKvHeads = 2;

struct Tiles {
  int a_seq, a_query, a_key, a_hidden_proj, a_kv_proj, a_head_dim, a_qhp, a_kvhp;
  int m_seq, m_hidden, m_ff;
};

// reference default tiles (hls/common/qwen2_model_config.h:55-69)
constexpr Tiles kDefaultTiles{128, 32, 64, 64, 64, 128, 2, 1, 128, 256, 640};

// qwen_prefill_attention_kernel.cpp:2252-2268 (tile part of the checks)
int attention_tile_status(const Tiles& t, int seq_len) {
  if (seq_len <= 0 || t.a_seq <= 0 || t.a_query <= 0 || t.a_key <= 0 || t.a_hidden_proj <= 0 || t.a_kv_proj <= 0 ||
      t.a_head_dim != 128 || t.a_qhp <= 0 || t.a_kvhp <= 0) {
    return 1;
  }
  const int cap = qb::prefill_seq_capacity();
  if (seq_len > cap || t.a_seq > cap || t.a_query > 32 || t.a_key > 64 || t.a_hidden_proj > 64 ||
      t.a_kv_proj > 64 || t.a_qhp > kHeads || t.a_kvhp > kKvHeads) {
    return 2;
  }
  return 0;
}

// qwen_prefill_mlp_kernel.cpp:277-283 (tile part)
bool mlp_tiles_ok(const Tiles& t, int seq_len) {
  return !(seq_len <= 0 || t.m_seq <= 0 || t.m_hidden <= 0 || t.m_ff <= 0 || t.m_hidden > 256 || t.m_ff > 640);
}

// llm_layer_dispatch.h:50-61
bool valid_prefill_tile_config(const Tiles& t) {
  const bool hd = t.a_head_dim == 64 || t.a_head_dim == 128;
  return t.a_seq > 0 && t.a_query == 32 && t.a_key == 64 && t.a_hidden_proj == 64 && t.a_kv_proj == 64 && hd &&
         t.a_qhp > 0 && t.a_kvhp > 0 && t.m_seq > 0 && t.m_hidden > 0 && t.m_ff > 0;
}

bool attention_ptrs_ok(const qb::LayerPtrs& L, const float* x, const float* kc, const float* vc, const float* out) {
  return x && out && L.input_ln && L.q_w && L.k_w && L.v_w && L.o_w && L.q_b && L.k_b && L.v_b && L.q_s && L.k_s &&
         L.v_s && L.o_s && kc && vc;
}

bool mlp_ptrs_ok(const qb::LayerPtrs& L, const float* a, const float* out) {
  return a && out && L.post_ln && L.gate_w && L.up_w && L.down_w && L.gate_s && L.up_s && L.down_s;
}

qb::LayerPtrs make_layer(const float* in_ln, const float* post_ln, const uint8_t* qw, const uint8_t* kw,
                         const uint8_t* vw, const uint8_t* ow, const uint8_t* gw, const uint8_t* uw,
                         const uint8_t* dw, const float* qb_, const float* kb, const float* vb, const float* qs,
                         const float* ks, const float* vs, const float* os, const float* gs, const float* us,
                         const float* ds) {
  qb::LayerPtrs L;
  L.q_w = qw;
  L.k_w = kw;
  L.v_w = vw;
  L.o_w = ow;
  L.gate_w = gw;
  L.up_w = uw;
  L.down_w = dw;
  L.input_ln = in_ln;
  L.post_ln = post_ln;
  L.q_b = qb_;
  L.k_b = kb;
  L.v_b = vb;
  L.q_s = qs;
  L.k_s = ks;
  L.v_s = vs;
  L.o_s = os;
  L.gate_s = gs;
  L.up_s = us;
  L.down_s = ds;
  return L;
}

// Attention stage then MLP stage with the reference's per-stage checks; `attn` receives the attention
// output (caller scratch) and `block_status` selects the top path's block null-check code (21) versus the
// kernel's (1).
int layer_run(int wbits, const qb::LayerPtrs& L, const Tiles& t, const float* x, int seq_len, float* kc, float* vc,
              float* attn, float* out, int null_status) {
  if (!attention_ptrs_ok(L, x, kc, vc, attn)) return null_status;
  if (int st = attention_tile_status(t, seq_len)) return st;
  const bool mlp_ok = mlp_ptrs_ok(L, attn, out) && mlp_tiles_ok(t, seq_len);
  if (!mlp_ok) {
    if (int st = qb::run_prefill(wbits, L, true, false, x, seq_len, kc, vc, attn, nullptr)) return st;
    return mlp_ptrs_ok(L, attn, out) ? 1 : null_status;
  }
  return qb::run_prefill(wbits, L, true, true, x, seq_len, kc, vc, attn, out);
}

int layer_entry(int wbits, const float* x, int seq_len, const Tiles& t, const float* in_ln, const float* post_ln,
                const uint8_t* qw, const uint8_t* kw, const uint8_t* vw, const uint8_t* ow, const uint8_t* gw,
                const uint8_t* uw, const uint8_t* dw, const float* qb_, const float* kb, const float* vb,
                const float* qs, const float* ks, const float* vs, const float* os, const float* gs, const float* us,
                const float* ds, float* kc, float* vc, float* out) {
  // qwen_prefill_host_wrapper.cpp:389-476: attention into a temporary [seq][1536], then the MLP.
  const qb::LayerPtrs L = make_layer(in_ln, post_ln, qw, kw, vw, ow, gw, uw, dw, qb_, kb, vb, qs, ks, vs, os, gs, us,
                                     ds);
  if (!attention_ptrs_ok(L, x, kc, vc, out)) return 1;
  if (int st = attention_tile_status(t, seq_len)) return st;
  std::vector<float> attn((size_t)seq_len * kHidden);
  return layer_run(wbits, L, t, x, seq_len, kc, vc, attn.data(), out, 1);
}

bool scalar_aligned(uint64_t off) { return off % 4 == 0; }
bool range_fits(uint64_t off, uint64_t n, uint64_t cap) { return off <= cap && n <= cap - off; }
bool overlap(uint64_t a, uint64_t an, uint64_t b, uint64_t bn) { return a < b + bn && b < a + an; }

// qwen_prefill_top_core.cpp:42-80 with the capacity-dependent windows of qwen_prefill_top_core.h:16-24;
// the layout constants come from the 4-bit reference layout or its 1-byte-weight twin.
bool valid_memory_windows(int wbits, int seq_len, uint64_t in, uint64_t out, uint64_t scratch, uint64_t wb,
                          uint64_t sb, uint64_t kb, uint64_t vb) {
  const int cap = qb::prefill_seq_capacity();
  if (seq_len <= 0 || seq_len > cap) return false;
  const uint64_t w_per = (uint64_t)wbits;
  const uint64_t q_bytes = (uint64_t)kHidden * kHidden * w_per / 8, kv_bytes_w = (uint64_t)kHidden * kKvWidth * w_per / 8;
  const uint64_t gate_bytes = (uint64_t)kHidden * kInter * w_per / 8;
  const uint64_t layer_bytes = 2 * q_bytes + 2 * kv_bytes_w + 3 * gate_bytes + 2ull * kHidden * 4 +
                               (uint64_t)(kHidden + 2 * kKvWidth) * 4 +
                               (uint64_t)(3 * kHidden + 2 * kKvWidth + 2 * kInter) * 4;
  // offsets within the layer (llm_memory_layout.h:84-128)
  const uint64_t q_off = (uint64_t)kHidden * 4;
  const uint64_t down_off = q_off + 2 * q_bytes + 2 * kv_bytes_w + (uint64_t)kHidden * 4 + 2 * gate_bytes;
  const uint64_t down_scale_off = layer_bytes - (uint64_t)kHidden * 4;
  const uint64_t seq_bytes = (uint64_t)seq_len * kHidden * 4;
  const uint64_t kv_bytes = (uint64_t)seq_len * kKvWidth * 4;
  const uint64_t packed_weight_bytes = down_off + gate_bytes - q_off;
  const uint64_t scale_bytes = down_scale_off + (uint64_t)kHidden * 4;
  const uint64_t weight_window = layer_bytes;
  const uint64_t scale_window = ((layer_bytes + 3) / 4) * 4;
  const uint64_t kv_window = 2ull * cap * kKvWidth * 4;
  const uint64_t act_window = 3ull * cap * kHidden * 4;
  if (!scalar_aligned(in) || !scalar_aligned(out) || !scalar_aligned(kb) || !scalar_aligned(vb) ||
      !scalar_aligned(scratch) || !scalar_aligned(sb)) {
    return false;
  }
  if (!range_fits(in, seq_bytes, act_window) || !range_fits(out, seq_bytes, act_window) ||
      !range_fits(scratch, seq_bytes, act_window) || !range_fits(kb, kv_bytes, kv_window) ||
      !range_fits(vb, kv_bytes, kv_window) || !range_fits(wb + q_off, packed_weight_bytes, weight_window) ||
      !range_fits(sb, scale_bytes, scale_window)) {
    return false;
  }
  if (overlap(in, seq_bytes, out, seq_bytes) || overlap(in, seq_bytes, scratch, seq_bytes) ||
      overlap(out, seq_bytes, scratch, seq_bytes) || overlap(kb, kv_bytes, vb, kv_bytes)) {
    return false;
  }
  return true;
}

int top_entry(int wbits, int layer_id, int seq_len, const Tiles& t, uint64_t in, uint64_t out, uint64_t wb,
              uint64_t sb, uint64_t kb, uint64_t vb, const uint8_t* weight_ddr, const float* scale_ddr,
              float* kv_cache_ddr, float* activation_ddr, uint8_t* weight_sram, float* kv_sram, int32_t* psum_sram,
              float* softmax_sram, float* control_sram) {
  // qwen_prefill_top_wrapper.cpp:7-18
  if (seq_len <= 0 || seq_len > kMaxSeq) return 20;
  if (seq_len > qb::prefill_seq_capacity()) return 20;
  // qwen_prefill_top_core.cpp:84-98
  if (layer_id < 0 || layer_id >= kLayers || seq_len <= 0 || !valid_prefill_tile_config(t)) return 20;
  if (!weight_ddr || !scale_ddr || !kv_cache_ddr || !activation_ddr || !weight_sram || !kv_sram || !psum_sram ||
      !softmax_sram || !control_sram) {
    return 21;
  }
  // scratch = output + seq * 1536 * 4 (qwen_prefill_host_wrapper.cpp:690)
  const uint64_t scratch = out + (uint64_t)seq_len * kHidden * 4;
  if (!valid_memory_windows(wbits, seq_len, in, out, scratch, wb, sb, kb, vb)) return 22;
  const qb::LayerPtrs L = qb::layer_ptrs_from_ddr(weight_ddr, wb, scale_ddr, sb, wbits);
  return layer_run(wbits, L, t, activation_ddr + in / 4, seq_len, kv_cache_ddr + kb / 4, kv_cache_ddr + vb / 4,
                   activation_ddr + scratch / 4, activation_ddr + out / 4, 21);
}

Tiles tiles(int as, int aq, int ak, int ah, int akv, int ahd, int aqh, int akh, int ms, int mh, int mf) {
  return Tiles{as, aq, ak, ah, akv, ahd, aqh, akh, ms, mh, mf};
}

bool is_default(const Tiles& t) {
  const Tiles& d = kDefaultTiles;
  return t.a_seq == d.a_seq && t.a_query == d.a_query && t.a_key == d.a_key && t.a_hidden_proj == d.a_hidden_proj &&
         t.a_kv_proj == d.a_kv_proj && t.a_head_dim == 128 && t.a_qhp == d.a_qhp && t.a_kvhp == d.a_kvhp &&
         t.m_seq == d.m_seq && t.m_hidden == d.m_hidden && t.m_ff == d.m_ff;
}

}  // namespace

extern "C" {

int qwen_prefill_stub_forward(const float* input_sequence, int seq_len, int a_seq, int a_query, int a_key,
                              int a_hidden_proj, int a_kv_proj, int a_head_dim, int a_qhp, int a_kvhp, int m_seq,
                              int m_hidden, int m_ff, float* output_sequence) {
  // qwen_prefill_host_wrapper.cpp:205-298: all-zero int4 weights, unit scales / norm weights, zero biases.
  if (input_sequence == nullptr || output_sequence == nullptr || seq_len <= 0) return 1;
  const Tiles t = tiles(a_seq, a_query, a_key, a_hidden_proj, a_kv_proj, a_head_dim, a_qhp, a_kvhp, m_seq, m_hidden,
                        m_ff);
  if (int st = attention_tile_status(t, seq_len)) return st;
  const qb::LayerPtrs& Z = qb::zero_layer_device();
  if (Z.q_w == nullptr) return 31;
  std::vector<float> kv((size_t)seq_len * kKvWidth * 2), attn((size_t)seq_len * kHidden);
  return layer_run(4, Z, t, input_sequence, seq_len, kv.data(), kv.data() + (size_t)seq_len * kKvWidth, attn.data(),
                   output_sequence, 1);
}

int qwen_prefill_attention_smoke_forward(const float* input_sequence, int seq_len, int a_seq, int a_query, int a_key,
                                         int a_hidden_proj, int a_kv_proj, int a_head_dim, int a_qhp, int a_kvhp,
                                         const float* input_layernorm_weight, const uint8_t* q_packed_weights,
                                         const uint8_t* k_packed_weights, const uint8_t* v_packed_weights,
                                         const uint8_t* o_packed_weights, const float* q_bias, const float* k_bias,
                                         const float* v_bias, const float* q_scales, const float* k_scales,
                                         const float* v_scales, const float* o_scales, float* k_cache, float* v_cache,
                                         float* output_sequence) {
  const Tiles t = tiles(a_seq, a_query, a_key, a_hidden_proj, a_kv_proj, a_head_dim, a_qhp, a_kvhp, 1, 1, 1);
  const qb::LayerPtrs L = make_layer(input_layernorm_weight, nullptr, q_packed_weights, k_packed_weights,
                                     v_packed_weights, o_packed_weights, nullptr, nullptr, nullptr, q_bias, k_bias,
                                     v_bias, q_scales, k_scales, v_scales, o_scales, nullptr, nullptr, nullptr);
  if (!attention_ptrs_ok(L, input_sequence, k_cache, v_cache, output_sequence)) return 1;
  if (int st = attention_tile_status(t, seq_len)) return st;
  return qb::run_prefill(4, L, true, false, input_sequence, seq_len, k_cache, v_cache, output_sequence, nullptr);
}

int qwen_prefill_mlp_smoke_forward(const float* attention_residual_sequence, int seq_len, int m_seq, int m_hidden,
                                   int m_ff, const float* post_attention_layernorm_weight,
                                   const uint8_t* gate_packed_weights, const uint8_t* up_packed_weights,
                                   const uint8_t* down_packed_weights, const float* gate_scales,
                                   const float* up_scales, const float* down_scales, float* output_sequence) {
  const Tiles t = tiles(1, 1, 1, 1, 1, 128, 1, 1, m_seq, m_hidden, m_ff);
  const qb::LayerPtrs L = make_layer(nullptr, post_attention_layernorm_weight, nullptr, nullptr, nullptr, nullptr,
                                     gate_packed_weights, up_packed_weights, down_packed_weights, nullptr, nullptr,
                                     nullptr, nullptr, nullptr, nullptr, nullptr, gate_scales, up_scales, down_scales);
  if (!mlp_ptrs_ok(L, attention_residual_sequence, output_sequence) || !mlp_tiles_ok(t, seq_len)) return 1;
  return qb::run_prefill(4, L, false, true, attention_residual_sequence, seq_len, nullptr, nullptr, nullptr,
                         output_sequence);
}

int qwen_prefill_layer_smoke_forward(const float* input_sequence, int seq_len, int a_seq, int a_query, int a_key,
                                     int a_hidden_proj, int a_kv_proj, int a_head_dim, int a_qhp, int a_kvhp,
                                     int m_seq, int m_hidden, int m_ff, const float* input_layernorm_weight,
                                     const float* post_attention_layernorm_weight, const uint8_t* q_packed_weights,
                                     const uint8_t* k_packed_weights, const uint8_t* v_packed_weights,
                                     const uint8_t* o_packed_weights, const uint8_t* gate_packed_weights,
                                     const uint8_t* up_packed_weights, const uint8_t* down_packed_weights,
                                     const float* q_bias, const float* k_bias, const float* v_bias,
                                     const float* q_scales, const float* k_scales, const float* v_scales,
                                     const float* o_scales, const float* gate_scales, const float* up_scales,
                                     const float* down_scales, float* k_cache, float* v_cache,
                                     float* output_sequence) {
  const Tiles t = tiles(a_seq, a_query, a_key, a_hidden_proj, a_kv_proj, a_head_dim, a_qhp, a_kvhp, m_seq, m_hidden,
                        m_ff);
  return layer_entry(4, input_sequence, seq_len, t, input_layernorm_weight, post_attention_layernorm_weight,
                     q_packed_weights, k_packed_weights, v_packed_weights, o_packed_weights, gate_packed_weights,
                     up_packed_weights, down_packed_weights, q_bias, k_bias, v_bias, q_scales, k_scales, v_scales,
                     o_scales, gate_scales, up_scales, down_scales, k_cache, v_cache, output_sequence);
}

int qwen_prefill_glue_smoke_forward(const float* input_sequence, int seq_len, int a_seq, int a_query, int a_key,
                                    int a_hidden_proj, int a_kv_proj, int a_head_dim, int a_qhp, int a_kvhp,
                                    int m_seq, int m_hidden, int m_ff, const float* input_layernorm_weight,
                                    const float* post_attention_layernorm_weight, const uint8_t* q_packed_weights,
                                    const uint8_t* k_packed_weights, const uint8_t* v_packed_weights,
                                    const uint8_t* o_packed_weights, const uint8_t* gate_packed_weights,
                                    const uint8_t* up_packed_weights, const uint8_t* down_packed_weights,
                                    const float* q_bias, const float* k_bias, const float* v_bias,
                                    const float* q_scales, const float* k_scales, const float* v_scales,
                                    const float* o_scales, const float* gate_scales, const float* up_scales,
                                    const float* down_scales, float* k_cache, float* v_cache,
                                    float* output_sequence) {
  // qwen_prefill_host_wrapper.cpp:478-636: null checks -> 1, non-default tiles -> 2, then the stream tops,
  // which run the same host kernels as the layer path. A sequence above the stream capacity makes the
  // reference's stream top return without output (and its host harness then reads empty channels); here
  // it is reported as status 2.
  if (!input_sequence || !input_layernorm_weight || !post_attention_layernorm_weight || !q_packed_weights ||
      !k_packed_weights || !v_packed_weights || !o_packed_weights || !gate_packed_weights || !up_packed_weights ||
      !down_packed_weights || !q_bias || !k_bias || !v_bias || !q_scales || !k_scales || !v_scales || !o_scales ||
      !gate_scales || !up_scales || !down_scales || !k_cache || !v_cache || !output_sequence || seq_len <= 0) {
    return 1;
  }
  const Tiles t = tiles(a_seq, a_query, a_key, a_hidden_proj, a_kv_proj, a_head_dim, a_qhp, a_kvhp, m_seq, m_hidden,
                        m_ff);
  if (!is_default(t)) return 2;
  if (seq_len > qb::prefill_seq_capacity()) return 2;
  return layer_entry(4, input_sequence, seq_len, t, input_layernorm_weight, post_attention_layernorm_weight,
                     q_packed_weights, k_packed_weights, v_packed_weights, o_packed_weights, gate_packed_weights,
                     up_packed_weights, down_packed_weights, q_bias, k_bias, v_bias, q_scales, k_scales, v_scales,
                     o_scales, gate_scales, up_scales, down_scales, k_cache, v_cache, output_sequence);
}

int qwen_prefill_top_smoke_forward(int layer_id, int seq_len, int a_seq, int a_query, int a_key, int a_hidden_proj,
                                   int a_kv_proj, int a_head_dim, int a_qhp, int a_kvhp, int m_seq, int m_hidden,
                                   int m_ff, uint64_t input_sequence_addr, uint64_t output_sequence_addr,
                                   uint64_t layer_weights_base_addr, uint64_t layer_scales_base_addr,
                                   uint64_t k_cache_base_addr, uint64_t v_cache_base_addr, const uint8_t* weight_ddr,
                                   const float* scale_ddr, float* kv_cache_ddr, float* activation_ddr,
                                   uint8_t* weight_sram, float* kv_sram, int32_t* partial_sum_sram,
                                   float* softmax_sram, float* control_sram) {
  const Tiles t = tiles(a_seq, a_query, a_key, a_hidden_proj, a_kv_proj, a_head_dim, a_qhp, a_kvhp, m_seq, m_hidden,
                        m_ff);
  return top_entry(4, layer_id, seq_len, t, input_sequence_addr, output_sequence_addr, layer_weights_base_addr,
                   layer_scales_base_addr, k_cache_base_addr, v_cache_base_addr, weight_ddr, scale_ddr, kv_cache_ddr,
                   activation_ddr, weight_sram, kv_sram, partial_sum_sram, softmax_sram, control_sram);
}

int qwen_prefill_top_smoke_forward_w8(int layer_id, int seq_len, int a_seq, int a_query, int a_key, int a_hidden_proj,
                                      int a_kv_proj, int a_head_dim, int a_qhp, int a_kvhp, int m_seq, int m_hidden,
                                      int m_ff, uint64_t input_sequence_addr, uint64_t output_sequence_addr,
                                      uint64_t layer_weights_base_addr, uint64_t layer_scales_base_addr,
                                      uint64_t k_cache_base_addr, uint64_t v_cache_base_addr,
                                      const uint8_t* weight_ddr, const float* scale_ddr, float* kv_cache_ddr,
                                      float* activation_ddr, uint8_t* weight_sram, float* kv_sram,
                                      int32_t* partial_sum_sram, float* softmax_sram, float* control_sram) {
  const Tiles t = tiles(a_seq, a_query, a_key, a_hidden_proj, a_kv_proj, a_head_dim, a_qhp, a_kvhp, m_seq, m_hidden,
                        m_ff);
  return top_entry(8, layer_id, seq_len, t, input_sequence_addr, output_sequence_addr, layer_weights_base_addr,
                   layer_scales_base_addr, k_cache_base_addr, v_cache_base_addr, weight_ddr, scale_ddr, kv_cache_ddr,
                   activation_ddr, weight_sram, kv_sram, partial_sum_sram, softmax_sram, control_sram);
}

int qwen_prefill_layer_smoke_forward_w8(const float* input_sequence, int seq_len, int a_seq, int a_query, int a_key,
                                        int a_hidden_proj, int a_kv_proj, int a_head_dim, int a_qhp, int a_kvhp,
                                        int m_seq, int m_hidden, int m_ff, const float* input_layernorm_weight,
                                        const float* post_attention_layernorm_weight, const uint8_t* q_weights,
                                        const uint8_t* k_weights, const uint8_t* v_weights, const uint8_t* o_weights,
                                        const uint8_t* gate_weights, const uint8_t* up_weights,
                                        const uint8_t* down_weights, const float* q_bias, const float* k_bias,
                                        const float* v_bias, const float* q_scales, const float* k_scales,
                                        const float* v_scales, const float* o_scales, const float* gate_scales,
                                        const float* up_scales, const float* down_scales, float* k_cache,
                                        float* v_cache, float* output_sequence) {
  const Tiles t = tiles(a_seq, a_query, a_key, a_hidden_proj, a_kv_proj, a_head_dim, a_qhp, a_kvhp, m_seq, m_hidden,
                        m_ff);
  return layer_entry(8, input_sequence, seq_len, t, input_layernorm_weight, post_attention_layernorm_weight,
                     q_weights, k_weights, v_weights, o_weights, gate_weights, up_weights, down_weights, q_bias,
                     k_bias, v_bias, q_scales, k_scales, v_scales, o_scales, gate_scales, up_scales, down_scales,
                     k_cache, v_cache, output_sequence);
}

int qwen_prefill_layer0_reference_forward_with_cache(
    const float* input_sequence, int seq_len, const float* input_layernorm_weight, const float* q_weight,
    const float* q_bias, const float* k_weight, const float* k_bias, const float* v_weight, const float* v_bias,
    const float* o_weight, const float* o_bias, const float* post_attention_layernorm_weight,
    const float* gate_weight, const float* gate_bias, const float* up_weight, const float* up_bias,
    const float* down_weight, const float* down_bias, float rms_eps, float* output_sequence, float* k_cache,
    float* v_cache) {
  // qwen_prefill_layer0_reference_wrapper.cpp:82-88, then the pointers the reference dereferences unchecked
  if (input_sequence == nullptr || output_sequence == nullptr || seq_len <= 0 || seq_len > 32768) return 1;
  if ((k_cache == nullptr) != (v_cache == nullptr)) return 1;
  if (input_layernorm_weight == nullptr || q_weight == nullptr || k_weight == nullptr || v_weight == nullptr ||
      o_weight == nullptr || post_attention_layernorm_weight == nullptr || gate_weight == nullptr ||
      up_weight == nullptr || down_weight == nullptr)
    return 1;
  const qb::Layer0Ptrs W{input_layernorm_weight, q_weight, q_bias, k_weight, k_bias, v_weight, v_bias, o_weight,
                         o_bias, post_attention_layernorm_weight, gate_weight, gate_bias, up_weight, up_bias,
                         down_weight, down_bias};
  return qb::run_layer0_prefill(W, input_sequence, seq_len, rms_eps, output_sequence, k_cache, v_cache);
}

int qwen_prefill_layer0_reference_forward(const float* input_sequence, int seq_len,
                                          const float* input_layernorm_weight, const float* q_weight,
                                          const float* q_bias, const float* k_weight, const float* k_bias,
                                          const float* v_weight, const float* v_bias, const float* o_weight,
                                          const float* o_bias, const float* post_attention_layernorm_weight,
                                          const float* gate_weight, const float* gate_bias, const float* up_weight,
                                          const float* up_bias, const float* down_weight, const float* down_bias,
                                          float rms_eps, float* output_sequence) {
  return qwen_prefill_layer0_reference_forward_with_cache(
      input_sequence, seq_len, input_layernorm_weight, q_weight, q_bias, k_weight, k_bias, v_weight, v_bias,
      o_weight, o_bias, post_attention_layernorm_weight, gate_weight, gate_bias, up_weight, up_bias, down_weight,
      down_bias, rms_eps, output_sequence, nullptr, nullptr);
}

}  // extern "C"
