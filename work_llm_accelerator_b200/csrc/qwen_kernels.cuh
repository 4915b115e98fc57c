// Host-side launch interface of the CUDA kernels (internal to libqwen_b200.so).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <map>
#include <mutex>
#include <utility>

#include "qwen_common.cuh"

namespace qb {

// Tokens processed together by one decode GEMV launch (the GEMV path serves batch 1..kGemvMaxTokens).
constexpr int kGemvMaxTokens = 4;

// Per-token decode metadata on the device: position of the new token (= past length) and the
// sequence slot used to address a paged KV cache.
struct DecodeTokens {
  const int* pos;  // [nt]
  const int* seq;  // [nt]
  int nt;
};

// Where a decode GEMV reads its input activations from.
struct XSource {
  const float* x;           // [nt][K] fp32, or nullptr when gathering from the embedding table
  const uint16_t* embed;    // fp16 [vocab][1536] (used when x == nullptr)
  const int* tokens;        // [nt] token ids for the embedding gather
};

// --- decode (batch 1..4), CUDA-core GEMV kernels --------------------------------------------------
// `pf`/`pf_bytes` optionally name weights of following kernels to stream into L2 before the kernel
// waits for its predecessor (programmatic dependent launch).
// q_out [nt][1536]; K and V rows written at each token's position through `kv`.
cudaError_t launch_decode_qkv(int wbits, const LayerDev& L, XSource src, DecodeTokens tok, const float* rope_cos,
                              const float* rope_sin, float* q_out, KvView kv, cudaStream_t s, bool pdl,
                              const void* pf = nullptr, size_t pf_bytes = 0);
// out [nt][1536] = o_proj(ctx)
cudaError_t launch_decode_o(int wbits, const LayerDev& L, const float* ctx, int nt, float* out, cudaStream_t s,
                            bool pdl, const void* pf = nullptr, size_t pf_bytes = 0);
// h [nt][8960] = silu(gate(norm(a))) * up(norm(a))
cudaError_t launch_decode_gateup(int wbits, const LayerDev& L, const float* a, int nt, float* h, cudaStream_t s,
                                 bool pdl, const void* pf = nullptr, size_t pf_bytes = 0);
// out [nt][1536] = a + down(h), optionally rounded to bf16 (RNE) for the next layer
cudaError_t launch_decode_down(int wbits, const LayerDev& L, const float* h, const float* a, int nt, float* out,
                               bool round_out, cudaStream_t s, bool pdl, const void* pf = nullptr,
                               size_t pf_bytes = 0);
// next_token[t] = argmax_v (E[v] . rmsnorm(x[t]) ); logits optional [nt][vocab]
cudaError_t launch_lm_head_argmax(const uint16_t* embed, const float* norm_w, const float* x, int nt, float* logits,
                                  float* partial, unsigned* counter, int* next_token, cudaStream_t s, bool pdl);
int lm_head_partial_floats();  // size of the `partial` scratch in floats
// Error flag of the streaming GEMV kernels (1 = a bounded mbarrier wait gave up); optionally cleared.
unsigned gemv_kernel_error(bool reset);

// --- decode attention (flash-decoding over 64-token chunks, then an in-order merge kernel) --------
// ctx [nt][1536]. scratch: attn_partial_floats(nt, max_len) floats; counters: unused (kept for callers).
// `prefetch`/`prefetch_bytes` optionally name weights of the following kernels to stream into L2 meanwhile.
// `max_ctas` > 0 caps the persistent grid (default: one CTA per SM); results do not depend on it.
cudaError_t launch_decode_attention(const float* q, KvView kv, DecodeTokens tok, int max_len, float* ctx,
                                    float* scratch, unsigned* counters, cudaStream_t s, bool pdl,
                                    const void* prefetch = nullptr, size_t prefetch_bytes = 0, int max_ctas = 0);
size_t attn_partial_floats(int nt, int max_len);
// Error flag of the decode attention kernel (1 = a bounded mbarrier wait gave up); optionally cleared.
unsigned decode_attn_kernel_error(bool reset);

// --- prefill -------------------------------------------------------------------------------------
// xn [S][1536] = prefill RMSNorm (serial fp32 sum, approx_sqrt), bit-identical to the reference.
cudaError_t launch_prefill_rmsnorm(const float* x, const float* w, int S, float* xn, cudaStream_t s);
// Prefill RoPE cos/sin table [npos][64] (approx_sincos), bit-identical to the reference.
cudaError_t launch_prefill_rope_table(int npos, float* cos_out, float* sin_out, cudaStream_t s);
// Projection GEMMs on CUDA cores (fp32): Y = X . dequant(W)^T with fused epilogues.
cudaError_t launch_prefill_qkv(int wbits, const LayerDev& L, const float* xn, int S, const float* rope_cos,
                               const float* rope_sin, float* q_out, float* k_cache, float* v_cache, cudaStream_t s);
cudaError_t launch_prefill_o(int wbits, const LayerDev& L, const float* ctx, int S, float* out, cudaStream_t s);
cudaError_t launch_prefill_gateup(int wbits, const LayerDev& L, const float* xn, int S, float* h, cudaStream_t s);
cudaError_t launch_prefill_down(int wbits, const LayerDev& L, const float* h, const float* a, int S, float* out,
                                bool round_out, cudaStream_t s);
// Causal two-pass GQA attention with approx_exp (scores and max bit-identical to the reference): S queries
// (rows of q and ctx) at positions qoff .. qoff + S - 1 over k_cache / v_cache rows 0 .. qoff + S - 1.
cudaError_t launch_prefill_attention(const float* q, const float* k_cache, const float* v_cache, int S, float* ctx,
                                     cudaStream_t s, int qoff = 0);
// Same kernel, run only when *only_if != 0 (read on the device; the CTAs return at once otherwise).
cudaError_t launch_prefill_attention_gated(const float* q, const float* k_cache, const float* v_cache, int S,
                                           float* ctx, const int* only_if, cudaStream_t s, int qoff = 0);

// --- misc ----------------------------------------------------------------------------------------
// Deterministic synthetic layer parameters written straight into a device DDR image of `wbits` layout.
cudaError_t launch_synth_layer(uint64_t seed, int layer, int wbits, float weight_sigma, uint8_t* weight_ddr,
                               float* scale_ddr, cudaStream_t s);
cudaError_t launch_synth_fill(uint64_t seed, uint64_t stream, uint64_t count, float mean, float sigma, float* out,
                              cudaStream_t s);
cudaError_t launch_synth_embedding(uint64_t seed, uint16_t* embed, cudaStream_t s);
cudaError_t launch_round_bf16(float* x, size_t n, cudaStream_t s);

// Raise `func`'s dynamic shared-memory limit to `bytes` on the current device (function attributes belong to a
// device's context, so a process that uses several GPUs needs them set on each), once per kernel and device.
inline cudaError_t ensure_smem_attr(const void* func, size_t bytes) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, size_t> done;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  size_t& have = done[std::make_pair(func, dev)];
  if (bytes <= have) return cudaSuccess;
  e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e == cudaSuccess) have = bytes;
  return e;
}

// Number of SMs of the current device (cached per device).
inline int device_sm_count() {
  static std::mutex mu;
  static std::map<int, int> sms;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  std::lock_guard<std::mutex> lock(mu);
  int& n = sms[dev];
  if (n <= 0 && (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)) n = 148;
  return n;
}

// Launch helper: cudaLaunchKernelEx with optional programmatic stream serialization.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl,
                            Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace qb
