// Causal prefill attention on the tensor cores (attention_tc.cu).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>

#include "qwen_kernels.cuh"

namespace qb {

// Device scratch of launch_prefill_attention_tc for S tokens, or Sq queries over S keys (a flag and the fp16
// operand planes).
size_t prefill_attn_tc_scratch_bytes(int S);
size_t prefill_attn_tc_scratch_bytes(int Sq, int S);

// ctx [Sq][1536] = causal GQA attention of q [Sq][1536] (positions qoff .. qoff + Sq - 1) over k_cache / v_cache
// [qoff + Sq][256] (token-major fp32), with the reference's two-pass approx_exp softmax; qoff > 0 is a prefill
// chunk after qoff cached tokens. scratch: 256-byte aligned, prefill_attn_tc_scratch_bytes(Sq, qoff + Sq).
// Inputs outside the fp16 split (|x| >= 32768, non-finite) are computed by the CUDA-core kernel instead.
cudaError_t launch_prefill_attention_tc(const float* q, const float* k_cache, const float* v_cache, int Sq, float* ctx,
                                        void* scratch, size_t scratch_bytes, cudaStream_t s, int qoff = 0);

unsigned attn_tc_kernel_error(bool reset);

}  // namespace qb
