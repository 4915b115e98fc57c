// Final RMSNorm + fp16 LM head + greedy argmax on the tensor cores (lmhead.cu).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "qwen_kernels.cuh"

namespace qb {

// Device scratch, allocated once (lm_scratch_bytes()): the two fp16 activation planes [2][128][1536],
// the per-token argmax words [128] (zero between calls; the kernel leaves them zero) and a counter (zero).
struct LmScratch {
  __half* planes;
  unsigned long long* packed;
  unsigned* counter;
};

struct LmArgs {
  int n;                       // tokens (1..128)
  float* logits;               // optional [n][151936]
  int* next;                   // [n] argmax
  unsigned long long* packed;  // [n] (orderable value << 32 | ~row), zero on entry
  unsigned* counter;
};

size_t lm_scratch_bytes();

// next[t] = argmax_v E[v] . rmsnorm(x[t]) for t < n (n <= 128), logits optional.
cudaError_t lm_head_tc(const uint16_t* embed, const float* norm_w, const float* x, int n, float* logits, int* next,
                       const LmScratch& sc, cudaStream_t s);

unsigned lm_head_kernel_error(bool reset);

}  // namespace qb
