// Many-token int8 tensor-core projections (tgemm.cu): prefill and batched decode.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "qwen_kernels.cuh"

namespace qb {

// Digit planes of S token rows of width K: planes [3][Spad][K] int8 (Spad = tgemm_pad(S), padded rows zero)
// and the per-token steps [Spad]. Row t: x = step[t] * (d0 + 256 d1 + 65536 d2).
struct DigitPlanes {
  int8_t* planes;
  float* steps;
  int S, Spad, K;
};

// Padded token count: 16, 32 or 64 for small batches (one token tile of that size), else a multiple of 128.
inline int tgemm_pad(int S) { return S <= 16 ? 16 : S <= 32 ? 32 : S <= 64 ? 64 : (S + 127) / 128 * 128; }
inline size_t tgemm_plane_bytes(int S, int K) { return (size_t)3 * tgemm_pad(S) * K; }

// x [S][K] fp32 -> digit planes (one CTA per token row).
cudaError_t tgemm_digitize(const float* x, DigitPlanes d, cudaStream_t s);
// Decode RMSNorm of x [S][1536] with weights w, then digit planes of the normalised rows: the same values
// as decode_rmsnorm followed by tgemm_digitize, in one kernel.
cudaError_t tgemm_rmsnorm_digitize(const float* x, const float* w, DigitPlanes d, cudaStream_t s);
// Prefill RMSNorm (serial fp32 sums, approx_sqrt) of x [S][1536] with weights w, then the digit planes of the
// normalised rows: the same values as launch_prefill_rmsnorm followed by tgemm_digitize, in one kernel.
cudaError_t tgemm_prefill_rmsnorm_digitize(const float* x, const float* w, DigitPlanes d, cudaStream_t s);

// Projections of all S tokens with the prefill epilogues (the same operations as the CUDA-core prefill
// GEMMs in prefill_simt.cu): q|k|v + RoPE (table rows = token index) + K/V rows of a flat cache (raw:
// [S][2048] fp32 scratch for the biased rows before RoPE); o_proj; gate|up + SiLU(approx_exp) * up;
// down + residual (optional bf16 rounding).
cudaError_t tgemm_qkv(const LayerDev& L, const DigitPlanes& x, const float* rope_cos, const float* rope_sin, float* q_out,
                      float* k_cache, float* v_cache, float* raw, cudaStream_t s);
cudaError_t tgemm_o(const LayerDev& L, const DigitPlanes& x, float* out, cudaStream_t s);
cudaError_t tgemm_gateup(const LayerDev& L, const DigitPlanes& x, float* h, cudaStream_t s);
cudaError_t tgemm_down(const LayerDev& L, const DigitPlanes& x, const float* resid, float* out, bool round_out,
                       cudaStream_t s);

// Batched-decode forms (the decode reference's operations): q|k|v with RoPE at pos[t] from the decode
// tables and the new K/V rows written through the paged view at (seq[t], pos[t]); gate|up with expf SiLU.
// o_proj and down are the same as for prefill.
cudaError_t tgemm_qkv_decode(const LayerDev& L, const DigitPlanes& x, const int* pos, const int* seq, KvView kv,
                             const float* rope_cos, const float* rope_sin, float* q_out, float* raw, cudaStream_t s);
cudaError_t tgemm_gateup_decode(const LayerDev& L, const DigitPlanes& x, float* h, cudaStream_t s);
// Decode RMSNorm (double accumulation) of n rows of 1536.
cudaError_t decode_rmsnorm(const float* x, const float* w, int n, float* out, cudaStream_t s);

// Raw integer products for tests: acc [3][S][rows] int32 = sum_k code(row, k) * digit_p(t, k).
cudaError_t tgemm_raw(const uint8_t* codes, int rows, const DigitPlanes& x, int* acc, cudaStream_t s);

unsigned tgemm_kernel_error(bool reset);

}  // namespace qb
