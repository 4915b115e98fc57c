// Host interface of the tcgen05 int8 projections (qgemm.cu).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "qwen_kernels.cuh"

namespace qb {

// Opaque storage for one CUtensorMap (128 bytes, 64-byte aligned) so that callers need not include cuda.h.
struct alignas(64) QgemmMap {
  unsigned char bytes[128];
};

// TMA descriptors of one layer's four int8 weight matrices (q|k|v, o, gate|up, down).
struct QgemmLayerMaps {
  QgemmMap qkv, o, gu, down;
};

// Split-K scratch shared by all projections on one stream: int32 accumulators [2048][16] and per-tile
// counters [16], zero-initialised once; every kernel leaves them zero.
struct QgemmScratch {
  int* acc;
  unsigned* cnt;
};

bool qgemm_make_map(QgemmMap* m, const uint8_t* w, int rows, int k_bytes, int box_rows);
bool qgemm_make_layer_maps(QgemmLayerMaps* m, const LayerDev& L);
size_t qgemm_acc_ints();
size_t qgemm_counter_count();

cudaError_t qgemm_qkv(const QgemmLayerMaps& m, const LayerDev& L, XSource src, DecodeTokens tok, const float* rope_cos,
                      const float* rope_sin, float* q_out, KvView kv, const QgemmScratch& sc, cudaStream_t s, bool pdl);
cudaError_t qgemm_o(const QgemmLayerMaps& m, const LayerDev& L, const float* ctx, int nt, float* out,
                    const QgemmScratch& sc, cudaStream_t s, bool pdl);
cudaError_t qgemm_gateup(const QgemmLayerMaps& m, const LayerDev& L, const float* x, int nt, float* h,
                         const QgemmScratch& sc, cudaStream_t s, bool pdl);
cudaError_t qgemm_down(const QgemmLayerMaps& m, const LayerDev& L, const float* h, const float* resid, int nt,
                       float* out, bool round_out, const QgemmScratch& sc, cudaStream_t s, bool pdl);

// Raw integer product for tests: acc[row][12] = sum_k code(row,k) * digit(n,k) for digit rows n = 4d + t
// (x taken as-is, no RMSNorm), and step[t] = the per-token quantisation step.
cudaError_t qgemm_raw(const QgemmMap& m, int rows, int K, const float* x, int nt, int* acc_out, float* step_out,
                      const QgemmScratch& sc, cudaStream_t s);

unsigned qgemm_kernel_error(bool reset);

}  // namespace qb
