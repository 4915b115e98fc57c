// Parameter synthesis on the device (bit-identical to the oracle's host generator and quantizer, so a
// full 28-layer model can be created in HBM in milliseconds and still be checked on the host) and small
// elementwise kernels.
//
// Quantizer: symmetric per output channel, scale = max|w| / qmax (1 for an all-zero row),
// code = clip(rint(w / scale)) -- verification/real_host_top_backend.py:31-41 for qmax = 7 (int4, two
// codes per byte, even flat index in the low nibble); qmax = 127 for the int8 track.
#include <cuda_fp16.h>

#include "qwen_kernels.cuh"

namespace qb {
namespace {

// Stream ids of the synthetic tensors (shared with the oracle's generator).
enum : int {
  kSInputLn = 0, kSQ = 1, kSK = 2, kSV = 3, kSO = 4, kSPostLn = 5, kSGate = 6, kSUp = 7, kSDown = 8,
  kSQb = 9, kSKb = 10, kSVb = 11,
};

struct MatDesc {
  int stream;
  int out_dim, in_dim;
  uint64_t w_off;   // byte offset of the codes in the DDR image
  uint64_t s_off;   // byte offset of the scales
};

__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float m = 0.0f;
  for (int w = 0; w < (int)(blockDim.x / 32); ++w) m = fmaxf(m, red[w]);
  __syncthreads();
  return m;
}

// One CTA per output row of one matrix.
__global__ void synth_quant_kernel(uint64_t seed, int layer, int wbits, float sigma, MatDesc m, int row_base,
                                   uint8_t* __restrict__ wddr, float* __restrict__ sddr) {
  __shared__ float red[32];
  const int o = row_base + blockIdx.x;
  const uint64_t key = synth_key(seed, (uint64_t)layer * 32 + m.stream);
  const uint64_t base = (uint64_t)o * m.in_dim;
  float mx = 0.0f;
  for (int i = threadIdx.x; i < m.in_dim; i += blockDim.x) mx = fmaxf(mx, fabsf(synth_normal_dev(key, base + i, 0.0f, sigma)));
  mx = block_max(mx, red);
  const float qmax = wbits == 8 ? 127.0f : 7.0f;
  const float s = mx > 0.0f ? __fdiv_rn(mx, qmax) : 1.0f;
  const int lo = wbits == 8 ? -128 : -8, hi = wbits == 8 ? 127 : 7;
  uint8_t* codes = wddr + m.w_off;
  if (wbits == 8) {
    for (int i = threadIdx.x; i < m.in_dim; i += blockDim.x) {
      int q = (int)rintf(__fdiv_rn(synth_normal_dev(key, base + i, 0.0f, sigma), s));
      q = min(hi, max(lo, q));
      codes[base + i] = (uint8_t)(int8_t)q;
    }
  } else {
    // in_dim is even for every matrix, so a row's nibbles never share a byte with another row
    for (int i = 2 * threadIdx.x; i < m.in_dim; i += 2 * blockDim.x) {
      int q0 = (int)rintf(__fdiv_rn(synth_normal_dev(key, base + i, 0.0f, sigma), s));
      int q1 = (int)rintf(__fdiv_rn(synth_normal_dev(key, base + i + 1, 0.0f, sigma), s));
      q0 = min(hi, max(lo, q0));
      q1 = min(hi, max(lo, q1));
      codes[(base + i) >> 1] = (uint8_t)((q0 & 0xF) | ((q1 & 0xF) << 4));
    }
  }
  if (threadIdx.x == 0) sddr[m.s_off / 4 + o] = s;
}

__global__ void synth_fill_kernel(uint64_t key, uint64_t count, float mean, float sigma, float* __restrict__ out) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < count; i += (uint64_t)gridDim.x * blockDim.x)
    out[i] = synth_normal_dev(key, i, mean, sigma);
}

__global__ void synth_embed_kernel(uint64_t key, uint64_t count, __half* __restrict__ out) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < count; i += (uint64_t)gridDim.x * blockDim.x)
    out[i] = __float2half_rn(synth_normal_dev(key, i, 0.0f, 0.02f));
}

__global__ void round_bf16_kernel(float* __restrict__ x, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    x[i] = round_bf16(x[i]);
}

}  // namespace

cudaError_t launch_synth_fill(uint64_t seed, uint64_t stream, uint64_t count, float mean, float sigma, float* out,
                              cudaStream_t s) {
  synth_fill_kernel<<<1184, 256, 0, s>>>(synth_key(seed, stream), count, mean, sigma, out);
  return cudaGetLastError();
}

cudaError_t launch_synth_embedding(uint64_t seed, uint16_t* embed, cudaStream_t s) {
  synth_embed_kernel<<<4736, 256, 0, s>>>(synth_key(seed, 1ull << 20), (uint64_t)kVocab * kHidden,
                                           reinterpret_cast<__half*>(embed));
  return cudaGetLastError();
}

cudaError_t launch_synth_layer(uint64_t seed, int layer, int wbits, float weight_sigma, uint8_t* wddr, float* sddr,
                               cudaStream_t s) {
  const LayerLayout l = layer_layout(wbits);
  const MatDesc mats[7] = {
      {kSQ, kHidden, kHidden, l.q_w, l.q_s},       {kSK, kKvWidth, kHidden, l.k_w, l.k_s},
      {kSV, kKvWidth, kHidden, l.v_w, l.v_s},      {kSO, kHidden, kHidden, l.o_w, l.o_s},
      {kSGate, kInter, kHidden, l.gate_w, l.gate_s}, {kSUp, kInter, kHidden, l.up_w, l.up_s},
      {kSDown, kHidden, kInter, l.down_w, l.down_s},
  };
  for (const MatDesc& m : mats) {
    synth_quant_kernel<<<m.out_dim, 256, 0, s>>>(seed, layer, wbits, weight_sigma, m, 0, wddr, sddr);
  }
  struct V {
    int stream, n;
    uint64_t off;
    float mean;
  };
  const V vecs[5] = {{kSInputLn, kHidden, l.input_ln, 1.0f}, {kSPostLn, kHidden, l.post_ln, 1.0f},
                     {kSQb, kHidden, l.q_b, 0.0f},           {kSKb, kKvWidth, l.k_b, 0.0f},
                     {kSVb, kKvWidth, l.v_b, 0.0f}};
  for (const V& v : vecs) {
    synth_fill_kernel<<<8, 256, 0, s>>>(synth_key(seed, (uint64_t)layer * 32 + v.stream), v.n, v.mean, 0.02f,
                                        sddr + v.off / 4);
  }
  return cudaGetLastError();
}

cudaError_t launch_round_bf16(float* x, size_t n, cudaStream_t s) {
  round_bf16_kernel<<<592, 256, 0, s>>>(x, n);
  return cudaGetLastError();
}

}  // namespace qb
