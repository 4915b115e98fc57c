// GQA attention kernels (12 query heads over 2 KV heads, head_dim 128).
//
// Decode (hls/decode_only/qwen_decode_attention_kernel.cpp:113-162): the reference makes two passes over
// the whole history (max, then expf(s - max)). Here the history is split into 64-token chunks, one CTA
// per (token, KV head, chunk) handling the 6 query heads that share the KV head, so each K/V row is read
// once for all six. Each chunk keeps its own max; the last CTA of a (token, KV head) to finish merges the
// chunks in chunk order (rescaling by expf(m_c - M)), so the result equals the two-pass value up to
// rounding and is deterministic. Scores q.k are summed serially over the 128 dims with separately
// rounded multiply and add, exactly as the reference does.
//
// Prefill (hls/prefill_only/qwen_prefill_attention_kernel.cpp:204-289): approx_exp(a) * approx_exp(b) is
// not approx_exp(a + b), so online rescaling would change results; the kernel keeps the reference's two
// passes: pass 1 takes the causal max of the scaled scores, pass 2 recomputes each score and accumulates
// approx_exp(score * scale - max). Scores, max and every exp value are bit-identical to the reference;
// only the order of the denominator and context sums differs.
#include "qwen_kernels.cuh"

namespace qb {
namespace {

constexpr int kChunk = 64;            // decode keys per CTA
constexpr int kPartStride = 2 + kHeadDim;  // m, l, acc[128]

__global__ void __launch_bounds__(64) decode_attn_kernel(const float* __restrict__ q, KvView kv, DecodeTokens tok,
                                                         int max_chunks, float* __restrict__ ctx,
                                                         float* __restrict__ part, unsigned* __restrict__ counters) {
  const int c = blockIdx.x, g = blockIdx.y, t = blockIdx.z;
  const int tid = threadIdx.x;
  __shared__ float qs[kGroups][kHeadDim];
  __shared__ float es[kGroups][kChunk];
  __shared__ float ms[kGroups], ls[kGroups];
  __shared__ bool last;

  griddep_wait();
  const int L = tok.pos[t] + 1;
  const int nchunks = (L + kChunk - 1) / kChunk;
  if (c >= nchunks) return;
  const int seq = tok.seq[t];
  const float scaling = (float)(1.0 / 1.4142135623730951 / 8.0);  // float(1/sqrt(128)), :119

  for (int i = tid; i < kGroups * kHeadDim; i += 64)
    qs[i / kHeadDim][i % kHeadDim] = q[(size_t)t * kHidden + g * kGroups * kHeadDim + i];
  __syncthreads();

  // scores: one key per thread, six serial dot products
  const int j = c * kChunk + tid;
  float sc[kGroups];
  if (j < L) {
    const float4* kr = reinterpret_cast<const float4*>(kv_row(kv, seq, j, 0) + g * kHeadDim);
#pragma unroll
    for (int h = 0; h < kGroups; ++h) sc[h] = 0.0f;
#pragma unroll 4
    for (int d4 = 0; d4 < kHeadDim / 4; ++d4) {
      const float4 kk = kr[d4];
#pragma unroll
      for (int h = 0; h < kGroups; ++h) {
        sc[h] = __fadd_rn(sc[h], __fmul_rn(qs[h][4 * d4 + 0], kk.x));
        sc[h] = __fadd_rn(sc[h], __fmul_rn(qs[h][4 * d4 + 1], kk.y));
        sc[h] = __fadd_rn(sc[h], __fmul_rn(qs[h][4 * d4 + 2], kk.z));
        sc[h] = __fadd_rn(sc[h], __fmul_rn(qs[h][4 * d4 + 3], kk.w));
      }
    }
#pragma unroll
    for (int h = 0; h < kGroups; ++h) es[h][tid] = __fmul_rn(sc[h], scaling);
  } else {
#pragma unroll
    for (int h = 0; h < kGroups; ++h) es[h][tid] = -INFINITY;
  }
  __syncthreads();
  const int n = min(kChunk, L - c * kChunk);
  if (tid < kGroups) {
    float m = -1.0e30f;
    for (int i = 0; i < n; ++i) m = m < es[tid][i] ? es[tid][i] : m;
    ms[tid] = m;
  }
  __syncthreads();
#pragma unroll
  for (int h = 0; h < kGroups; ++h) es[h][tid] = tid < n ? expf(es[h][tid] - ms[h]) : 0.0f;
  __syncthreads();
  if (tid < kGroups) {
    float l = 0.0f;
    for (int i = 0; i < n; ++i) l += es[tid][i];
    ls[tid] = l;
  }
  // P.V: thread owns dims 2*tid, 2*tid+1 for all six heads
  float acc[kGroups][2];
#pragma unroll
  for (int h = 0; h < kGroups; ++h) acc[h][0] = acc[h][1] = 0.0f;
  for (int i = 0; i < n; ++i) {
    const float2 vv = *reinterpret_cast<const float2*>(kv_row(kv, seq, c * kChunk + i, 1) + g * kHeadDim + 2 * tid);
#pragma unroll
    for (int h = 0; h < kGroups; ++h) {
      acc[h][0] = fmaf(es[h][i], vv.x, acc[h][0]);
      acc[h][1] = fmaf(es[h][i], vv.y, acc[h][1]);
    }
  }
  __syncthreads();
  float* my = part + (((size_t)t * kKvHeads + g) * max_chunks + c) * kGroups * kPartStride;
#pragma unroll
  for (int h = 0; h < kGroups; ++h) {
    my[h * kPartStride + 2 + 2 * tid] = acc[h][0];
    my[h * kPartStride + 3 + 2 * tid] = acc[h][1];
    if (tid == 0) {
      my[h * kPartStride + 0] = ms[h];
      my[h * kPartStride + 1] = ls[h];
    }
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned prev = atomicAdd(&counters[t * kKvHeads + g], 1u);
    last = (prev == (unsigned)nchunks - 1u);
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  // merge the chunks of this (token, KV head) in chunk order
  const float* base = part + ((size_t)t * kKvHeads + g) * max_chunks * kGroups * kPartStride;
#pragma unroll
  for (int h = 0; h < kGroups; ++h) {
    float M = -INFINITY;
    for (int cc = 0; cc < nchunks; ++cc) M = fmaxf(M, __ldcg(&base[(cc * kGroups + h) * kPartStride]));
    float Lsum = 0.0f, o0 = 0.0f, o1 = 0.0f;
    for (int cc = 0; cc < nchunks; ++cc) {
      const float* pc = base + (cc * kGroups + h) * kPartStride;
      const float w = expf(__ldcg(&pc[0]) - M);
      Lsum = fmaf(__ldcg(&pc[1]), w, Lsum);
      o0 = fmaf(__ldcg(&pc[2 + 2 * tid]), w, o0);
      o1 = fmaf(__ldcg(&pc[3 + 2 * tid]), w, o1);
    }
    const float inv = Lsum > 0.0f ? 1.0f / Lsum : 0.0f;
    float* out = ctx + (size_t)t * kHidden + (g * kGroups + h) * kHeadDim + 2 * tid;
    out[0] = o0 * inv;
    out[1] = o1 * inv;
  }
  if (tid == 0) counters[t * kKvHeads + g] = 0u;
}

// ------------------------------------------------------------------------------------------------
// prefill: CTA = (block of 16 queries, KV head); 8 warps; K/V tiles of 32 keys in shared memory
// ------------------------------------------------------------------------------------------------
constexpr int kPQ = 16;                 // queries per CTA
constexpr int kPK = 32;                 // keys per tile
constexpr int kPairs = kPQ * kGroups;   // 96 (query, head) pairs
constexpr int kPad = kHeadDim + 1;      // padded row length (bank-conflict free column walks)

struct PrefillSmem {
  float qs[kPairs][kPad];
  float ks[kPK][kPad];
  float vs[kPK][kHeadDim];
  float es[kPairs][kPK];
  float mx[kPairs];
  float den[kPairs];
};

__global__ void __launch_bounds__(256) prefill_attn_kernel(const float* __restrict__ q, const float* __restrict__ kc,
                                                           const float* __restrict__ vc, int S,
                                                           float* __restrict__ ctx) {
  extern __shared__ float4 smem4[];
  PrefillSmem& sm = *reinterpret_cast<PrefillSmem*>(smem4);
  const int q0 = blockIdx.x * kPQ, g = blockIdx.y;
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int nq = min(kPQ, S - q0);

  // load Q pairs: pair p = qi * 6 + h
  for (int i = tid; i < kPairs * kHeadDim; i += 256) {
    const int p = i / kHeadDim, d = i % kHeadDim;
    const int qi = p / kGroups, h = p % kGroups;
    sm.qs[p][d] = qi < nq ? q[(size_t)(q0 + qi) * kHidden + (g * kGroups + h) * kHeadDim + d] : 0.0f;
  }
  if (tid < kPairs) {
    sm.mx[tid] = -1.0e30f;
    sm.den[tid] = 0.0f;
  }
  const int kend = q0 + nq;  // keys [0, kend)
  const int ntiles = (kend + kPK - 1) / kPK;

  // pass 1: causal max of the scaled scores
  for (int tile = 0; tile < ntiles; ++tile) {
    const int k0 = tile * kPK;
    __syncthreads();
    for (int i = tid; i < kPK * kHeadDim; i += 256) {
      const int jj = i / kHeadDim, d = i % kHeadDim;
      sm.ks[jj][d] = (k0 + jj) < kend ? kc[(size_t)(k0 + jj) * kKvWidth + g * kHeadDim + d] : 0.0f;
    }
    __syncthreads();
    for (int p = warp; p < kPairs; p += 8) {
      const int qi = p / kGroups;
      const int key = k0 + lane;
      float s = 0.0f;
      for (int d = 0; d < kHeadDim; ++d) s = __fadd_rn(s, __fmul_rn(sm.qs[p][d], sm.ks[lane][d]));
      const float ss = __fmul_rn(s, kAttentionScaling);
      float m = (qi < nq && key <= q0 + qi) ? ss : -INFINITY;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      if (lane == 0) sm.mx[p] = m > sm.mx[p] ? m : sm.mx[p];
    }
  }
  __syncthreads();

  // pass 2: e = approx_exp(score * scale - max), denominator and context
  const int d = tid % kHeadDim;   // output dim owned by this thread
  const int ph = tid / kHeadDim;  // pairs ph, ph+2, ph+4, ...
  float acc[kPairs / 2];
#pragma unroll
  for (int i = 0; i < kPairs / 2; ++i) acc[i] = 0.0f;
  for (int tile = 0; tile < ntiles; ++tile) {
    const int k0 = tile * kPK;
    __syncthreads();
    for (int i = tid; i < kPK * kHeadDim; i += 256) {
      const int jj = i / kHeadDim, dd = i % kHeadDim;
      const bool ok = (k0 + jj) < kend;
      sm.ks[jj][dd] = ok ? kc[(size_t)(k0 + jj) * kKvWidth + g * kHeadDim + dd] : 0.0f;
      sm.vs[jj][dd] = ok ? vc[(size_t)(k0 + jj) * kKvWidth + g * kHeadDim + dd] : 0.0f;
    }
    __syncthreads();
    for (int p = warp; p < kPairs; p += 8) {
      const int qi = p / kGroups;
      const int key = k0 + lane;
      float s = 0.0f;
      for (int dd = 0; dd < kHeadDim; ++dd) s = __fadd_rn(s, __fmul_rn(sm.qs[p][dd], sm.ks[lane][dd]));
      const float ss = __fmul_rn(s, kAttentionScaling);
      const bool valid = qi < nq && key <= q0 + qi;
      const float e = valid ? approx_exp(__fsub_rn(ss, sm.mx[p])) : 0.0f;
      sm.es[p][lane] = e;
      float l = e;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
      if (lane == 0) sm.den[p] += l;
    }
    __syncthreads();
#pragma unroll 4
    for (int jj = 0; jj < kPK; ++jj) {
      const float vv = sm.vs[jj][d];
#pragma unroll
      for (int i = 0; i < kPairs / 2; ++i) acc[i] = fmaf(sm.es[ph + 2 * i][jj], vv, acc[i]);
    }
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < kPairs / 2; ++i) {
    const int p = ph + 2 * i;
    const int qi = p / kGroups, h = p % kGroups;
    if (qi < nq) {
      const float den = sm.den[p];
      const float inv = den > 0.0f ? 1.0f / den : 0.0f;
      ctx[(size_t)(q0 + qi) * kHidden + (g * kGroups + h) * kHeadDim + d] = acc[i] * inv;
    }
  }
}

}  // namespace

size_t attn_partial_floats(int nt, int max_len) {
  const int max_chunks = (max_len + kChunk - 1) / kChunk;
  return (size_t)nt * kKvHeads * max_chunks * kGroups * kPartStride;
}

cudaError_t launch_decode_attention(const float* q, KvView kv, DecodeTokens tok, int max_len, float* ctx,
                                    float* scratch, unsigned* counters, cudaStream_t s, bool pdl) {
  const int max_chunks = (max_len + kChunk - 1) / kChunk;
  return launch_k(decode_attn_kernel, dim3(max_chunks, kKvHeads, tok.nt), dim3(64), 0, s, pdl, q, kv, tok,
                  max_chunks, ctx, scratch, counters);
}

cudaError_t launch_prefill_attention(const float* q, const float* k_cache, const float* v_cache, int S, float* ctx,
                                     cudaStream_t s) {
  const size_t smem = sizeof(PrefillSmem);
  cudaError_t e = cudaFuncSetAttribute(prefill_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  prefill_attn_kernel<<<dim3((S + kPQ - 1) / kPQ, kKvHeads), 256, smem, s>>>(q, k_cache, v_cache, S, ctx);
  return cudaGetLastError();
}

}  // namespace qb
