// GQA attention kernels (12 query heads over 2 KV heads, head_dim 128).
//
// Decode (hls/decode_only/qwen_decode_attention_kernel.cpp:113-162): the reference makes two passes over
// the whole history (max, then expf(s - max)). Here the history is split into 64-token chunks, one CTA
// per (token, KV head, chunk) handling the 6 query heads that share the KV head, so each K/V row is read
// once for all six. The chunk's K and V rows are staged in shared memory with all loads in flight at
// once (history rows before the grid-dependency wait, the new row after it). Each chunk keeps its own
// max; the last CTA of a (token, KV head) to finish merges the chunks in chunk order (rescaling by
// expf(m_c - M)), so the result equals the two-pass value up to rounding and is deterministic; a history
// of one chunk writes the context directly.
//
// Prefill (hls/prefill_only/qwen_prefill_attention_kernel.cpp:204-289): approx_exp(a) * approx_exp(b) is
// not approx_exp(a + b), so online rescaling would change results; the kernel keeps the reference's two
// passes: pass 1 takes the causal max of the scaled scores, pass 2 recomputes each score and accumulates
// approx_exp(score * scale - max). Scores, max and every exp value are bit-identical to the reference;
// only the order of the denominator and context sums differs.
#include "qwen_kernels.cuh"

namespace qb {
namespace {

constexpr int kChunk = 64;                 // decode keys per CTA
constexpr int kPartStride = 2 + kHeadDim;  // m, l, acc[128]
constexpr int kAttnThreads = 128;
constexpr int kRow = kHeadDim + 4;         // padded smem row (16-byte aligned, conflict-free float4 reads)
constexpr int kMergeBatch = 8;             // chunk partials staged together by the merging CTA

static_assert(kMergeBatch * kGroups * kPartStride <= kChunk * kRow, "merge staging fits in the K tile");

struct DecodeAttnSmem {
  float ks[kChunk][kRow];  // also the merge staging area: kMergeBatch x 6 x 130 floats fit
  float qs[kGroups][kRow];
  float es[kChunk][8];  // per key: the six heads' scores, then weights (padded to 8)
  float ms[kGroups], ls[kGroups];
  bool last;
};

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  const unsigned d = (unsigned)__cvta_generic_to_shared(smem_dst);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(gmem_src) : "memory");
}

__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__device__ __forceinline__ void prefetch_l2(const void* p, unsigned bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Hint: stream `bytes` of the next kernels' weights into L2 while this latency-bound kernel runs; the
// region is split evenly over the grid's CTAs.
__device__ __forceinline__ void prefetch_region(const uint8_t* pf, size_t bytes, unsigned cta, unsigned ctas) {
  if (pf == nullptr || bytes == 0) return;
  const size_t per = ((bytes + ctas - 1) / ctas + 15) & ~size_t(15);
  const size_t b0 = (size_t)cta * per;
  const size_t b1 = min(bytes, b0 + per);
  for (size_t off = b0 + (size_t)threadIdx.x * 16384; off < b1; off += (size_t)blockDim.x * 16384)
    prefetch_l2(pf + off, (unsigned)min((size_t)16384, b1 - off));
}

__global__ void __launch_bounds__(kAttnThreads) decode_attn_kernel(const float* __restrict__ q, KvView kv,
                                                                   DecodeTokens tok, int max_chunks,
                                                                   float* __restrict__ ctx, float* __restrict__ part,
                                                                   unsigned* __restrict__ counters,
                                                                   const uint8_t* pf, size_t pf_bytes) {
  extern __shared__ float4 smem4[];
  DecodeAttnSmem& sm = *reinterpret_cast<DecodeAttnSmem*>(smem4);
  const int c = blockIdx.x, g = blockIdx.y, t = blockIdx.z;
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  prefetch_region(pf, pf_bytes, (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x,
                  gridDim.x * gridDim.y * gridDim.z);

  // Positions and history rows were written before the preceding kernel started, so they are read
  // before the grid-dependency wait; only the new row and the query depend on that kernel.
  const int L = tok.pos[t] + 1;
  const int nchunks = (L + kChunk - 1) / kChunk;
  if (c >= nchunks) return;
  const int seq = tok.seq[t];
  const int k0 = c * kChunk;
  const int n = min(kChunk, L - k0);
  const int pos = L - 1;
  // A chunk is exactly one KV page (kChunk == kPage): rows are 256 floats apart from the chunk's first row,
  // in the paged and in the flat layout, so one page-table lookup serves the whole chunk.
  static_assert(kChunk == kPage, "a decode chunk must map onto one KV page");
  const float* kbase = kv_row(kv, seq, k0, 0) + g * kHeadDim;
  const float* vbase = kv_row(kv, seq, k0, 1) + g * kHeadDim;
  const int nhist = min(n, pos - k0);  // rows of this chunk that precede the new token
  // every row of the chunk in flight at once: K by asynchronous global->shared copies, V straight into
  // registers (thread = one of the 128 dims of every key: 512 contiguous bytes per key), one wait. Keeping
  // V out of shared memory lets more CTAs share an SM.
  for (int i = tid; i < nhist * 32; i += kAttnThreads) {
    const int r = i >> 5, f = i & 31;
    cp_async16(&sm.ks[r][4 * f], kbase + (size_t)r * kKvWidth + 4 * f);
  }
  float vr[kChunk];
#pragma unroll
  for (int k = 0; k < kChunk; ++k) vr[k] = k < nhist ? __ldg(vbase + (size_t)k * kKvWidth + tid) : 0.0f;
  griddep_wait();
  const int knew = pos - k0;  // the new token's row in this chunk (if 0 <= knew < kChunk)
  float vnew = 0.0f;
  if (knew >= 0 && knew < kChunk) {
    if (tid < 32) cp_async16(&sm.ks[knew][4 * tid], kbase + (size_t)knew * kKvWidth + 4 * tid);
    vnew = vbase[(size_t)knew * kKvWidth + tid];
  }
  for (int i = tid; i < kGroups * 32; i += kAttnThreads) {
    const int h = i >> 5, f = i & 31;
    cp_async16(&sm.qs[h][4 * f], q + (size_t)t * kHidden + (g * kGroups + h) * kHeadDim + 4 * f);
  }
  cp_async_wait_all();
  __syncthreads();
  griddep_launch();

  // scores: thread = (key, three of the six heads); K read once per key pair (broadcast). Each score is
  // the sum of two 64-dim halves (FMA chains over dims 0..63 and 64..127), the order the persistent
  // decode kernel uses, so both paths round alike.
  const float scaling = kAttentionScaling;  // == float(1 / sqrt(128)), qwen_decode_attention_kernel.cpp:119
  {
    const int key = tid >> 1, h0 = (tid & 1) * 3;
    float lo[3], hi[3];
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      float s0 = 0.f, s1 = 0.f, s2 = 0.f;
#pragma unroll 8
      for (int f = 16 * half; f < 16 * half + 16; ++f) {
        const float4 kk = *reinterpret_cast<const float4*>(&sm.ks[key][4 * f]);
        const float4 a = *reinterpret_cast<const float4*>(&sm.qs[h0][4 * f]);
        const float4 b = *reinterpret_cast<const float4*>(&sm.qs[h0 + 1][4 * f]);
        const float4 d = *reinterpret_cast<const float4*>(&sm.qs[h0 + 2][4 * f]);
        s0 = fmaf(a.x, kk.x, fmaf(a.y, kk.y, fmaf(a.z, kk.z, fmaf(a.w, kk.w, s0))));
        s1 = fmaf(b.x, kk.x, fmaf(b.y, kk.y, fmaf(b.z, kk.z, fmaf(b.w, kk.w, s1))));
        s2 = fmaf(d.x, kk.x, fmaf(d.y, kk.y, fmaf(d.z, kk.z, fmaf(d.w, kk.w, s2))));
      }
      float* dst = half ? hi : lo;
      dst[0] = s0;
      dst[1] = s1;
      dst[2] = s2;
    }
    const float s0 = __fadd_rn(lo[0], hi[0]), s1 = __fadd_rn(lo[1], hi[1]), s2 = __fadd_rn(lo[2], hi[2]);
    const bool ok = key < n;
    sm.es[key][h0] = ok ? s0 * scaling : -INFINITY;
    sm.es[key][h0 + 1] = ok ? s1 * scaling : -INFINITY;
    sm.es[key][h0 + 2] = ok ? s2 * scaling : -INFINITY;
  }
  __syncthreads();
  // softmax statistics of this chunk: warp w < 3 handles heads 2w, 2w+1 over the 64 keys
  if (warp < 3) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int h = 2 * warp + j;
      const float a = sm.es[lane][h], b = sm.es[lane + 32][h];
      float m = fmaxf(a, b);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      m = fmaxf(m, -1.0e30f);  // the reference's initial max
      const float ea = lane < n ? expf(a - m) : 0.f;
      const float eb = lane + 32 < n ? expf(b - m) : 0.f;
      sm.es[lane][h] = ea;
      sm.es[lane + 32][h] = eb;
      float l = ea + eb;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
      if (lane == 0) {
        sm.ms[h] = m;
        sm.ls[h] = l;
      }
    }
  }
  __syncthreads();
  // P.V: thread = one of the 128 dims, six heads
  float acc[kGroups];
#pragma unroll
  for (int h = 0; h < kGroups; ++h) acc[h] = 0.f;
#pragma unroll
  for (int key = 0; key < kChunk; ++key) {
    if (key >= n) break;
    const float vv = key == knew ? vnew : vr[key];
    const float4 e03 = *reinterpret_cast<const float4*>(&sm.es[key][0]);
    const float2 e45 = *reinterpret_cast<const float2*>(&sm.es[key][4]);
    acc[0] = fmaf(e03.x, vv, acc[0]);
    acc[1] = fmaf(e03.y, vv, acc[1]);
    acc[2] = fmaf(e03.z, vv, acc[2]);
    acc[3] = fmaf(e03.w, vv, acc[3]);
    acc[4] = fmaf(e45.x, vv, acc[4]);
    acc[5] = fmaf(e45.y, vv, acc[5]);
  }
  float* out_base = ctx + (size_t)t * kHidden + g * kGroups * kHeadDim + tid;
  if (nchunks == 1) {
#pragma unroll
    for (int h = 0; h < kGroups; ++h) {
      const float inv = sm.ls[h] > 0.0f ? 1.0f / sm.ls[h] : 0.0f;
      out_base[h * kHeadDim] = acc[h] * inv;
    }
    return;
  }
  float* my = part + (((size_t)t * kKvHeads + g) * max_chunks + c) * kGroups * kPartStride;
#pragma unroll
  for (int h = 0; h < kGroups; ++h) my[h * kPartStride + 2 + tid] = acc[h];
  if (tid < kGroups) {
    my[tid * kPartStride + 0] = sm.ms[tid];
    my[tid * kPartStride + 1] = sm.ls[tid];
  }
  // One gpu-scope acquire-release add by one thread publishes the whole CTA's partial (the barrier orders
  // the other threads' writes before it) and, for the last CTA, acquires every other CTA's partial.
  __syncthreads();
  if (tid == 0) {
    unsigned prev;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(&counters[t * kKvHeads + g])
                 : "memory");
    sm.last = (prev == (unsigned)nchunks - 1u);
  }
  __syncthreads();
  if (!sm.last) return;
  // Merge this (token, KV head)'s chunks in chunk order, online (deterministic, the same operations as the
  // persistent decode kernel): M' = max(M, m_c), o = o e^(M - M') + acc_c e^(m_c - M'), L likewise.
  const float* base = part + ((size_t)t * kKvHeads + g) * max_chunks * kGroups * kPartStride;
  float o[kGroups], Lsum[kGroups], M[kGroups];
#pragma unroll
  for (int h = 0; h < kGroups; ++h) {
    o[h] = 0.f;
    Lsum[h] = 0.f;
    M[h] = -INFINITY;
  }
  // the partials of kMergeBatch chunks at a time are staged in shared memory (the K tile space, free now)
  // with all loads in flight together, then merged one chunk after the other
  float* stg = &sm.ks[0][0];
  for (int c0 = 0; c0 < nchunks; c0 += kMergeBatch) {
    const int nb = min(kMergeBatch, nchunks - c0);
    __syncthreads();
    const float* src = base + (size_t)c0 * kGroups * kPartStride;
    for (int i = tid; i < nb * kGroups * kPartStride; i += kAttnThreads) stg[i] = __ldcg(src + i);
    __syncthreads();
    for (int cc = 0; cc < nb; ++cc) {
      const float* pc = stg + cc * kGroups * kPartStride;
#pragma unroll
      for (int h = 0; h < kGroups; ++h) {
        const float mv = pc[h * kPartStride], lv = pc[h * kPartStride + 1], av = pc[h * kPartStride + 2 + tid];
        const float Mn = fmaxf(M[h], mv);
        const float sa = expf(M[h] - Mn), sb = expf(mv - Mn);
        o[h] = __fadd_rn(__fmul_rn(o[h], sa), __fmul_rn(av, sb));
        Lsum[h] = __fadd_rn(__fmul_rn(Lsum[h], sa), __fmul_rn(lv, sb));
        M[h] = Mn;
      }
    }
  }
#pragma unroll
  for (int h = 0; h < kGroups; ++h) {
    const float inv = Lsum[h] > 0.0f ? 1.0f / Lsum[h] : 0.0f;
    out_base[h * kHeadDim] = o[h] * inv;
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
                                                           float* __restrict__ ctx, const int* only_if) {
  if (only_if != nullptr && *reinterpret_cast<const volatile int*>(only_if) == 0) return;
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
                                    float* scratch, unsigned* counters, cudaStream_t s, bool pdl,
                                    const void* prefetch, size_t prefetch_bytes) {
  const int max_chunks = (max_len + kChunk - 1) / kChunk;
  const size_t smem = sizeof(DecodeAttnSmem);
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(decode_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  return launch_k(decode_attn_kernel, dim3(max_chunks, kKvHeads, tok.nt), dim3(kAttnThreads), smem, s, pdl, q, kv,
                  tok, max_chunks, ctx, scratch, counters, static_cast<const uint8_t*>(prefetch), prefetch_bytes);
}

cudaError_t launch_prefill_attention(const float* q, const float* k_cache, const float* v_cache, int S, float* ctx,
                                     cudaStream_t s) {
  const size_t smem = sizeof(PrefillSmem);
  cudaError_t e = cudaFuncSetAttribute(prefill_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  prefill_attn_kernel<<<dim3((S + kPQ - 1) / kPQ, kKvHeads), 256, smem, s>>>(q, k_cache, v_cache, S, ctx, nullptr);
  return cudaGetLastError();
}

cudaError_t launch_prefill_attention_gated(const float* q, const float* k_cache, const float* v_cache, int S,
                                           float* ctx, const int* only_if, cudaStream_t s) {
  const size_t smem = sizeof(PrefillSmem);
  cudaError_t e = cudaFuncSetAttribute(prefill_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  prefill_attn_kernel<<<dim3((S + kPQ - 1) / kPQ, kKvHeads), 256, smem, s>>>(q, k_cache, v_cache, S, ctx, only_if);
  return cudaGetLastError();
}

}  // namespace qb
