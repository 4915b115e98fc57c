// Persistent decode kernel: one W8 decode step through all 28 decoder layers in a single cooperative
// launch, one CTA per SM.
//
// Per layer the work is the reference's decode top (hls/decode_only/qwen_decode_top_wrapper.cpp:79-112):
// q|k|v projection + RoPE + KV append, attention over the history, o_proj, gate|up + SiLU, down + the
// attention-output residual, then the caller's bf16 rounding (verification/real_host_top_backend.py:260).
// The projections use the int8 tensor-core formulation of qgemm.cu (fp32 activations written exactly as
// three int8 digits per element, int32 accumulation in TMEM), with the same arithmetic.
//
// Why one kernel: at batch 1 a layer streams 46.8 MB of int8 weights, 7 us of HBM time, split over five
// dependent steps. As separate launches every step pays launch, pipeline fill and drain. Here each CTA
// owns a fixed list of 16 KB weight units per layer (host-built schedule, balanced by units) and its
// producer warp streams them with bulk copies into a ring of shared-memory stages without ever waiting
// for activations: weights do not depend on them. While the CTA waits for the previous step's results,
// the ring keeps filling (9 x 16 KB per SM, 21 MB over the GPU), so HBM stays busy across step
// boundaries and layer boundaries.
//
// Roles (192 threads):
//   warp 0      producer: cp.async.bulk of pre-swizzled 16 KB weight units into the ring
//   warp 1      TMEM owner (32 columns = two 16-column accumulators) and MMA issuer (one lane)
//   warps 2-5   workers: wait for a step's inputs (global completion counters), build the activation
//               digits for the CTA's K blocks, read accumulators from TMEM, split-K reduction with
//               integer atomics (exact, order-free), the step's epilogue; attention chunks
// Cross-CTA dependencies are monotonic per-launch counters (tiles finished per layer and step), read with
// acquire loads in bounded spins; every CTA is resident (cooperative launch), so the spins make progress.
// Every wait gives up after ~1 s, raising an abort flag that ends all other waits quickly, and records
// the failure in the kernel error flag; the last CTA to leave clears the counters for the next launch.
#include <cuda_fp16.h>

#include <algorithm>
#include <mutex>

#include "decode_stack.h"
#include "umma_sm100.cuh"

namespace qb {
namespace stack {
namespace {

using namespace umma;

constexpr int kRing = 9;           // weight stages per CTA
constexpr int kThreads = 192;
constexpr int kWorkers = 128;
constexpr int kBarW = 1;           // named barrier of the worker warps
constexpr int kTmemCols = 32;
constexpr int kDigitBlocks = 12;   // digit buffer capacity in 128-byte K blocks
constexpr int kDigitBytes = kDigitBlocks * kDigitBlockBytes;
constexpr int kChunk = 64;         // attention keys per work item (one KV page)
constexpr int kPartStride = 2 + kHeadDim;
constexpr int kRow = kHeadDim + 4;
constexpr long long kSpinLimit = 2000000000ll;  // clock cycles, ~1 s

struct AttnSmem {
  float ks[kChunk][kRow];
  float vs[kChunk][kHeadDim];
  float qs[kGroups][kRow];
  float es[kChunk][8];
  float ms[kGroups], ls[kGroups];
};

constexpr size_t cmax(size_t x, size_t y) { return x > y ? x : y; }
// attention scratch and the two digit buffers share one region (never live at the same time)
constexpr size_t kUnionBytes = (cmax(sizeof(AttnSmem), 2 * (size_t)kDigitBytes) + 1023) / 1024 * 1024;

struct Ctrl {
  uint64_t full[kRing], empty[kRing];
  uint64_t dig_ready[2], acc_full[2], acc_empty[2];
  uint32_t tmem_base;
  int flag;
  float ys[kTileM][4];
  double red[4][4];
  float redf[4][4];
};

constexpr size_t kSmemBytes = 1024 + (size_t)kRing * kUnitBytes + kUnionBytes + sizeof(Ctrl);
static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");

// ---------------------------------------------------------------------------------------------------
// synchronisation helpers
// ---------------------------------------------------------------------------------------------------
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ unsigned ld_relaxed(const unsigned* p) {
  unsigned v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void give_up(unsigned* abort_flag) {
  atomicExch(&g_kernel_error, kErrMbarTimeout);
  atomicExch(abort_flag, 1u);
}

// Spin until *p >= target; false after the time limit or once another CTA has aborted.
__device__ bool wait_count(const unsigned* p, unsigned target, unsigned* abort_flag) {
  if (ld_acquire(p) >= target) return true;
  const long long t0 = clock64();
  while (true) {
    if (ld_acquire(p) >= target) return true;
    if (ld_relaxed(abort_flag)) return false;
    if (clock64() - t0 > kSpinLimit) {
      give_up(abort_flag);
      return false;
    }
  }
}

// mbarrier phase wait with the same limits.
__device__ bool mwait(uint64_t* bar, unsigned parity, unsigned* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  for (unsigned i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63) == 0) {
      if (ld_relaxed(abort_flag)) return false;
      if (clock64() - t0 > kSpinLimit) {
        give_up(abort_flag);
        return false;
      }
    }
  }
}

// All workers continue once *p >= target (one thread spins; the barrier releases the rest).
__device__ __forceinline__ void workers_wait(const unsigned* p, unsigned target, unsigned* abort_flag, int tid) {
  if (tid == 0) {
    wait_count(p, target, abort_flag);
    __threadfence();
  }
  named_sync(kBarW, kWorkers);
}

__device__ __forceinline__ void stamp(const Args& a, int l, int slot) {
  if (a.trace == nullptr) return;
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  a.trace[((size_t)blockIdx.x * kLayers + l) * kTraceSlots + slot] = t;
}

__device__ __forceinline__ float warp_max(float m) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  return m;
}

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src) : "memory");
}

__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// ---------------------------------------------------------------------------------------------------
// producer and MMA issuer
// ---------------------------------------------------------------------------------------------------
__device__ void producer(const Args& a, uint8_t* ring, Ctrl& cs, uint32_t i0, uint32_t i1, unsigned* abort_flag) {
  int s = 0;
  unsigned ph = 0, issued = 0, last_ph = 0;
  bool ok = true;
  for (int l = 0; l < kLayers && ok; ++l) {
    const uint8_t* wl = a.wtiles + (size_t)l * kLayerTileBytes;
    int cur = -1;
    for (uint32_t i = i0; i < i1 && ok; ++i) {
      const Item it = a.items[i];
      const uint8_t* src = wl + ((size_t)unit_base(it.stage) + (size_t)it.tile * nkb(it.stage)) * kUnitBytes;
      for (int kb = it.kb0; kb < it.kb1; ++kb) {
        if (!(ok = mwait(&cs.empty[s], ph ^ 1, abort_flag))) break;
        if (it.stage != cur) {
          cur = it.stage;
          stamp(a, l, kTraceIssue + cur);
        }
        mbar_arrive_expect_tx(&cs.full[s], kUnitBytes);
        bulk_g2s(ring + (size_t)s * kUnitBytes, src + (size_t)kb * kUnitBytes, kUnitBytes, &cs.full[s]);
        issued |= 1u << s;
        last_ph = (last_ph & ~(1u << s)) | (ph << s);
        if (++s == kRing) {
          s = 0;
          ph ^= 1;
        }
      }
    }
  }
  // no copy may still be in flight when the CTA exits
  for (int r = 0; r < kRing; ++r)
    if ((issued >> r) & 1) mbar_wait(&cs.full[r], (last_ph >> r) & 1);
}

__device__ void mma_issuer(const Args& a, uint8_t* ring, uint8_t* digits, Ctrl& cs, uint32_t tmem, uint32_t i0,
                           uint32_t i1, unsigned* abort_flag) {
  int s = 0;
  unsigned ph = 0, item_no = 0, inst = 0;
  bool ok = true;
  for (int l = 0; l < kLayers; ++l) {
    int cur = -1;
    uint32_t dbase = 0;
    for (uint32_t i = i0; i < i1; ++i) {
      const Item it = a.items[i];
      if (it.stage != cur) {  // first item of a stage: its digits must be in shared memory
        cur = it.stage;
        const unsigned p = inst & 1;
        ok = ok && mwait(&cs.dig_ready[p], (inst >> 1) & 1, abort_flag);
        fence_after();
        dbase = smem_u32(digits + (size_t)p * kDigitBytes);
        ++inst;
      }
      const unsigned b = item_no & 1;
      ok = ok && mwait(&cs.acc_empty[b], ((item_no >> 1) & 1) ^ 1, abort_flag);
      fence_after();
      const uint32_t d = tmem + b * kTileN;
      for (int kb = it.kb0; kb < it.kb1; ++kb) {
        ok = ok && mwait(&cs.full[s], ph, abort_flag);
        fence_after();
        if (ok) {
          const uint32_t abase = smem_u32(ring + (size_t)s * kUnitBytes);
          const uint32_t bbase = dbase + (uint32_t)(it.dslot + kb - it.kb0) * kDigitBlockBytes;
#pragma unroll
          for (int j = 0; j < kKBlock / 32; ++j)
            mma_i8(d, sw128_desc(abase + 32 * j), sw128_desc(bbase + 32 * j), (kb > it.kb0 || j > 0) ? 1u : 0u);
        }
        mma_commit(&cs.empty[s]);
        if (++s == kRing) {
          s = 0;
          ph ^= 1;
        }
      }
      mma_commit(&cs.acc_full[b]);
      ++item_no;
      if (i + 1 == i1 || a.items[i + 1].stage != it.stage) stamp(a, l, kTraceMma + it.stage);
    }
  }
}

// ---------------------------------------------------------------------------------------------------
// workers: activation digits
// ---------------------------------------------------------------------------------------------------
__device__ __forceinline__ void put_digits(uint8_t* blk, int t, int kk, const float (&v)[4], float step) {
  uint32_t w0 = 0, w1 = 0, w2 = 0;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int X = (int)rintf(__fdiv_rn(v[e], step));
    int d0, d1, d2;
    split_digits(X, d0, d1, d2);
    w0 |= (uint32_t)(d0 & 255) << (8 * e);
    w1 |= (uint32_t)(d1 & 255) << (8 * e);
    w2 |= (uint32_t)(d2 & 255) << (8 * e);
  }
  *reinterpret_cast<uint32_t*>(blk + sw128_offset(t, kk)) = w0;
  *reinterpret_cast<uint32_t*>(blk + sw128_offset(4 + t, kk)) = w1;
  *reinterpret_cast<uint32_t*>(blk + sw128_offset(8 + t, kk)) = w2;
}

// Digits of a whole 1536-wide row per token: x (or the embedding rows of the tokens when x is null),
// optionally RMS-normalised with norm_w (double accumulation, as the decode reference). Thread tid owns
// elements 512 j + 4 tid .. +3, j < 3.
__device__ void build_full(const Args& a, Ctrl& cs, uint8_t* dbuf, const float* x, const float* norm_w, int tid,
                           float (&step)[4]) {
  const int warp = tid >> 5, lane = tid & 31;
  for (int t = 0; t < a.nt; ++t) {
    float v[3][4];
    if (x != nullptr) {
#pragma unroll
      for (int j = 0; j < 3; ++j) {
        const float4 f = __ldcg(reinterpret_cast<const float4*>(x + (size_t)t * kHidden + 512 * j + 4 * tid));
        v[j][0] = f.x;
        v[j][1] = f.y;
        v[j][2] = f.z;
        v[j][3] = f.w;
      }
    } else {
      const int tok = __ldcg(&a.tokens[t]);
      const __half* row = reinterpret_cast<const __half*>(a.embed) + (size_t)tok * kHidden;
#pragma unroll
      for (int j = 0; j < 3; ++j) {
        const uint2 u = __ldg(reinterpret_cast<const uint2*>(row + 512 * j + 4 * tid));
        const __half2 h0 = *reinterpret_cast<const __half2*>(&u.x), h1 = *reinterpret_cast<const __half2*>(&u.y);
        v[j][0] = __low2float(h0);
        v[j][1] = __high2float(h0);
        v[j][2] = __low2float(h1);
        v[j][3] = __high2float(h1);
      }
    }
    if (norm_w != nullptr) {
      double ss = 0.0;
#pragma unroll
      for (int j = 0; j < 3; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) ss += (double)v[j][e] * (double)v[j][e];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if (lane == 0) cs.red[warp][t] = ss;
      named_sync(kBarW, kWorkers);
      const double tot = cs.red[0][t] + cs.red[1][t] + cs.red[2][t] + cs.red[3][t];
      const double inv = 1.0 / sqrt(tot / (double)kHidden + (double)kEps);
#pragma unroll
      for (int j = 0; j < 3; ++j) {
        const float4 w = __ldg(reinterpret_cast<const float4*>(norm_w + 512 * j + 4 * tid));
        v[j][0] = (float)((double)v[j][0] * inv * (double)w.x);
        v[j][1] = (float)((double)v[j][1] * inv * (double)w.y);
        v[j][2] = (float)((double)v[j][2] * inv * (double)w.z);
        v[j][3] = (float)((double)v[j][3] * inv * (double)w.w);
      }
    }
    float m = 0.0f;
#pragma unroll
    for (int j = 0; j < 3; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) m = fmaxf(m, fabsf(v[j][e]));
    m = warp_max(m);
    if (lane == 0) cs.redf[warp][t] = m;
    named_sync(kBarW, kWorkers);
    const float mx = fmaxf(fmaxf(cs.redf[0][t], cs.redf[1][t]), fmaxf(cs.redf[2][t], cs.redf[3][t]));
    const float st = mx > 0.0f ? mx / kDigitRange : 1.0f;
    step[t] = st;
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      const int k = 512 * j + 4 * tid;
      put_digits(dbuf + (size_t)(k >> 7) * kDigitBlockBytes, t, k & 127, v[j], st);
    }
  }
}

// Digits of the down projection's input h (8960 wide) for this CTA's items only; the step comes from
// max|h| gathered by the gate|up epilogues.
__device__ void build_down(const Args& a, uint8_t* dbuf, int l, uint32_t b0, uint32_t b1, int tid, float (&step)[4]) {
  for (int t = 0; t < a.nt; ++t) {
    const float mx = __uint_as_float(__ldcg(&a.sync->hmax[l][t]));
    const float st = mx > 0.0f ? mx / kDigitRange : 1.0f;
    step[t] = st;
    for (uint32_t i = b0; i < b1; ++i) {
      const Item it = a.items[i];
      const int n4 = (it.kb1 - it.kb0) * 32;
      for (int f = tid; f < n4; f += kWorkers) {
        const int k = it.kb0 * kKBlock + 4 * f;
        const float4 x = __ldcg(reinterpret_cast<const float4*>(a.h + (size_t)t * kInter + k));
        const float v[4] = {x.x, x.y, x.z, x.w};
        put_digits(dbuf + (size_t)(it.dslot + (f >> 5)) * kDigitBlockBytes, t, 4 * (f & 31), v, st);
      }
    }
  }
}

// ---------------------------------------------------------------------------------------------------
// workers: accumulator read-out, split-K reduction and the per-stage epilogues
// ---------------------------------------------------------------------------------------------------
struct WorkerCtx {
  int tid, quarter, lane, r;
  unsigned item_no;
  uint32_t tmem;
};

__device__ void item_epilogue(const Args& a, Ctrl& cs, WorkerCtx& w, const Item it, int l, const float (&step)[4],
                              unsigned* abort_flag) {
  const int nt = a.nt, r = w.r, tid = w.tid;
  const unsigned b = w.item_no & 1;
  mwait(&cs.acc_full[b], (w.item_no >> 1) & 1, abort_flag);
  __syncwarp();
  fence_after();
  int v[16];
  tmem_ld16(w.tmem + b * kTileN + ((uint32_t)(w.quarter * 32) << 16), v);
  fence_before();
  mbar_arrive(&cs.acc_empty[b]);
  ++w.item_no;
  const int s = it.stage;
  if (split(s) > 1) {
    const int at = acc_tile_base(s) + it.tile;
    int* g = a.acc + ((size_t)at * kTileM + r) * 12;
#pragma unroll
    for (int c = 0; c < 12; ++c)
      if ((c & 3) < nt) atomicAdd(&g[c], v[c]);
    __threadfence();
    named_sync(kBarW, kWorkers);
    if (tid == 0) cs.flag = atomicAdd(&a.sync->tile_cnt[at], 1u) == (unsigned)(split(s) - 1);
    named_sync(kBarW, kWorkers);
    if (!cs.flag) return;
    __threadfence();
#pragma unroll
    for (int c = 0; c < 12; ++c) {
      if ((c & 3) < nt) {
        v[c] = __ldcg(&g[c]);
        g[c] = 0;
      }
    }
    if (tid == 0) a.sync->tile_cnt[at] = 0u;
  }
  float yv[4];
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    const long long tot = (long long)v[t] + 256ll * (long long)v[4 + t] + 65536ll * (long long)v[8 + t];
    yv[t] = (float)((double)tot * (double)step[t]);
  }
  const LayerDev& L = a.layers[l];
  int done_slot = kDoneQkv;
  if (s == kQkv) {
    // tile = head (12 q, 2 k, 2 v); rotate-half pairs (r, r ^ 64) exchanged through shared memory
    const int row = it.tile * kTileM + r;
    const float bb = __ldg(L.qkv_b + row), sc = __ldg(L.qkv_s + row);
#pragma unroll
    for (int t = 0; t < 4; ++t) cs.ys[r][t] = __fmaf_rn(sc, yv[t], bb);
    named_sync(kBarW, kWorkers);
    const int h = it.tile;
    const KvView kv{a.kv_pool, nullptr, a.page_table, l, a.max_pages};
    for (int t = 0; t < nt; ++t) {
      const float mine = cs.ys[r][t], other = cs.ys[r ^ 64][t];
      float y = mine;
      const int pos = __ldcg(&a.pos[t]);
      if (h < kHeads + kKvHeads) {
        const int p = r & 63;
        const float c = __ldg(a.rope_cos + (size_t)pos * 64 + p), sn = __ldg(a.rope_sin + (size_t)pos * 64 + p);
        y = r < 64 ? __fsub_rn(__fmul_rn(mine, c), __fmul_rn(other, sn))
                   : __fadd_rn(__fmul_rn(mine, c), __fmul_rn(other, sn));
      }
      if (h < kHeads) {
        a.q[(size_t)t * kHidden + row] = y;
      } else {
        const int which = h < kHeads + kKvHeads ? 0 : 1;
        kv_row(kv, __ldcg(&a.seq[t]), pos, which)[row - kHidden - which * kKvWidth] = y;
      }
    }
    done_slot = kDoneQkv;
  } else if (s == kO) {
    const int row = it.tile * kTileM + r;
    const float sc = __ldg(L.o_s + row);
    for (int t = 0; t < nt; ++t) a.a[(size_t)t * kHidden + row] = sc * yv[t];
    done_slot = kDoneO;
  } else if (s == kGu) {
    // tile rows 0..63: gate rows 64 j.., rows 64..127: the matching up rows
    const int row = r < 64 ? it.tile * 64 + r : kInter + it.tile * 64 + (r - 64);
    const float sc = __ldg(L.gu_s + row);
#pragma unroll
    for (int t = 0; t < 4; ++t) cs.ys[r][t] = sc * yv[t];
    named_sync(kBarW, kWorkers);
    if (r < 64) {  // warps of TMEM quarters 0 and 1
      for (int t = 0; t < nt; ++t) {
        const float gv = cs.ys[r][t], uv = cs.ys[r + 64][t];
        const float silu = __fdiv_rn(gv, __fadd_rn(1.0f, expf(-gv)));
        const float hv = __fmul_rn(silu, uv);
        a.h[(size_t)t * kInter + it.tile * 64 + r] = hv;
        const float m = warp_max(fabsf(hv));
        if (w.lane == 0) atomicMax(&a.sync->hmax[l][t], __float_as_uint(m));
      }
    }
    done_slot = kDoneGu;
  } else {
    const int row = it.tile * kTileM + r;
    const float sc = __ldg(L.down_s + row);
    float* yout = (l & 1) ? a.y1 : a.y0;
    for (int t = 0; t < nt; ++t) {
      float y = __fadd_rn(__ldcg(&a.a[(size_t)t * kHidden + row]), sc * yv[t]);
      y = round_bf16(y);
      yout[(size_t)t * kHidden + row] = y;
      if (a.dump != nullptr) a.dump[((size_t)l * nt + t) * kHidden + row] = y;
    }
    done_slot = kDoneDown;
  }
  __threadfence();
  named_sync(kBarW, kWorkers);
  if (tid == 0) atomicAdd(&a.sync->done[l][done_slot], 1u);
}

// ---------------------------------------------------------------------------------------------------
// workers: attention (hls/decode_only/qwen_decode_attention_kernel.cpp:113-162), one 64-key chunk of one
// (token, KV head) per item; chunk partials merged in chunk order by the last chunk to finish.
// ---------------------------------------------------------------------------------------------------
__device__ void attn_item(const Args& a, AttnSmem& sm, Ctrl& cs, int l, int t, int g, int c, int nchunks, int tid) {
  const int warp = tid >> 5, lane = tid & 31;
  const int L = __ldcg(&a.pos[t]) + 1;
  const int seq = __ldcg(&a.seq[t]);
  const int k0 = c * kChunk;
  const int n = min(kChunk, L - k0);
  const KvView kv{a.kv_pool, nullptr, a.page_table, l, a.max_pages};
  static_assert(kChunk == kPage, "an attention chunk must map onto one KV page");
  const float* kbase = kv_row(kv, seq, k0, 0) + g * kHeadDim;
  const float* vbase = kv_row(kv, seq, k0, 1) + g * kHeadDim;
  named_sync(kBarW, kWorkers);  // the previous item is done with the shared buffers
  for (int i = tid; i < n * 32; i += kWorkers) {
    const int rr = i >> 5, f = i & 31;
    cp_async16(&sm.ks[rr][4 * f], kbase + (size_t)rr * kKvWidth + 4 * f);
    cp_async16(&sm.vs[rr][4 * f], vbase + (size_t)rr * kKvWidth + 4 * f);
  }
  for (int i = tid; i < kGroups * 32; i += kWorkers) {
    const int hh = i >> 5, f = i & 31;
    cp_async16(&sm.qs[hh][4 * f], a.q + (size_t)t * kHidden + (g * kGroups + hh) * kHeadDim + 4 * f);
  }
  cp_async_wait_all();
  named_sync(kBarW, kWorkers);
  const float scaling = kAttentionScaling;
  {
    const int key = tid >> 1, h0 = (tid & 1) * 3;
    float s0 = 0.f, s1 = 0.f, s2 = 0.f;
#pragma unroll 8
    for (int f = 0; f < 32; ++f) {
      const float4 kk = *reinterpret_cast<const float4*>(&sm.ks[key][4 * f]);
      const float4 x0 = *reinterpret_cast<const float4*>(&sm.qs[h0][4 * f]);
      const float4 x1 = *reinterpret_cast<const float4*>(&sm.qs[h0 + 1][4 * f]);
      const float4 x2 = *reinterpret_cast<const float4*>(&sm.qs[h0 + 2][4 * f]);
      s0 = fmaf(x0.x, kk.x, fmaf(x0.y, kk.y, fmaf(x0.z, kk.z, fmaf(x0.w, kk.w, s0))));
      s1 = fmaf(x1.x, kk.x, fmaf(x1.y, kk.y, fmaf(x1.z, kk.z, fmaf(x1.w, kk.w, s1))));
      s2 = fmaf(x2.x, kk.x, fmaf(x2.y, kk.y, fmaf(x2.z, kk.z, fmaf(x2.w, kk.w, s2))));
    }
    const bool ok = key < n;
    sm.es[key][h0] = ok ? s0 * scaling : -INFINITY;
    sm.es[key][h0 + 1] = ok ? s1 * scaling : -INFINITY;
    sm.es[key][h0 + 2] = ok ? s2 * scaling : -INFINITY;
  }
  named_sync(kBarW, kWorkers);
  if (warp < 3) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int hh = 2 * warp + j;
      const float x0 = sm.es[lane][hh], x1 = sm.es[lane + 32][hh];
      float m = warp_max(fmaxf(x0, x1));
      m = fmaxf(m, -1.0e30f);  // the reference's initial max
      const float e0 = lane < n ? expf(x0 - m) : 0.f;
      const float e1 = lane + 32 < n ? expf(x1 - m) : 0.f;
      sm.es[lane][hh] = e0;
      sm.es[lane + 32][hh] = e1;
      float s = e0 + e1;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (lane == 0) {
        sm.ms[hh] = m;
        sm.ls[hh] = s;
      }
    }
  }
  named_sync(kBarW, kWorkers);
  float acc[kGroups];
#pragma unroll
  for (int hh = 0; hh < kGroups; ++hh) acc[hh] = 0.f;
#pragma unroll 4
  for (int key = 0; key < n; ++key) {
    const float vv = sm.vs[key][tid];
    const float4 e03 = *reinterpret_cast<const float4*>(&sm.es[key][0]);
    const float2 e45 = *reinterpret_cast<const float2*>(&sm.es[key][4]);
    acc[0] = fmaf(e03.x, vv, acc[0]);
    acc[1] = fmaf(e03.y, vv, acc[1]);
    acc[2] = fmaf(e03.z, vv, acc[2]);
    acc[3] = fmaf(e03.w, vv, acc[3]);
    acc[4] = fmaf(e45.x, vv, acc[4]);
    acc[5] = fmaf(e45.y, vv, acc[5]);
  }
  float* out_base = a.ctx + (size_t)t * kHidden + g * kGroups * kHeadDim + tid;
  bool finished = false;
  if (nchunks == 1) {
#pragma unroll
    for (int hh = 0; hh < kGroups; ++hh) {
      const float inv = sm.ls[hh] > 0.0f ? 1.0f / sm.ls[hh] : 0.0f;
      out_base[hh * kHeadDim] = acc[hh] * inv;
    }
    finished = true;
  } else {
    float* my = a.attn_part + (((size_t)t * kKvHeads + g) * a.attn_max_chunks + c) * kGroups * kPartStride;
#pragma unroll
    for (int hh = 0; hh < kGroups; ++hh) my[hh * kPartStride + 2 + tid] = acc[hh];
    if (tid < kGroups) {
      my[tid * kPartStride + 0] = sm.ms[tid];
      my[tid * kPartStride + 1] = sm.ls[tid];
    }
    __threadfence();
    named_sync(kBarW, kWorkers);
    if (tid == 0) cs.flag = atomicAdd(&a.sync->attn_cnt[t][g], 1u) == (unsigned)nchunks - 1u;
    named_sync(kBarW, kWorkers);
    if (cs.flag) {
      __threadfence();
      const float* base = a.attn_part + ((size_t)t * kKvHeads + g) * a.attn_max_chunks * kGroups * kPartStride;
      float o[kGroups], Lsum[kGroups], M[kGroups];
#pragma unroll
      for (int hh = 0; hh < kGroups; ++hh) {
        o[hh] = 0.f;
        Lsum[hh] = 0.f;
        M[hh] = -INFINITY;
      }
      for (int cc = 0; cc < nchunks; ++cc) {
#pragma unroll
        for (int hh = 0; hh < kGroups; ++hh) M[hh] = fmaxf(M[hh], __ldcg(&base[(cc * kGroups + hh) * kPartStride]));
      }
      for (int c0 = 0; c0 < nchunks; c0 += kChunk) {
        const int cn = min(kChunk, nchunks - c0);
        named_sync(kBarW, kWorkers);
        for (int i = tid; i < cn * kGroups; i += kWorkers) {
          const int cc = i / kGroups, hh = i % kGroups;
          const float* pc = base + ((c0 + cc) * kGroups + hh) * kPartStride;
          const float wgt = expf(__ldcg(&pc[0]) - M[hh]);
          sm.es[cc][hh] = wgt;
          sm.vs[cc][hh] = __ldcg(&pc[1]) * wgt;
        }
        named_sync(kBarW, kWorkers);
#pragma unroll 4
        for (int cc = 0; cc < cn; ++cc) {
          const float* pc = base + (size_t)(c0 + cc) * kGroups * kPartStride + 2 + tid;
#pragma unroll
          for (int hh = 0; hh < kGroups; ++hh) {
            o[hh] = fmaf(__ldcg(&pc[hh * kPartStride]), sm.es[cc][hh], o[hh]);
            Lsum[hh] += sm.vs[cc][hh];
          }
        }
      }
#pragma unroll
      for (int hh = 0; hh < kGroups; ++hh) {
        const float inv = Lsum[hh] > 0.0f ? 1.0f / Lsum[hh] : 0.0f;
        out_base[hh * kHeadDim] = o[hh] * inv;
      }
      if (tid == 0) a.sync->attn_cnt[t][g] = 0u;
      finished = true;
    }
  }
  if (finished) {  // uniform across the workers
    __threadfence();
    named_sync(kBarW, kWorkers);
    if (tid == 0) atomicAdd(&a.sync->done[l][kDoneAttn], 1u);
  }
}

__device__ void attention_stage(const Args& a, AttnSmem& sm, Ctrl& cs, int l, int tid, unsigned* abort_flag) {
  int nch[4] = {0, 0, 0, 0}, total = 0;
  for (int t = 0; t < a.nt; ++t) {
    nch[t] = (__ldcg(&a.pos[t]) + 1 + kChunk - 1) / kChunk;
    total += kKvHeads * nch[t];
  }
  if ((int)blockIdx.x >= total) return;
  workers_wait(&a.sync->done[l][kDoneQkv], (unsigned)tiles(kQkv), abort_flag, tid);
  if (tid == 0) stamp(a, l, kTraceWait + 1);
  for (int i = blockIdx.x; i < total; i += gridDim.x) {
    int t = 0, rem = i;
    while (rem >= kKvHeads * nch[t]) {
      rem -= kKvHeads * nch[t];
      ++t;
    }
    attn_item(a, sm, cs, l, t, rem / nch[t], rem % nch[t], nch[t], tid);
  }
  if (tid == 0) stamp(a, l, kTraceDone + 1);
}

__device__ void workers(const Args& a, uint8_t* uni, Ctrl& cs, uint32_t tmem, uint32_t i0, uint32_t i1,
                        unsigned* abort_flag) {
  WorkerCtx w;
  w.tid = threadIdx.x - 64;
  w.lane = threadIdx.x & 31;
  w.quarter = (threadIdx.x >> 5) & 3;  // TMEM lanes this warp may read
  w.r = w.quarter * 32 + w.lane;
  w.item_no = 0;
  w.tmem = tmem;
  uint32_t sb[kNumProj], se[kNumProj];
  for (int s = 0; s < kNumProj; ++s) sb[s] = se[s] = i0;
  for (uint32_t i = i0; i < i1; ++i) {
    const int s = a.items[i].stage;
    if (se[s] == sb[s]) sb[s] = i;
    se[s] = i + 1;
  }
  unsigned inst = 0;
  float step[4] = {1.f, 1.f, 1.f, 1.f};
  AttnSmem& asm_ = *reinterpret_cast<AttnSmem*>(uni);
  auto digits = [&](unsigned j) { return uni + (size_t)(j & 1) * kDigitBytes; };
  auto ready = [&]() {
    fence_async_smem();
    mbar_arrive(&cs.dig_ready[inst & 1]);
    ++inst;
  };
  const bool tr = w.tid == 0;
  for (int l = 0; l < kLayers; ++l) {
    const LayerDev& L = a.layers[l];
    unsigned* done = a.sync->done[l];
    // q|k|v (input: previous layer's output, or the token embeddings)
    if (sb[kQkv] < se[kQkv]) {
      if (l > 0) workers_wait(&a.sync->done[l - 1][kDoneDown], (unsigned)tiles(kDown), abort_flag, w.tid);
      if (tr) stamp(a, l, kTraceWait + 0);
      const float* xin = l == 0 ? nullptr : (((l - 1) & 1) ? a.y1 : a.y0);
      build_full(a, cs, digits(inst), xin, L.input_ln, w.tid, step);
      ready();
      if (tr) stamp(a, l, kTraceBuilt + 0);
      for (uint32_t i = sb[kQkv]; i < se[kQkv]; ++i) item_epilogue(a, cs, w, a.items[i], l, step, abort_flag);
      if (tr) stamp(a, l, kTraceDone + 0);
    }
    attention_stage(a, asm_, cs, l, w.tid, abort_flag);
    if (sb[kO] < se[kO]) {
      workers_wait(&done[kDoneAttn], (unsigned)(kKvHeads * a.nt), abort_flag, w.tid);
      if (tr) stamp(a, l, kTraceWait + 2);
      build_full(a, cs, digits(inst), a.ctx, nullptr, w.tid, step);
      ready();
      if (tr) stamp(a, l, kTraceBuilt + 2);
      for (uint32_t i = sb[kO]; i < se[kO]; ++i) item_epilogue(a, cs, w, a.items[i], l, step, abort_flag);
      if (tr) stamp(a, l, kTraceDone + 2);
    }
    if (sb[kGu] < se[kGu]) {
      workers_wait(&done[kDoneO], (unsigned)tiles(kO), abort_flag, w.tid);
      if (tr) stamp(a, l, kTraceWait + 3);
      build_full(a, cs, digits(inst), a.a, L.post_ln, w.tid, step);
      ready();
      if (tr) stamp(a, l, kTraceBuilt + 3);
      for (uint32_t i = sb[kGu]; i < se[kGu]; ++i) item_epilogue(a, cs, w, a.items[i], l, step, abort_flag);
      if (tr) stamp(a, l, kTraceDone + 3);
    }
    if (sb[kDown] < se[kDown]) {
      workers_wait(&done[kDoneGu], (unsigned)tiles(kGu), abort_flag, w.tid);
      if (tr) stamp(a, l, kTraceWait + 4);
      build_down(a, digits(inst), l, sb[kDown], se[kDown], w.tid, step);
      ready();
      if (tr) stamp(a, l, kTraceBuilt + 4);
      for (uint32_t i = sb[kDown]; i < se[kDown]; ++i) item_epilogue(a, cs, w, a.items[i], l, step, abort_flag);
      if (tr) stamp(a, l, kTraceDone + 4);
    }
  }
}

__global__ void __launch_bounds__(kThreads, 1) decode_stack_kernel(const __grid_constant__ Args a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = base;
  uint8_t* uni = base + (size_t)kRing * kUnitBytes;
  Ctrl& cs = *reinterpret_cast<Ctrl*>(uni + kUnionBytes);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t i0 = a.item_off[blockIdx.x], i1 = a.item_off[blockIdx.x + 1];
  unsigned* abort_flag = &a.sync->abort_flag;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kRing; ++s) {
      mbar_init(&cs.full[s], 1);
      mbar_init(&cs.empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&cs.dig_ready[b], kWorkers);
      mbar_init(&cs.acc_full[b], 1);
      mbar_init(&cs.acc_empty[b], kWorkers);
    }
    mbar_fence_init();
  }
  if (warp == 1) tmem_alloc(&cs.tmem_base, kTmemCols);
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = cs.tmem_base;

  if (warp == 0) {
    if (lane == 0) producer(a, ring, cs, i0, i1, abort_flag);
  } else if (warp == 1) {
    if (lane == 0) mma_issuer(a, ring, uni, cs, tmem, i0, i1, abort_flag);
  } else {
    workers(a, uni, cs, tmem, i0, i1, abort_flag);
  }

  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned prev = atomicAdd(&a.sync->exit_cnt, 1u);
    if (prev == gridDim.x - 1) {  // every CTA is past its last wait: clear the words for the next launch
      __threadfence();
      unsigned* wds = reinterpret_cast<unsigned*>(a.sync);
      for (size_t i = 0; i < sizeof(SyncWords) / 4; ++i) wds[i] = 0u;
      __threadfence();
    }
  }
}

// One 16 KB unit per CTA: rows of the DDR-image matrix into the 128-byte-swizzled tile layout.
__global__ void tile_layer_kernel(LayerDev L, uint8_t* __restrict__ dst) {
  const int u = blockIdx.x;
  const int s = u < unit_base(kO) ? kQkv : u < unit_base(kGu) ? kO : u < unit_base(kDown) ? kGu : kDown;
  const int rel = u - unit_base(s);
  const int tile = rel / nkb(s), kb = rel % nkb(s);
  for (int i = threadIdx.x; i < kTileM * 8; i += blockDim.x) {
    const int r = i >> 3, c = i & 7;
    const uint8_t* src;
    if (s == kQkv) src = L.qkv_w + (size_t)(tile * kTileM + r) * kHidden;
    else if (s == kO) src = L.o_w + (size_t)(tile * kTileM + r) * kHidden;
    else if (s == kGu) src = L.gu_w + (size_t)(r < 64 ? tile * 64 + r : kInter + tile * 64 + (r - 64)) * kHidden;
    else src = L.down_w + (size_t)(tile * kTileM + r) * kInter;
    const uint4 v = *reinterpret_cast<const uint4*>(src + (size_t)kb * kKBlock + c * 16);
    *reinterpret_cast<uint4*>(dst + (size_t)u * kUnitBytes + sw128_offset(r, c * 16)) = v;
  }
}

}  // namespace

Schedule build_schedule(int ctas) {
  struct Cand {
    int stage, tile, seg, kb0, kb1;
  };
  std::vector<Cand> all;
  for (int s = 0; s < kNumProj; ++s)
    for (int tile = 0; tile < tiles(s); ++tile)
      for (int seg = 0; seg < split(s); ++seg) {
        const int kb0 = seg * seg_blocks(s), kb1 = std::min(nkb(s), kb0 + seg_blocks(s));
        if (kb0 < kb1) all.push_back({s, tile, seg, kb0, kb1});
      }
  // largest items first onto the least-loaded CTA (load = 16 KB units streamed per layer)
  std::stable_sort(all.begin(), all.end(), [](const Cand& x, const Cand& y) { return x.kb1 - x.kb0 > y.kb1 - y.kb0; });
  std::vector<int> load(ctas, 0), down_blocks(ctas, 0);
  std::vector<std::vector<Cand>> per(ctas);
  for (const Cand& c : all) {
    const int units = c.kb1 - c.kb0;
    int best = -1;
    for (int k = 0; k < ctas; ++k) {
      if (c.stage == kDown && down_blocks[k] + units > kDigitBlocks) continue;
      if (best < 0 || load[k] < load[best]) best = k;
    }
    per[best].push_back(c);
    load[best] += units;
    if (c.stage == kDown) down_blocks[best] += units;
  }
  Schedule sc;
  sc.off.push_back(0);
  for (int k = 0; k < ctas; ++k) {
    std::sort(per[k].begin(), per[k].end(), [](const Cand& x, const Cand& y) {
      return x.stage != y.stage ? x.stage < y.stage : x.tile != y.tile ? x.tile < y.tile : x.seg < y.seg;
    });
    int dslot = 0;
    for (const Cand& c : per[k]) {
      Item it;
      it.tile = (uint16_t)c.tile;
      it.stage = (uint8_t)c.stage;
      it.kb0 = (uint8_t)c.kb0;
      it.kb1 = (uint8_t)c.kb1;
      if (c.stage == kDown) {
        it.dslot = (uint8_t)dslot;
        dslot += c.kb1 - c.kb0;
      } else {
        it.dslot = (uint8_t)c.kb0;  // full-row digits: block kb at slot kb
      }
      it.seg = (uint16_t)c.seg;
      sc.items.push_back(it);
    }
    sc.off.push_back((uint32_t)sc.items.size());
    sc.max_units = std::max(sc.max_units, load[k]);
  }
  return sc;
}

size_t decode_stack_smem() { return kSmemBytes; }

cudaError_t launch_decode_stack(const Args& a, int ctas, cudaStream_t s) {
  static std::mutex mu;
  static unsigned long long attr_set = 0;  // per device
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (dev < 64 && !((attr_set >> dev) & 1ull)) {
      e = cudaFuncSetAttribute(decode_stack_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
      if (e != cudaSuccess) return e;
      attr_set |= 1ull << dev;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ctas);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeCooperative;
  at[0].val.cooperative = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, decode_stack_kernel, a);
}

cudaError_t launch_tile_layer(const LayerDev& L, uint8_t* dst, cudaStream_t s) {
  tile_layer_kernel<<<kUnitsPerLayer, 256, 0, s>>>(L, dst);
  return cudaGetLastError();
}

unsigned decode_stack_kernel_error(bool reset) {
  unsigned v = 0;
  if (cudaMemcpyFromSymbol(&v, g_kernel_error, sizeof(v)) != cudaSuccess) return 0xFFFFFFFFu;
  if (reset && v) {
    const unsigned z = 0;
    cudaMemcpyToSymbol(g_kernel_error, &z, sizeof(z));
  }
  return v;
}

}  // namespace stack
}  // namespace qb
