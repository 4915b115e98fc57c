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
// Roles (224 threads):
//   warp 0      producer: cp.async.bulk of pre-swizzled 16 KB weight units into the ring
//   warps 1, 6  MMA issuers (one lane each), alternate 16 KB units of an item into their own accumulators;
//               warp 1 also owns the TMEM allocation (64 columns: two items in flight x two 16-column parts)
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

static_assert(kKBlock == 4 * 32, "one 128-byte K block = four kind::i8 MMAs of K = 32 bytes");
constexpr int kRing = 9;           // weight stages per CTA (shared memory); Args::ring uses 2..kRing of them
constexpr int kThreads = 224;      // producer, MMA issuer, 4 worker warps, second MMA issuer
constexpr int kWorkers = 128;
constexpr int kBarW = 1;           // named barrier of the worker warps
// Two MMA-issuing warps (1 and 6) take alternate 16 KB units of an item, each into its own accumulator
// (summed when read out): one thread's wait-on-data and commit latencies then overlap the other's MMAs
// (measured on B200: 491 -> ~260 cycles per unit). Two items in flight: 2 x 2 x 16 TMEM columns.
constexpr int kIssuers = 2;
constexpr int kAccParts = kIssuers;
constexpr int kTmemCols = 2 * kAccParts * kTileN;
constexpr int kDigitBlocks = 12;   // digit buffer capacity in 128-byte K blocks
constexpr int kDigitBytes = kDigitBlocks * kDigitBlockBytes;
constexpr int kChunk = 64;         // attention keys per work item (one KV page)
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

// Completion signals: the workers' writes are ordered before one thread's release operation by a CTA
// barrier, so a single gpu-scope release (instead of a fence in every thread) publishes all of them; the
// waiting side acquires with one thread and releases its workers with a barrier.
__device__ __forceinline__ void red_release(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned atom_add_acq_rel(unsigned* p, unsigned v) {
  unsigned old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

__device__ __forceinline__ void give_up(unsigned* abort_flag) {
  atomicExch(&g_kernel_error, kErrMbarTimeout);
  atomicExch(abort_flag, 1u);
}

// Spin until *p >= target; false after the time limit or once another CTA has aborted.
__device__ __forceinline__ void fence_acquire() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

__device__ bool wait_count(const unsigned* p, unsigned target, unsigned* abort_flag) {
  if (ld_acquire(p) >= target) return true;
  const long long t0 = clock64();
  while (true) {
    if (ld_relaxed(p) >= target) {
      fence_acquire();
      return true;
    }
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
  if (tid == 0) wait_count(p, target, abort_flag);
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

__device__ __forceinline__ int ring_depth(const Args& a) { return a.ring < 2 ? 2 : a.ring > kRing ? kRing : a.ring; }

// ---------------------------------------------------------------------------------------------------
// producer and MMA issuer
// ---------------------------------------------------------------------------------------------------
__device__ void producer(const Args& a, uint8_t* ring_smem, Ctrl& cs, uint32_t i0, uint32_t i1,
                         unsigned* abort_flag) {
  const int ring = ring_depth(a);
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
        bulk_g2s(ring_smem + (size_t)s * kUnitBytes, src + (size_t)kb * kUnitBytes, kUnitBytes, &cs.full[s]);
        issued |= 1u << s;
        last_ph = (last_ph & ~(1u << s)) | (ph << s);
        if (++s == ring) {
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

__device__ void mma_issuer(const Args& a, uint8_t* ring_smem, uint8_t* digits, Ctrl& cs, uint32_t tmem, uint32_t i0,
                           uint32_t i1, unsigned* abort_flag, int issuer) {
  const int ring = ring_depth(a);
  int s = 0;
  unsigned ph = 0, item_no = 0, inst = 0;
  bool ok = true;
  // Descriptors are built once; a unit / digit block / 32-byte K step only moves the start-address field
  // (16-byte units, far from overflowing its 14 bits inside shared memory).
  const uint64_t ring_desc = sw128_desc(smem_u32(ring_smem));
  constexpr uint64_t kUnitStep = kUnitBytes >> 4, kBlockStep = kDigitBlockBytes >> 4, kKStep = 32 >> 4;
  for (int l = 0; l < kLayers; ++l) {
    int cur = -1;
    uint64_t dig_desc = 0;
    for (uint32_t i = i0; i < i1; ++i) {
      const Item it = a.items[i];
      if (it.stage != cur) {  // first item of a stage: its digits must be in shared memory
        cur = it.stage;
        const unsigned p = inst & 1;
        ok = ok && mwait(&cs.dig_ready[p], (inst >> 1) & 1, abort_flag);
        fence_after();
        if (issuer == 0) stamp(a, l, kTraceMmaStart + cur);
        if (a.trace != nullptr && issuer == 0)  // SM clock at the same point, to relate the unit times
          a.trace[((size_t)blockIdx.x * kLayers + l) * kTraceSlots + 36 + (cur == kGu ? 1 : cur == kDown ? 2 : 3)] =
              (unsigned long long)clock64();
        dig_desc = sw128_desc(smem_u32(digits + (size_t)p * kDigitBytes));
        ++inst;
      }
      const unsigned b = item_no & 1;
      ok = ok && mwait(&cs.acc_empty[b], ((item_no >> 1) & 1) ^ 1, abort_flag);
      fence_after();
      const uint32_t d = tmem + b * (kAccParts * kTileN) + issuer * kTileN;
      uint64_t bd = dig_desc + (uint64_t)it.dslot * kBlockStep;
      for (int kb = it.kb0; kb < it.kb1; ++kb, bd += kBlockStep) {
        const int u = kb - it.kb0;
        if (u % kIssuers == issuer) {  // this issuer's unit; the ring position advances for every unit
          ok = ok && mwait(&cs.full[s], ph, abort_flag);
          fence_after();
          if (a.trace != nullptr && u < 12 && (it.stage == kGu || it.stage == kDown))  // SM clock, not global time
            a.trace[((size_t)blockIdx.x * kLayers + l) * kTraceSlots + kTraceUnit + (it.stage == kGu ? 0 : 12) + u] =
                (unsigned long long)clock64();
          if (ok) {
            const uint64_t ad = ring_desc + (uint64_t)s * kUnitStep;
            mma_i8(d, ad, bd, u >= kIssuers ? 1u : 0u);
            mma_i8_acc(d, ad + kKStep, bd + kKStep);
            mma_i8_acc(d, ad + 2 * kKStep, bd + 2 * kKStep);
            mma_i8_acc(d, ad + 3 * kKStep, bd + 3 * kKStep);
          }
          mma_commit(&cs.empty[s]);
        }
        if (++s == ring) {
          s = 0;
          ph ^= 1;
        }
      }
      mma_commit(&cs.acc_full[b]);
      ++item_no;
      if (issuer == 0 && (i + 1 == i1 || a.items[i + 1].stage != it.stage)) stamp(a, l, kTraceMma + it.stage);
    }
  }
}

// ---------------------------------------------------------------------------------------------------
// workers: activation digits
// ---------------------------------------------------------------------------------------------------
__device__ __forceinline__ void put_digits(uint8_t* blk, int t, int kk, const float (&v)[4], double r) {
  uint32_t w0 = 0, w1 = 0, w2 = 0;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int X = umma::digit_quotient(v[e], r);
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

// This thread's 12 elements (512 j + 4 tid .. +3, j < 3) of a 1536-float parameter vector.
__device__ __forceinline__ void load_norm(const float* vec, int tid, float4 (&wv)[3]) {
#pragma unroll
  for (int j = 0; j < 3; ++j) wv[j] = __ldg(reinterpret_cast<const float4*>(vec + 512 * j + 4 * tid));
}

// Chunk partials: [token][q head][chunk] x {m, l, -, -, acc[128]} (acc 16-byte aligned).
constexpr int kPartStride = 4 + kHeadDim;
__device__ __forceinline__ float* part_ptr(const Args& a, int t, int h, int c) {
  return a.attn_part + (((size_t)t * kHeads + h) * a.attn_max_chunks + c) * kPartStride;
}

// Merge of chunk partials in chunk order for 4 consecutive dims d0.. of head h, online: for each chunk c,
// M' = max(M, m_c), o = o e^(M - M') + acc_c e^(m_c - M'), L likewise; out = o / L. Loads are issued a
// batch of kMergeBatch chunks at a time so that one L2 round trip serves the whole batch.
constexpr int kMergeBatch = 16;

__device__ __forceinline__ void merge_chunks(const Args& a, int t, int h, int nch, int d0, float (&out)[4]) {
  float M = -INFINITY, L = 0.f, o[4] = {0.f, 0.f, 0.f, 0.f};
  for (int c0 = 0; c0 < nch; c0 += kMergeBatch) {
    float mv[kMergeBatch], lv[kMergeBatch];
    float4 av[kMergeBatch];
#pragma unroll
    for (int j = 0; j < kMergeBatch; ++j) {
      if (c0 + j < nch) {
        const float* pc = part_ptr(a, t, h, c0 + j);
        mv[j] = __ldcg(pc);
        lv[j] = __ldcg(pc + 1);
        av[j] = __ldcg(reinterpret_cast<const float4*>(pc + 4 + d0));
      } else {
        mv[j] = -INFINITY;
        lv[j] = 0.f;
        av[j] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
#pragma unroll
    for (int j = 0; j < kMergeBatch; ++j) {
      if (c0 + j < nch) {
        const float Mn = fmaxf(M, mv[j]);
        const float sa = expf(M - Mn), sb = expf(mv[j] - Mn);
        o[0] = __fadd_rn(__fmul_rn(o[0], sa), __fmul_rn(av[j].x, sb));
        o[1] = __fadd_rn(__fmul_rn(o[1], sa), __fmul_rn(av[j].y, sb));
        o[2] = __fadd_rn(__fmul_rn(o[2], sa), __fmul_rn(av[j].z, sb));
        o[3] = __fadd_rn(__fmul_rn(o[3], sa), __fmul_rn(av[j].w, sb));
        L = __fadd_rn(__fmul_rn(L, sa), __fmul_rn(lv[j], sb));
        M = Mn;
      }
    }
  }
  const float inv = L > 0.0f ? 1.0f / L : 0.0f;
#pragma unroll
  for (int e = 0; e < 4; ++e) out[e] = o[e] * inv;
}

// Where a 1536-wide projection input comes from.
enum InMode { kInEmbed = 0, kInY = 1, kInCtx = 2, kInA = 3 };

__device__ __forceinline__ int* acc_ptr(const Args& a, int parity, int t, int d) {
  return a.acc + ((size_t)(parity * 4 + t) * 3 + d) * kAccRows;
}

// Finished value of 4 consecutive output rows of a split projection from its integer accumulators:
// (float)(step * (acc0 + 256 acc1 + 65536 acc2)), the exact integer sum scaled once.
__device__ __forceinline__ void acc_values(const Args& a, int parity, int t, int row, float step, float (&out)[4]) {
  const int4 d0 = __ldcg(reinterpret_cast<const int4*>(acc_ptr(a, parity, t, 0) + row));
  const int4 d1 = __ldcg(reinterpret_cast<const int4*>(acc_ptr(a, parity, t, 1) + row));
  const int4 d2 = __ldcg(reinterpret_cast<const int4*>(acc_ptr(a, parity, t, 2) + row));
  const int x0[4] = {d0.x, d0.y, d0.z, d0.w}, x1[4] = {d1.x, d1.y, d1.z, d1.w}, x2[4] = {d2.x, d2.y, d2.z, d2.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const long long tot = (long long)x0[e] + 256ll * (long long)x1[e] + 65536ll * (long long)x2[e];
    out[e] = (float)((double)tot * (double)step);
  }
}

struct InSrc {
  int mode;
  int parity;           // kInA / kInY: accumulator parity of the layer that produced them
  int layer;            // kInA / kInY: that layer
  float4 os[3], ds[3];  // o_s / down_s of this thread's elements (kInA: os; kInY: both)
  float* y_write;       // kInY: also store the layer output here ([nt][1536]) when non-null
  float* dump_write;    // kInY: and here when non-null
};

// This thread's elements 512 j + 4 tid .. +3 of token t's input row.
__device__ __forceinline__ void load_input(const Args& a, const InSrc& src, int t, int tid, float (&v)[3][4]) {
  if (src.mode == kInEmbed) {
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
  } else if (src.mode == kInCtx) {
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      const float4 f = __ldcg(reinterpret_cast<const float4*>(a.ctx + (size_t)t * kHidden + 512 * j + 4 * tid));
      v[j][0] = f.x;
      v[j][1] = f.y;
      v[j][2] = f.z;
      v[j][3] = f.w;
    }
  } else {
    // o_proj output a = o_s * (step * acc); for kInY the layer output y = bf16(a + down_s * (step * acc)).
    // Every load is issued before any is used: one L2 round trip.
    const bool y = src.mode == kInY;
    const float st_o = __ldcg(&a.steps[(src.layer * 4 + kO) * 4 + t]);
    const float st_d = y ? __ldcg(&a.steps[(src.layer * 4 + kDown) * 4 + t]) : 0.f;
    int4 ro[3][3], rd[3][3];
#pragma unroll
    for (int j = 0; j < 3; ++j)
#pragma unroll
      for (int d = 0; d < 3; ++d) {
        const int k = 512 * j + 4 * tid;
        ro[j][d] = __ldcg(reinterpret_cast<const int4*>(acc_ptr(a, src.parity, t, d) + acc_row_base(kO) + k));
        rd[j][d] = y ? __ldcg(reinterpret_cast<const int4*>(acc_ptr(a, src.parity, t, d) + acc_row_base(kDown) + k))
                     : make_int4(0, 0, 0, 0);
      }
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      const int k = 512 * j + 4 * tid;
      const float osc[4] = {src.os[j].x, src.os[j].y, src.os[j].z, src.os[j].w};
      const float dsc[4] = {src.ds[j].x, src.ds[j].y, src.ds[j].z, src.ds[j].w};
      const int o0[4] = {ro[j][0].x, ro[j][0].y, ro[j][0].z, ro[j][0].w};
      const int o1[4] = {ro[j][1].x, ro[j][1].y, ro[j][1].z, ro[j][1].w};
      const int o2[4] = {ro[j][2].x, ro[j][2].y, ro[j][2].z, ro[j][2].w};
      const int d0[4] = {rd[j][0].x, rd[j][0].y, rd[j][0].z, rd[j][0].w};
      const int d1[4] = {rd[j][1].x, rd[j][1].y, rd[j][1].z, rd[j][1].w};
      const int d2[4] = {rd[j][2].x, rd[j][2].y, rd[j][2].z, rd[j][2].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const long long to = (long long)o0[e] + 256ll * (long long)o1[e] + 65536ll * (long long)o2[e];
        v[j][e] = osc[e] * (float)((double)to * (double)st_o);
        if (y) {
          const long long td = (long long)d0[e] + 256ll * (long long)d1[e] + 65536ll * (long long)d2[e];
          v[j][e] = round_bf16(__fadd_rn(v[j][e], dsc[e] * (float)((double)td * (double)st_d)));
        }
      }
      if (y) {
        const float4 yv = make_float4(v[j][0], v[j][1], v[j][2], v[j][3]);
        if (src.y_write) *reinterpret_cast<float4*>(src.y_write + (size_t)t * kHidden + k) = yv;
        if (src.dump_write) *reinterpret_cast<float4*>(src.dump_write + (size_t)t * kHidden + k) = yv;
      }
    }
  }
}

// Digits of a whole 1536-wide input row per token, optionally RMS-normalised (double accumulation, as the
// decode reference; wv = this thread's norm weights). Records the step of each token in step[] and, for
// the designated CTA, in the global step table (every CTA computes the same value).
__device__ void build_full(const Args& a, Ctrl& cs, uint8_t* dbuf, const InSrc& src, bool norm, const float4 (&wv)[3],
                           int tid, float (&step)[4], float* step_out) {
  const int warp = tid >> 5, lane = tid & 31;
  for (int t = 0; t < a.nt; ++t) {
    float v[3][4];
    load_input(a, src, t, tid, v);
    if (norm) {
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
        const float4 w = wv[j];
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
    if (step_out != nullptr && tid == 0) step_out[t] = st;
    const double r = umma::digit_recip(st);
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      const int k = 512 * j + 4 * tid;
      put_digits(dbuf + (size_t)(k >> 7) * kDigitBlockBytes, t, k & 127, v[j], r);
    }
  }
}

// Digits of the down projection's input h (8960 wide) for this CTA's items only; the step comes from
// max|h| gathered by the gate|up epilogues.
__device__ void build_down(const Args& a, uint8_t* dbuf, int l, uint32_t b0, uint32_t b1, int tid, float (&step)[4],
                           float* step_out) {
  for (int t = 0; t < a.nt; ++t) {
    const float mx = __uint_as_float(__ldcg(&a.sync->hmax[l].pad[t]));
    const float st = mx > 0.0f ? mx / kDigitRange : 1.0f;
    step[t] = st;
    if (step_out != nullptr && tid == 0) step_out[t] = st;
    const double r = umma::digit_recip(st);
    for (uint32_t i = b0; i < b1; ++i) {
      const Item it = a.items[i];
      const int n4 = (it.kb1 - it.kb0) * 32;
      for (int f = tid; f < n4; f += kWorkers) {
        const int k = it.kb0 * kKBlock + 4 * f;
        const float4 x = __ldcg(reinterpret_cast<const float4*>(a.h + (size_t)t * kInter + k));
        const float v[4] = {x.x, x.y, x.z, x.w};
        put_digits(dbuf + (size_t)(it.dslot + (f >> 5)) * kDigitBlockBytes, t, 4 * (f & 31), v, r);
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
  int pos[4], seq[4];     // per token, constant for the launch
  float* kvrow[4];        // this step's KV row of layer 0 (K), per token; other layers/V at fixed offsets
};

// Accumulator read-out of one item. Split projections (q|k|v, o, down) add their partial sums to the
// integer accumulators with atomics and signal; the consumers of the next step read the exact totals
// themselves, so no CTA waits for the other K segments of its tile. The item also clears its share of
// the accumulator rows of the other parity, which the next layer uses (every reader of those rows has
// finished by now). gate|up (one CTA per tile) finishes here: SiLU(gate) * up and max |h|.
__device__ void item_epilogue(const Args& a, Ctrl& cs, WorkerCtx& w, const Item it, int l, const float (&step)[4],
                              unsigned* abort_flag) {
  const int nt = a.nt, r = w.r, tid = w.tid;
  const int s = it.stage;
  float gsc = 0.f;
  float* hdst = nullptr;
  if (s == kGu) {
    const int row = r < 64 ? it.tile * 64 + r : kInter + it.tile * 64 + (r - 64);
    gsc = __ldg(a.layers[l].gu_s + row);
    hdst = a.h + it.tile * 64 + (r & 63);
  } else {
    // clear this item's share of the rows for layer l + 1 (other parity)
    const int row = acc_row_base(s) + it.tile * kTileM + r;
    if (r % split(s) == it.seg) {
#pragma unroll
      for (int t = 0; t < 4; ++t)
#pragma unroll
        for (int d = 0; d < 3; ++d) acc_ptr(a, (l + 1) & 1, t, d)[row] = 0;
    }
  }
  const unsigned b = w.item_no & 1;
  mwait(&cs.acc_full[b], (w.item_no >> 1) & 1, abort_flag);
  const int ts = s == kQkv ? 0 : s == kO ? 1 : s == kDown ? 2 : -1;  // trace slots of split stages
  if (tid == 0 && ts >= 0) stamp(a, l, kTraceAcc + ts);
  __syncwarp();
  fence_after();
  int v[16];
  {
    const uint32_t ta = w.tmem + b * (kAccParts * kTileN) + ((uint32_t)(w.quarter * 32) << 16);
    tmem_ld16(ta, v);
    // issuer p wrote part p only if the item has more than p units
#pragma unroll
    for (int p = 1; p < kAccParts; ++p) {
      if (it.kb1 - it.kb0 > p) {
        int u[16];
        tmem_ld16(ta + p * kTileN, u);
#pragma unroll
        for (int c = 0; c < 16; ++c) v[c] += u[c];
      }
    }
  }
  fence_before();
  mbar_arrive(&cs.acc_empty[b]);
  ++w.item_no;
  int done_slot;
  if (s != kGu) {
    const int row = acc_row_base(s) + it.tile * kTileM + r;
    for (int t = 0; t < nt; ++t)
#pragma unroll
      for (int d = 0; d < 3; ++d) atomicAdd(acc_ptr(a, l & 1, t, d) + row, v[4 * d + t]);
    done_slot = s == kQkv ? kDoneQkv : s == kO ? kDoneO : kDoneDown;
  } else {
    // tile rows 0..63: gate rows 64 j.., rows 64..127: the matching up rows
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const long long tot = (long long)v[t] + 256ll * (long long)v[4 + t] + 65536ll * (long long)v[8 + t];
      cs.ys[r][t] = gsc * (float)((double)tot * (double)step[t]);
    }
    named_sync(kBarW, kWorkers);
    if (r < 64) {  // warps of TMEM quarters 0 and 1
      for (int t = 0; t < nt; ++t) {
        const float gv = cs.ys[r][t], uv = cs.ys[r + 64][t];
        const float silu = __fdiv_rn(gv, __fadd_rn(1.0f, expf(-gv)));
        const float hv = __fmul_rn(silu, uv);
        hdst[(size_t)t * kInter] = hv;
        const float m = warp_max(fabsf(hv));
        if (w.lane == 0) atomicMax(&a.sync->hmax[l].pad[t], __float_as_uint(m));
      }
    }
    done_slot = kDoneGu;
  }
  named_sync(kBarW, kWorkers);
  if (tid == 0) {
    red_release(&a.sync->done[l][done_slot].v, 1u);
    if (ts >= 0) stamp(a, l, kTraceArrived + ts);
  }
}

// ---------------------------------------------------------------------------------------------------
// workers: attention (hls/decode_only/qwen_decode_attention_kernel.cpp:113-162), one 64-key chunk of one
// (token, KV head) per item; chunk partials merged in chunk order by the last chunk to finish.
// ---------------------------------------------------------------------------------------------------
// Attention work items: one 64-key chunk (= one KV page) x one KV group x one half of its six query
// heads, so each of the many small items keeps all 128 workers busy.
constexpr int kHalf = 3;  // query heads per item

struct AttnItem {
  int t, g, hp, c, nchunks, n, nhist;
  const float* kbase;
  const float* vbase;
};

__device__ __forceinline__ int attn_items_of(int nch) { return kKvHeads * 2 * nch; }

__device__ __forceinline__ AttnItem attn_decode(const Args& a, const WorkerCtx& w, int l, int i, const int (&nch)[4]) {
  AttnItem it;
  int t = 0, rem = i;
  while (rem >= attn_items_of(nch[t])) {
    rem -= attn_items_of(nch[t]);
    ++t;
  }
  it.t = t;
  it.g = rem / (2 * nch[t]);
  it.hp = (rem / nch[t]) & 1;
  it.c = rem % nch[t];
  it.nchunks = nch[t];
  const int L = w.pos[t] + 1;
  const int k0 = it.c * kChunk;
  it.n = min(kChunk, L - k0);
  it.nhist = min(it.n, w.pos[t] - k0);  // rows written by earlier steps
  static_assert(kChunk == kPage, "an attention chunk must map onto one KV page");
  const KvView kv{a.kv_pool, nullptr, a.page_table, l, a.max_pages};
  it.kbase = kv_row(kv, w.seq[t], k0, 0) + it.g * kHeadDim;
  it.vbase = kv_row(kv, w.seq[t], k0, 1) + it.g * kHeadDim;
  return it;
}

// cp.async of chunk rows [r0, r1) of K and V (the rows of a chunk are 256 floats apart: one KV page)
__device__ __forceinline__ void attn_load_rows(AttnSmem& sm, const AttnItem& it, int r0, int r1, int tid) {
  for (int i = r0 * 32 + tid; i < r1 * 32; i += kWorkers) {
    const int rr = i >> 5, f = i & 31;
    cp_async16(&sm.ks[rr][4 * f], it.kbase + (size_t)rr * kKvWidth + 4 * f);
    cp_async16(&sm.vs[rr][4 * f], it.vbase + (size_t)rr * kKvWidth + 4 * f);
  }
}

// Constants of the q|k|v epilogue for the rows this thread finishes in attention: dim d = tid of the item's
// three query heads, of the K head and of the V head, plus the RoPE factors at the token position.
struct QkvConst {
  float qs[kHalf], qb[kHalf];
  float ks, kb, vs, vb;
  float rc, rs;
};

__device__ __forceinline__ int q_head(const AttnItem& it, int j) { return it.g * kGroups + it.hp * kHalf + j; }

__device__ __forceinline__ void qkv_const(const Args& a, const WorkerCtx& w, int l, const AttnItem& it, QkvConst& k) {
  const LayerDev& L = a.layers[l];
  const int d = w.tid;
#pragma unroll
  for (int j = 0; j < kHalf; ++j) {
    const int row = q_head(it, j) * kHeadDim + d;
    k.qs[j] = __ldg(L.qkv_s + row);
    k.qb[j] = __ldg(L.qkv_b + row);
  }
  const int krow = kHidden + it.g * kHeadDim + d, vrow = kHidden + kKvWidth + it.g * kHeadDim + d;
  k.ks = __ldg(L.qkv_s + krow);
  k.kb = __ldg(L.qkv_b + krow);
  k.vs = __ldg(L.qkv_s + vrow);
  k.vb = __ldg(L.qkv_b + vrow);
  const size_t ri = (size_t)w.pos[it.t] * 64 + (d & 63);
  k.rc = __ldg(a.rope_cos + ri);
  k.rs = __ldg(a.rope_sin + ri);
}

// q|k|v value of one row from the integer accumulators: bias + scale * (step * acc)
__device__ __forceinline__ float qkv_value(const Args& a, int parity, int t, int row, float step, float sc, float bb) {
  const int* p0 = acc_ptr(a, parity, t, 0);
  const int* p1 = acc_ptr(a, parity, t, 1);
  const int* p2 = acc_ptr(a, parity, t, 2);
  const long long tot =
      (long long)__ldcg(p0 + row) + 256ll * (long long)__ldcg(p1 + row) + 65536ll * (long long)__ldcg(p2 + row);
  return __fmaf_rn(sc, (float)((double)tot * (double)step), bb);
}

// rotate-half RoPE of dim d given its partner dim d ^ 64
__device__ __forceinline__ float rope(float mine, float other, int d, float c, float sn) {
  return d < 64 ? __fsub_rn(__fmul_rn(mine, c), __fmul_rn(other, sn)) : __fadd_rn(__fmul_rn(mine, c), __fmul_rn(other, sn));
}

// One item: the history rows are already in flight; finishes q (three heads) and, in the chunk that holds
// it, the new token's K/V row from the q|k|v accumulators, then scores, softmax statistics and P.V of the
// chunk, written as a partial; the last chunk of a (token, group, half) to finish merges them in chunk
// order and writes the three heads' context.
__device__ void attn_item(const Args& a, AttnSmem& sm, Ctrl& cs, const WorkerCtx& w, int l, const AttnItem& it,
                          const QkvConst& qc) {
  const int tid = w.tid, warp = tid >> 5, lane = tid & 31;
  const int t = it.t, n = it.n, nchunks = it.nchunks;
  {
    const int d = tid, parity = l & 1;
    const float st = __ldcg(&a.steps[(l * 4 + kQkv) * 4 + t]);
    const bool has_new = it.nhist < n;  // the new token is row nhist of this chunk
    float qv[kHalf], kv = 0.f, vv = 0.f;
#pragma unroll
    for (int j = 0; j < kHalf; ++j) qv[j] = qkv_value(a, parity, t, q_head(it, j) * kHeadDim + d, st, qc.qs[j], qc.qb[j]);
    if (has_new) {
      kv = qkv_value(a, parity, t, kHidden + it.g * kHeadDim + d, st, qc.ks, qc.kb);
      vv = qkv_value(a, parity, t, kHidden + kKvWidth + it.g * kHeadDim + d, st, qc.vs, qc.vb);
    }
#pragma unroll
    for (int j = 0; j < kHalf; ++j) sm.qs[j][d] = qv[j];
    if (has_new) sm.ks[it.nhist][d] = kv;
    named_sync(kBarW, kWorkers);
    float qr[kHalf], kr = 0.f;
#pragma unroll
    for (int j = 0; j < kHalf; ++j) qr[j] = rope(qv[j], sm.qs[j][d ^ 64], d, qc.rc, qc.rs);
    if (has_new) kr = rope(kv, sm.ks[it.nhist][d ^ 64], d, qc.rc, qc.rs);
    named_sync(kBarW, kWorkers);
#pragma unroll
    for (int j = 0; j < kHalf; ++j) sm.qs[j][d] = qr[j];
    if (has_new) {
      sm.ks[it.nhist][d] = kr;
      sm.vs[it.nhist][d] = vv;
      if (it.hp == 0) {  // the cache row of this step, for later steps
        float* krow = w.kvrow[t] + ((size_t)l * 2) * kPage * kKvWidth + it.g * kHeadDim + d;
        krow[0] = kr;
        krow[kPage * kKvWidth] = vv;
      }
    }
  }
  cp_async_wait_all();
  named_sync(kBarW, kWorkers);
  if (tid == 0) stamp(a, l, kTraceAttnQ);
  const float scaling = kAttentionScaling;
  {
    // thread = (key, half of the head dims): three heads over 64 dims, the two halves added
    const int key = tid >> 1, f0 = (tid & 1) * 16;
    float s0 = 0.f, s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int f = f0; f < f0 + 16; ++f) {
      const float4 kk = *reinterpret_cast<const float4*>(&sm.ks[key][4 * f]);
      const float4 x0 = *reinterpret_cast<const float4*>(&sm.qs[0][4 * f]);
      const float4 x1 = *reinterpret_cast<const float4*>(&sm.qs[1][4 * f]);
      const float4 x2 = *reinterpret_cast<const float4*>(&sm.qs[2][4 * f]);
      s0 = fmaf(x0.x, kk.x, fmaf(x0.y, kk.y, fmaf(x0.z, kk.z, fmaf(x0.w, kk.w, s0))));
      s1 = fmaf(x1.x, kk.x, fmaf(x1.y, kk.y, fmaf(x1.z, kk.z, fmaf(x1.w, kk.w, s1))));
      s2 = fmaf(x2.x, kk.x, fmaf(x2.y, kk.y, fmaf(x2.z, kk.z, fmaf(x2.w, kk.w, s2))));
    }
    s0 = __fadd_rn(s0, __shfl_xor_sync(0xffffffffu, s0, 1));
    s1 = __fadd_rn(s1, __shfl_xor_sync(0xffffffffu, s1, 1));
    s2 = __fadd_rn(s2, __shfl_xor_sync(0xffffffffu, s2, 1));
    if ((tid & 1) == 0) {
      const bool ok = key < n;
      sm.es[key][0] = ok ? s0 * scaling : -INFINITY;
      sm.es[key][1] = ok ? s1 * scaling : -INFINITY;
      sm.es[key][2] = ok ? s2 * scaling : -INFINITY;
    }
  }
  named_sync(kBarW, kWorkers);
  if (warp < kHalf) {
    const int j = warp;
    const float x0 = sm.es[lane][j], x1 = sm.es[lane + 32][j];
    float m = warp_max(fmaxf(x0, x1));
    m = fmaxf(m, -1.0e30f);  // the reference's initial max
    const float e0 = lane < n ? expf(x0 - m) : 0.f;
    const float e1 = lane + 32 < n ? expf(x1 - m) : 0.f;
    sm.es[lane][j] = e0;
    sm.es[lane + 32][j] = e1;
    float sum = e0 + e1;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) {
      sm.ms[j] = m;
      sm.ls[j] = sum;
    }
  }
  named_sync(kBarW, kWorkers);
  float acc[kHalf] = {0.f, 0.f, 0.f};
#pragma unroll 4
  for (int key = 0; key < n; ++key) {
    const float vv = sm.vs[key][tid];
    const float4 e = *reinterpret_cast<const float4*>(&sm.es[key][0]);
    acc[0] = fmaf(e.x, vv, acc[0]);
    acc[1] = fmaf(e.y, vv, acc[1]);
    acc[2] = fmaf(e.z, vv, acc[2]);
  }
  // the chunk partial
#pragma unroll
  for (int j = 0; j < kHalf; ++j) {
    float* pc = part_ptr(a, t, q_head(it, j), it.c);
    pc[4 + tid] = acc[j];
    if (tid == 0) {
      pc[0] = sm.ms[j];
      pc[1] = sm.ls[j];
    }
  }
  named_sync(kBarW, kWorkers);
  if (tid == 0) {
    cs.flag = atom_add_acq_rel(&a.sync->attn_cnt[t][it.g * 2 + it.hp].v, 1u) == (unsigned)nchunks - 1u;
    stamp(a, l, kTraceAttnPart);
  }
  named_sync(kBarW, kWorkers);
  if (!cs.flag) return;
  // last chunk of this (token, group, half): merge and write the three heads' context; thread = 4 dims of
  // one head (96 threads)
  if (tid < kHalf * 32) {
    const int j = tid >> 5, d0 = 4 * (tid & 31), h = q_head(it, j);
    float out[4];
    merge_chunks(a, t, h, nchunks, d0, out);
    *reinterpret_cast<float4*>(a.ctx + (size_t)t * kHidden + h * kHeadDim + d0) = make_float4(out[0], out[1], out[2], out[3]);
  }
  named_sync(kBarW, kWorkers);
  if (tid == 0) {
    a.sync->attn_cnt[t][it.g * 2 + it.hp].v = 0u;
    red_release(&a.sync->done[l][kDoneAttn].v, 1u);
    stamp(a, l, kTraceAttnMerge);
  }
}

__device__ __forceinline__ int attn_chunks(const WorkerCtx& w, int t) { return (w.pos[t] + 1 + kChunk - 1) / kChunk; }

// Completion count of the attention step: one per (token, group, half), by its merging chunk.
__device__ __forceinline__ unsigned attn_done_target(const Args& a) { return (unsigned)(a.nt * kKvHeads * 2); }

// Attention of layer l over this CTA's items (blockIdx.x, + gridDim.x, ...). The history rows of the
// first item do not depend on this step and are requested before the wait for q|k|v.
__device__ void attention_stage(const Args& a, AttnSmem& sm, Ctrl& cs, const WorkerCtx& w, int l,
                                unsigned* abort_flag) {
  const int tid = w.tid;
  int nch[4] = {0, 0, 0, 0}, total = 0;
  for (int t = 0; t < a.nt; ++t) {
    nch[t] = attn_chunks(w, t);
    total += attn_items_of(nch[t]);
  }
  if ((int)blockIdx.x >= total) return;
  named_sync(kBarW, kWorkers);  // shared memory free: this CTA's earlier epilogues are done
  AttnItem it = attn_decode(a, w, l, blockIdx.x, nch);
  attn_load_rows(sm, it, 0, it.nhist, tid);
  QkvConst qc;
  qkv_const(a, w, l, it, qc);
  workers_wait(&a.sync->done[l][kDoneQkv].v, (unsigned)stage_items(kQkv), abort_flag, tid);
  if (tid == 0) stamp(a, l, kTraceWait + 1);
  for (int i = blockIdx.x;;) {
    attn_item(a, sm, cs, w, l, it, qc);
    i += gridDim.x;
    if (i >= total) break;
    const AttnItem nx = attn_decode(a, w, l, i, nch);
    if (nx.t != it.t || nx.g != it.g || nx.hp != it.hp) qkv_const(a, w, l, nx, qc);
    it = nx;
    named_sync(kBarW, kWorkers);  // previous chunk done with the shared buffers
    attn_load_rows(sm, it, 0, it.nhist, tid);
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
  {
    const KvView kv0{a.kv_pool, nullptr, a.page_table, 0, a.max_pages};
    for (int t = 0; t < 4; ++t) {
      w.pos[t] = t < a.nt ? __ldcg(&a.pos[t]) : 0;
      w.seq[t] = t < a.nt ? __ldcg(&a.seq[t]) : 0;
      w.kvrow[t] = t < a.nt ? kv_row(kv0, w.seq[t], w.pos[t], 0) : nullptr;
    }
  }
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
  // The CTA holding q|k|v tile 0, segment 0 writes each layer's output y (needed by the LM head and the
  // hidden-state dump); every other CTA only uses it on chip.
  bool y_writer = false;
  for (uint32_t i = sb[kQkv]; i < se[kQkv]; ++i) y_writer |= a.items[i].tile == 0 && a.items[i].seg == 0;
  const bool tr = w.tid == 0;
  for (int l = 0; l < kLayers; ++l) {
    const LayerDev& L = a.layers[l];
    SyncWord* done = a.sync->done[l];
    float* const step_tab = a.steps + (size_t)l * 16;
    float4 wv[3];
    InSrc src;
    // q|k|v: input = previous layer's output, finished here from its o_proj and down accumulators (or the
    // token embeddings for layer 0)
    if (sb[kQkv] < se[kQkv]) {
      load_norm(L.input_ln, w.tid, wv);
      src.mode = l == 0 ? kInEmbed : kInY;
      if (l > 0) {
        const LayerDev& P = a.layers[l - 1];
        src.parity = (l - 1) & 1;
        src.layer = l - 1;
        load_norm(P.o_s, w.tid, src.os);
        load_norm(P.down_s, w.tid, src.ds);
        src.y_write = y_writer ? (((l - 1) & 1) ? a.y1 : a.y0) : nullptr;
        src.dump_write = y_writer && a.dump ? a.dump + (size_t)(l - 1) * a.nt * kHidden : nullptr;
        workers_wait(&a.sync->done[l - 1][kDoneDown].v, (unsigned)stage_items(kDown), abort_flag, w.tid);
      }
      if (tr) stamp(a, l, kTraceWait + 0);
      build_full(a, cs, digits(inst), src, true, wv, w.tid, step, step_tab + kQkv * 4);
      ready();
      if (tr) stamp(a, l, kTraceBuilt + 0);
      for (uint32_t i = sb[kQkv]; i < se[kQkv]; ++i) item_epilogue(a, cs, w, a.items[i], l, step, abort_flag);
      if (tr) stamp(a, l, kTraceDone + 0);
    }
    attention_stage(a, asm_, cs, w, l, abort_flag);
    if (sb[kO] < se[kO]) {
      src.mode = kInCtx;
      workers_wait(&done[kDoneAttn].v, attn_done_target(a), abort_flag, w.tid);
      if (tr) stamp(a, l, kTraceWait + 2);
      build_full(a, cs, digits(inst), src, false, wv, w.tid, step, step_tab + kO * 4);
      ready();
      if (tr) stamp(a, l, kTraceBuilt + 2);
      for (uint32_t i = sb[kO]; i < se[kO]; ++i) item_epilogue(a, cs, w, a.items[i], l, step, abort_flag);
      if (tr) stamp(a, l, kTraceDone + 2);
    }
    if (sb[kGu] < se[kGu]) {
      // input = RMSNorm(a), a finished here from the o_proj accumulators
      load_norm(L.post_ln, w.tid, wv);
      src.mode = kInA;
      src.parity = l & 1;
      src.layer = l;
      load_norm(L.o_s, w.tid, src.os);
      workers_wait(&done[kDoneO].v, (unsigned)stage_items(kO), abort_flag, w.tid);
      if (tr) stamp(a, l, kTraceWait + 3);
      build_full(a, cs, digits(inst), src, true, wv, w.tid, step, step_tab + kGu * 4);
      ready();
      if (tr) stamp(a, l, kTraceBuilt + 3);
      for (uint32_t i = sb[kGu]; i < se[kGu]; ++i) item_epilogue(a, cs, w, a.items[i], l, step, abort_flag);
      if (tr) stamp(a, l, kTraceDone + 3);
    }
    if (sb[kDown] < se[kDown]) {
      workers_wait(&done[kDoneGu].v, (unsigned)stage_items(kGu), abort_flag, w.tid);
      if (tr) stamp(a, l, kTraceWait + 4);
      build_down(a, digits(inst), l, sb[kDown], se[kDown], w.tid, step, step_tab + kDown * 4);
      ready();
      if (tr) stamp(a, l, kTraceBuilt + 4);
      for (uint32_t i = sb[kDown]; i < se[kDown]; ++i) item_epilogue(a, cs, w, a.items[i], l, step, abort_flag);
      if (tr) stamp(a, l, kTraceDone + 4);
    }
  }
  // the last layer's output, for the LM head (and the dump)
  if (y_writer) {
    const int l = kLayers - 1;
    InSrc src;
    src.mode = kInY;
    src.parity = l & 1;
    src.layer = l;
    load_norm(a.layers[l].o_s, w.tid, src.os);
    load_norm(a.layers[l].down_s, w.tid, src.ds);
    src.y_write = (l & 1) ? a.y1 : a.y0;
    src.dump_write = a.dump ? a.dump + (size_t)l * a.nt * kHidden : nullptr;
    workers_wait(&a.sync->done[l][kDoneDown].v, (unsigned)stage_items(kDown), abort_flag, w.tid);
    for (int t = 0; t < a.nt; ++t) {
      float v[3][4];
      load_input(a, src, t, w.tid, v);
    }
  }
}

__global__ void __launch_bounds__(kThreads, 1) decode_stack_kernel(const __grid_constant__ Args a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = align_smem_1024(smem_raw);
  uint8_t* ring = base;
  uint8_t* uni = base + (size_t)kRing * kUnitBytes;
  Ctrl& cs = *reinterpret_cast<Ctrl*>(uni + kUnionBytes);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t i0 = a.item_off[blockIdx.x], i1 = a.item_off[blockIdx.x + 1];
  unsigned* abort_flag = &a.sync->abort_flag.v;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kRing; ++s) {
      mbar_init(&cs.full[s], 1);
      mbar_init(&cs.empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&cs.dig_ready[b], kWorkers);
      mbar_init(&cs.acc_full[b], kIssuers);
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
  } else if (warp == 1 || warp == 6) {
    if (lane == 0) mma_issuer(a, ring, uni, cs, tmem, i0, i1, abort_flag, warp == 1 ? 0 : 1);
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
    const unsigned prev = atomicAdd(&a.sync->exit_cnt.v, 1u);
    if (prev == gridDim.x - 1) {  // every CTA is past its last wait: clear the words for the next launch
      __threadfence();
      SyncWord* wds = reinterpret_cast<SyncWord*>(a.sync);
      for (size_t i = 0; i < sizeof(SyncWords) / sizeof(SyncWord); ++i) {
        wds[i].v = 0u;
        for (int j = 0; j < 4; ++j) wds[i].pad[j] = 0u;  // hmax keeps its words here
      }
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
  // Largest items first onto the least-loaded CTA (load = 16 KB units streamed per layer), preferring CTAs
  // that have no item of the same stage yet: a CTA's epilogues of one stage run one after another, so one
  // item per stage and CTA keeps every stage's tail short.
  std::stable_sort(all.begin(), all.end(), [](const Cand& x, const Cand& y) { return x.kb1 - x.kb0 > y.kb1 - y.kb0; });
  std::vector<int> load(ctas, 0), down_blocks(ctas, 0);
  std::vector<std::vector<int>> per_stage(kNumProj, std::vector<int>(ctas, 0));
  std::vector<std::vector<Cand>> per(ctas);
  for (const Cand& c : all) {
    const int units = c.kb1 - c.kb0;
    int best = -1;
    for (int k = 0; k < ctas; ++k) {
      if (c.stage == kDown && down_blocks[k] + units > kDigitBlocks) continue;
      if (best < 0) {
        best = k;
        continue;
      }
      const int nk = per_stage[c.stage][k], nb = per_stage[c.stage][best];
      if (nk < nb || (nk == nb && load[k] < load[best])) best = k;
    }
    per[best].push_back(c);
    load[best] += units;
    ++per_stage[c.stage][best];
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
