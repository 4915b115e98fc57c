// Persistent batch-1 decode step: every layer of one W8 decode step of one sequence in a single cooperative
// launch, one CTA per SM, the projections on the CUDA cores.
//
// Per layer the work is the reference's decode top (hls/decode_only/qwen_decode_top_wrapper.cpp:79-112):
// q|k|v projection + RoPE + KV append, attention over the history, o_proj, gate|up + SiLU, down + the
// attention-output residual, then the caller's bf16 rounding (verification/real_host_top_backend.py:260).
// The arithmetic is that of the tensor-core kernels (qgemm.cu, decode_stack.cu): fp32 activations written
// exactly as three int8 digits per element with one step per row, int32 sums of digit x weight products,
// the same epilogue expressions, the attention chunks merged in chunk order with the same formula. The
// results are bit-identical to them.
//
// Why a second persistent kernel. At batch 1 only 3 of the 16 digit rows of an M128 x N16 int8 MMA carry
// data, and each stage of the tensor-core kernel pays an MMA hand-off chain (digits ready -> issue ->
// commit -> TMEM read) of 1.5-3 us. Here the four worker warps form the int32 dot products themselves with
// dp4a from the same shared-memory weight units (thread = 4 rows x 32 bytes of each 128-byte K block), so a
// stage's results leave the CTA as soon as its last unit has been read.
//
// Cross-CTA data is self-validating, so no stage waits for a completion counter:
//   - split-K projections add (count << 48) + (segment total + 2^43) into one 64-bit word per output row;
//     a consumer reads the word until the count equals the number of K segments (the total is exact);
//   - single-writer data (attention chunk partials, the merged context and its maxima, h = SiLU(gate) * up,
//     per-item max |h|, digit steps) is stored as 64-bit words {tag, fp32 value}, tag = (launch epoch + 1)
//     << 5 | layer; a consumer reads a word until its tag is the current one.
// A 64-bit word is written and read by single accesses (strong loads: a weak load may keep returning an
// older copy of a word another SM rewrote), so a consumer sees either the old or the new word. Every data
// word a stage reads was produced by work that precedes it in the layer's dependency chain, and every
// buffer that is reused (layer parity) is rewritten only by work that depends on all of its readers.
// Every worker reads its own input words until they are all current (one L2 round trip once the data has
// landed; a separate completion signal would add one).
//
// Roles (160 threads):
//   warp 0      lane 0: producer, cp.async.bulk of pre-swizzled 16 KB weight units into a ring of shared
//               memory stages, never waiting for activations; lanes 1-31 zero the other launch parity of
//               the packed words at the start
//   warps 1-4   workers: read a stage's inputs, build the digits of their K blocks, dp4a over the ring
//               units, publish the results; attention chunks (the item of a merge group's last chunk also
//               merges the group)
// Every wait gives up after ~1 s, raising an abort flag that ends all other waits quickly, and records the
// failure in the kernel error flag.
#include <cuda_fp16.h>

#include <algorithm>
#include <mutex>

#include "decode_bs1.h"
#include "umma_sm100.cuh"

namespace qb {
namespace bs1 {
namespace {

using stack::Item;
using stack::kDown;
using stack::kGu;
using stack::kNumProj;
using stack::kO;
using stack::kQkv;
using stack::nkb;
using stack::tiles;
using stack::unit_base;
using umma::kKBlock;
using umma::kUnitBytes;

constexpr int kRing = 9;           // weight stages per CTA; Args::ring uses 2..kRing of them
constexpr int kWorkers = 128;
constexpr int kThreads = 32 + kWorkers;
constexpr int kBarW = 1;           // named barrier of the worker warps
constexpr int kDigitStride = kHidden;  // bytes per digit plane (the widest K range of one item)
constexpr int kChunk = 64;         // attention keys per work item (one KV page)
// K and q rows in shared memory: dims 64..127 start 68 floats into a 136-float row, so that the QK loop's
// 16-byte reads (thread = key x half of the dims) of four keys and both halves fall into eight different
// 16-byte bank groups, and the two halves of a q row into two
constexpr int kRow = 136;
constexpr int kHalfCol = 68;
constexpr int kHalf = 3;           // query heads per attention item
constexpr int kMergeBatch = 12;    // chunk partials read per round trip by the merge
// the merge's rescale factors (3 heads x chunks x 3 floats) reuse the attention chunk rows
static_assert(kChunk * kRow >= kHalf * 3 * ((kMaxSeq + 1024) / kChunk), "rescale factors of every chunk");
constexpr long long kSpinLimit = 2000000000ll;  // clock cycles, ~1 s
constexpr unsigned long long kBias = 1ull << 43;
constexpr unsigned long long kLow48 = (1ull << 48) - 1;
static_assert(kChunk == kPage, "an attention chunk must map onto one KV page");
static_assert(seg_len(stack::kO) == kHalf, "an o_proj K segment is one attention merge group");

__device__ __forceinline__ int kcol(int d) { return d < 64 ? d : d - 64 + kHalfCol; }

struct AttnSmem {
  float ks[kChunk][kRow];
  float vs[kChunk][kHeadDim];
  float qs[kHalf][kRow];
  float es[kChunk][4];
  float ms[kHalf], ls[kHalf];
};

// the attention scratch and the digit planes have separate regions, so that a layer's attention rows can be
// requested before its q|k|v stage
constexpr size_t kAttnBytes = (sizeof(AttnSmem) + 127) / 128 * 128;
constexpr size_t kDigitBytes = 3 * (size_t)kDigitStride;

struct Ctrl {
  uint64_t full[kRing], empty[kRing];
  double red[4];
  float redf[4];
  float ys[128];
  float av[kHidden];  // this layer's attention output a (o_proj + residual), kept by the gate|up item's load
};

constexpr size_t kSmemBytes = 1024 + (size_t)kRing * kUnitBytes + kAttnBytes + kDigitBytes + sizeof(Ctrl);
static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");

// ---------------------------------------------------------------------------------------------------
// words and waits
// ---------------------------------------------------------------------------------------------------
__device__ __forceinline__ unsigned ld_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ unsigned long long ld_word(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Two adjacent words (16-byte aligned); each is read by a single access.
__device__ __forceinline__ void ld_word2(const unsigned long long* p, unsigned long long& x, unsigned long long& y) {
  asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(x), "=l"(y) : "l"(p) : "memory");
}

__device__ __forceinline__ void st_word(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ void red_word(unsigned long long* p, unsigned long long v) {
  asm volatile("red.relaxed.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned tag_of(unsigned epoch, int l) { return ((epoch + 1u) << 5) | (unsigned)l; }
__device__ __forceinline__ unsigned long long tagged(unsigned tag, float v) {
  return ((unsigned long long)tag << 32) | __float_as_uint(v);
}
__device__ __forceinline__ bool tag_ok(unsigned long long w, unsigned tag) { return (unsigned)(w >> 32) == tag; }
__device__ __forceinline__ float word_value(unsigned long long w) { return __uint_as_float((unsigned)w); }

// Packed split-K word of one segment total (|total| < 2^43).
__device__ __forceinline__ unsigned long long packed(long long total) {
  return (1ull << 48) + (unsigned long long)(total + (long long)kBias);
}
__device__ __forceinline__ bool count_ok(unsigned long long w, int n) { return (int)(w >> 48) == n; }
__device__ __forceinline__ long long packed_total(unsigned long long w, int n) {
  return (long long)(w & kLow48) - (long long)n * (long long)kBias;
}

__device__ __forceinline__ void give_up(unsigned* abort_flag) {
  atomicExch(&g_kernel_error, kErrMbarTimeout);
  atomicExch(abort_flag, 1u);
}

// Bounded polling: keep_going() after each failed check; false once the time limit has passed (the abort
// flag is then raised) or another CTA has aborted.
struct Spin {
  long long t0 = -1;
  unsigned n = 0;
  __device__ __forceinline__ bool keep_going(unsigned* abort_flag) {
    if (t0 < 0) t0 = clock64();
    if ((++n & 15) == 0) {
      if (ld_u32(abort_flag)) return false;
      if (clock64() - t0 > kSpinLimit) {
        give_up(abort_flag);
        return false;
      }
    }
    return true;
  }
};

// mbarrier phase wait with the same limits.
__device__ bool mwait(uint64_t* bar, unsigned parity, unsigned* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  for (unsigned i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63) == 0) {
      if (ld_u32(abort_flag)) return false;
      if (clock64() - t0 > kSpinLimit) {
        give_up(abort_flag);
        return false;
      }
    }
  }
}

__device__ __forceinline__ void stamp(const Args& a, int l, int slot) {
  if (a.trace == nullptr) return;
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  a.trace[((size_t)blockIdx.x * kLayers + l) * stack::kTraceSlots + slot] = t;
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

__device__ __forceinline__ unsigned long long* acc_layer(const Args& a, unsigned par, int l) {
  return a.buf.acc + ((size_t)par * kLayers + l) * kAccRows;
}
__device__ __forceinline__ unsigned long long* part_ptr(const Args& a, int l, int h, int c) {
  return a.buf.part + (((size_t)(l & 1) * kHeads + h) * a.max_chunks + c) * kPartWords;
}

// ---------------------------------------------------------------------------------------------------
// producer
// ---------------------------------------------------------------------------------------------------
__device__ void producer(const Args& a, uint8_t* ring_smem, Ctrl& cs, uint32_t i0, uint32_t i1,
                         unsigned* abort_flag) {
  const int ring = ring_depth(a);
  int s = 0;
  unsigned ph = 0, issued = 0, last_ph = 0;
  bool ok = true;
  for (int l = 0; l < kLayers && ok; ++l) {
    const uint8_t* wl = a.wtiles + (size_t)l * stack::kLayerTileBytes;
    for (uint32_t i = i0; i < i1 && ok; ++i) {
      const Item it = a.items[i];
      const uint8_t* src = wl + ((size_t)unit_base(it.stage) + (size_t)it.tile * nkb(it.stage)) * kUnitBytes;
      stamp(a, l, stack::kTraceIssue + it.stage);
      for (int kb = it.kb0; kb < it.kb1; ++kb) {
        if (!(ok = mwait(&cs.empty[s], ph ^ 1, abort_flag))) break;
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

// Lanes 1-31 of the producer warp: zero this CTA's share of the other launch parity's packed words, which
// the next launch accumulates into (this launch neither reads nor writes them).
__device__ void clear_other_parity(const Args& a, unsigned par) {
  const size_t n2 = (size_t)kLayers * kAccRows / 2;  // 16-byte stores
  const size_t b = n2 * blockIdx.x / gridDim.x, e = n2 * (blockIdx.x + 1) / gridDim.x;
  uint4* base = reinterpret_cast<uint4*>(a.buf.acc + (size_t)(par ^ 1u) * kLayers * kAccRows);
  for (size_t i = b + (threadIdx.x - 1); i < e; i += 31) base[i] = make_uint4(0u, 0u, 0u, 0u);
}

// ---------------------------------------------------------------------------------------------------
// workers
// ---------------------------------------------------------------------------------------------------
struct Worker {
  int tid, lane, warp;
  int pos, seq;
  float* kvrow;      // this step's K row of layer 0; other layers / V at fixed offsets
  unsigned epoch, par;
  int s;             // ring position
  unsigned ph;
  unsigned* abort_flag;
};

// Digits of 4 consecutive elements at byte k of each plane (plane stride kDigitStride); r = digit_recip(step).
__device__ __forceinline__ void put_digits(uint8_t* dig, int k, const float (&v)[4], double r) {
  uint32_t w0 = 0, w1 = 0, w2 = 0;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int X = umma::digit_quotient(v[e], r);
    int d0, d1, d2;
    umma::split_digits(X, d0, d1, d2);
    w0 |= (uint32_t)(d0 & 255) << (8 * e);
    w1 |= (uint32_t)(d1 & 255) << (8 * e);
    w2 |= (uint32_t)(d2 & 255) << (8 * e);
  }
  *reinterpret_cast<uint32_t*>(dig + k) = w0;
  *reinterpret_cast<uint32_t*>(dig + kDigitStride + k) = w1;
  *reinterpret_cast<uint32_t*>(dig + 2 * kDigitStride + k) = w2;
}

// This thread's 12 elements (512 j + 4 tid .. +3, j < 3) of a 1536-float parameter vector.
__device__ __forceinline__ void load_vec(const float* vec, int tid, float4 (&wv)[3]) {
#pragma unroll
  for (int j = 0; j < 3; ++j) wv[j] = __ldg(reinterpret_cast<const float4*>(vec + 512 * j + 4 * tid));
}

// Block-wide max of a non-negative value over the workers.
__device__ __forceinline__ float block_max(Ctrl& cs, float m, const Worker& w) {
  m = warp_max(m);
  named_sync(kBarW, kWorkers);  // redf free (its previous readers are done)
  if (w.lane == 0) cs.redf[w.warp] = m;
  named_sync(kBarW, kWorkers);
  return fmaxf(fmaxf(cs.redf[0], cs.redf[1]), fmaxf(cs.redf[2], cs.redf[3]));
}

// In place: v = decode RMSNorm(v) * wv (double accumulation, as the decode reference,
// qwen_decode_attention_kernel.cpp:13-27); returns the digit step max|v| / range of the row.
__device__ float norm_and_step(Ctrl& cs, float (&v)[3][4], bool norm, const float4 (&wv)[3], const Worker& w) {
  if (norm) {
    double ss = 0.0;
#pragma unroll
    for (int j = 0; j < 3; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) ss += (double)v[j][e] * (double)v[j][e];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    named_sync(kBarW, kWorkers);
    if (w.lane == 0) cs.red[w.warp] = ss;
    named_sync(kBarW, kWorkers);
    const double tot = cs.red[0] + cs.red[1] + cs.red[2] + cs.red[3];
    const double inv = 1.0 / sqrt(tot / (double)kHidden + (double)kEps);
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      const float4 x = wv[j];
      v[j][0] = (float)((double)v[j][0] * inv * (double)x.x);
      v[j][1] = (float)((double)v[j][1] * inv * (double)x.y);
      v[j][2] = (float)((double)v[j][2] * inv * (double)x.z);
      v[j][3] = (float)((double)v[j][3] * inv * (double)x.w);
    }
  }
  float m = 0.0f;
#pragma unroll
  for (int j = 0; j < 3; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) m = fmaxf(m, fabsf(v[j][e]));
  const float mx = block_max(cs, m, w);
  return mx > 0.0f ? mx / umma::kDigitRange : 1.0f;
}

// Digits of this thread's elements of a 1536-wide row that fall into K blocks [kb0, kb1).
__device__ __forceinline__ void row_digits(uint8_t* dig, const float (&v)[3][4], double r, int kb0, int kb1,
                                           int tid) {
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const int k = 512 * j + 4 * tid;
    if (k >= kb0 * kKBlock && k < kb1 * kKBlock) put_digits(dig, k - kb0 * kKBlock, v[j], r);
  }
}

// int32 dot products of the next n ring units (128 weight rows x one 128-byte K block each) with the digit
// planes (block u of the item at byte 128 u of each plane): thread = 4 rows x bytes {16 q.., 64 + 16 q..}
// of every block (conflict-free in the 128-byte swizzle); returns the exact total of row tid,
// sum_k (d0 + 256 d1 + 65536 d2)[k] * w[k].
__device__ long long gemv_units(Worker& w, Ctrl& cs, const Args& a, uint8_t* ring, const uint8_t* dig, int n,
                                int trace_l = -1) {
  const int q = w.tid & 3, g = w.tid >> 2;
  const int ring_n = ring_depth(a);
  int acc[4][3];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int p = 0; p < 3; ++p) acc[i][p] = 0;
  for (int u = 0; u < n; ++u) {
    mwait(&cs.full[w.s], w.ph, w.abort_flag);
    if (trace_l >= 0 && w.tid == 0 && a.trace != nullptr && (u == 0 || u == 8 || u == n - 1)) {
      stamp(a, trace_l, stack::kTraceUnit + (u == 0 ? 0 : u == 8 ? 1 : 2));
      a.trace[((size_t)blockIdx.x * kLayers + trace_l) * stack::kTraceSlots + stack::kTraceUnit + 3 +
              (u == 0 ? 0 : u == 8 ? 1 : 2)] = (unsigned long long)clock64();
    }
    const uint8_t* wu = ring + (size_t)w.s * kUnitBytes;
    int4 dv[3][2];
#pragma unroll
    for (int p = 0; p < 3; ++p) {
      dv[p][0] = *reinterpret_cast<const int4*>(dig + p * kDigitStride + u * kKBlock + 16 * q);
      dv[p][1] = *reinterpret_cast<const int4*>(dig + p * kDigitStride + u * kKBlock + 64 + 16 * q);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = 4 * g + i;
      const int4 w0 = *reinterpret_cast<const int4*>(wu + r * kKBlock + ((q ^ (r & 7)) << 4));
      const int4 w1 = *reinterpret_cast<const int4*>(wu + r * kKBlock + (((q + 4) ^ (r & 7)) << 4));
#pragma unroll
      for (int p = 0; p < 3; ++p) {
        int x = acc[i][p];
        x = __dp4a(w0.x, dv[p][0].x, x);
        x = __dp4a(w0.y, dv[p][0].y, x);
        x = __dp4a(w0.z, dv[p][0].z, x);
        x = __dp4a(w0.w, dv[p][0].w, x);
        x = __dp4a(w1.x, dv[p][1].x, x);
        x = __dp4a(w1.y, dv[p][1].y, x);
        x = __dp4a(w1.z, dv[p][1].z, x);
        x = __dp4a(w1.w, dv[p][1].w, x);
        acc[i][p] = x;
      }
    }
    __syncwarp();
    if (w.lane == 0) mbar_arrive(&cs.empty[w.s]);
    if (++w.s == ring_n) {
      w.s = 0;
      w.ph ^= 1;
    }
  }
  if (trace_l >= 0 && w.lane == 0 && a.trace != nullptr)
    a.trace[((size_t)blockIdx.x * kLayers + trace_l) * stack::kTraceSlots + stack::kTraceUnit + 6 + w.warp] =
        (unsigned long long)clock64();
  // the four threads of a row group hold disjoint K bytes of the same 4 rows: add them; thread q keeps row
  // 4 g + q = tid
  int r0 = 0, r1 = 0, r2 = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    int x0 = acc[i][0], x1 = acc[i][1], x2 = acc[i][2];
    x0 += __shfl_xor_sync(0xffffffffu, x0, 1);
    x1 += __shfl_xor_sync(0xffffffffu, x1, 1);
    x2 += __shfl_xor_sync(0xffffffffu, x2, 1);
    x0 += __shfl_xor_sync(0xffffffffu, x0, 2);
    x1 += __shfl_xor_sync(0xffffffffu, x1, 2);
    x2 += __shfl_xor_sync(0xffffffffu, x2, 2);
    if (i == q) {
      r0 = x0;
      r1 = x1;
      r2 = x2;
    }
  }
  return (long long)r0 + 256ll * (long long)r1 + 65536ll * (long long)r2;
}

// Layer lp's output y = bf16(a + down_s * (step_d * down_total)) with a = o_s * (step_o * o_total), this
// thread's elements, from the packed words (the expressions of the tensor-core kernels' epilogues).
// av: the layer's a = o_proj output (as load_a forms it), when this CTA already read it for its gate|up item;
// then only the down words are polled.
__device__ void load_y(const Args& a, const Worker& w, int lp, const float4 (&os)[3], const float4 (&ds)[3],
                       const float* av, float (&v)[3][4]) {
  const unsigned long long* acc = acc_layer(a, w.par, lp);
  const unsigned long long* sw = a.buf.steps + (size_t)lp * 4;
  const unsigned tag = tag_of(w.epoch, lp);
  const bool need_o = av == nullptr;
  unsigned long long wo[3][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}, {0, 0, 0, 0}}, wd[3][4], so = 0, sd;
  Spin sp;
  while (true) {
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      const int k = 512 * j + 4 * w.tid;
      if (need_o) {
        ld_word2(acc + acc_row(kO) + k, wo[j][0], wo[j][1]);
        ld_word2(acc + acc_row(kO) + k + 2, wo[j][2], wo[j][3]);
      }
      ld_word2(acc + acc_row(kDown) + k, wd[j][0], wd[j][1]);
      ld_word2(acc + acc_row(kDown) + k + 2, wd[j][2], wd[j][3]);
    }
    if (need_o) so = ld_word(sw + kO);
    sd = ld_word(sw + kDown);
    bool ok = tag_ok(sd, tag) && (!need_o || tag_ok(so, tag));
#pragma unroll
    for (int j = 0; j < 3; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) ok = ok && count_ok(wd[j][e], nseg(kDown)) && (!need_o || count_ok(wo[j][e], nseg(kO)));
    if (ok || !sp.keep_going(w.abort_flag)) break;
  }
  const float st_o = word_value(so), st_d = word_value(sd);
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const float osc[4] = {os[j].x, os[j].y, os[j].z, os[j].w};
    const float dsc[4] = {ds[j].x, ds[j].y, ds[j].z, ds[j].w};
    float4 a4 = make_float4(0.f, 0.f, 0.f, 0.f);
    if (!need_o) a4 = *reinterpret_cast<const float4*>(av + 512 * j + 4 * w.tid);
    const float ak[4] = {a4.x, a4.y, a4.z, a4.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const long long td = packed_total(wd[j][e], nseg(kDown));
      const float avv = need_o ? osc[e] * (float)((double)packed_total(wo[j][e], nseg(kO)) * (double)st_o) : ak[e];
      v[j][e] = round_bf16(__fadd_rn(avv, dsc[e] * (float)((double)td * (double)st_d)));
    }
  }
}

__device__ void load_a(const Args& a, const Worker& w, int l, const float4 (&os)[3], float (&v)[3][4]) {
  const unsigned long long* acc = acc_layer(a, w.par, l);
  const unsigned long long* sw = a.buf.steps + (size_t)l * 4;
  const unsigned tag = tag_of(w.epoch, l);
  unsigned long long wo[3][4], so;
  Spin sp;
  while (true) {
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      const int k = 512 * j + 4 * w.tid;
      ld_word2(acc + acc_row(kO) + k, wo[j][0], wo[j][1]);
      ld_word2(acc + acc_row(kO) + k + 2, wo[j][2], wo[j][3]);
    }
    so = ld_word(sw + kO);
    bool ok = tag_ok(so, tag);
#pragma unroll
    for (int j = 0; j < 3; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) ok = ok && count_ok(wo[j][e], nseg(kO));
    if (ok || !sp.keep_going(w.abort_flag)) break;
  }
  const float st_o = word_value(so);
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const float osc[4] = {os[j].x, os[j].y, os[j].z, os[j].w};
#pragma unroll
    for (int e = 0; e < 4; ++e) v[j][e] = osc[e] * (float)((double)packed_total(wo[j][e], nseg(kO)) * (double)st_o);
  }
}

// ---------------------------------------------------------------------------------------------------
// attention (hls/decode_only/qwen_decode_attention_kernel.cpp:113-162): one 64-key chunk x one KV group x
// three of its six query heads per item; each item stores its chunk partial (m, l, acc) as tagged words, and
// the item of the group's last chunk merges the group's chunks (a merging item waits only for items of lower
// index, which every CTA runs first: no wait can go round in a circle).
// ---------------------------------------------------------------------------------------------------
struct AttnItem {
  int g, hp, c, n, nhist;
  const float* kbase;
  const float* vbase;
};

__device__ __forceinline__ AttnItem attn_decode(const Args& a, const Worker& w, int l, int i, int nch) {
  AttnItem it;
  it.g = i / (2 * nch);
  it.hp = (i / nch) & 1;
  it.c = i % nch;
  const int L = w.pos + 1, k0 = it.c * kChunk;
  it.n = min(kChunk, L - k0);
  it.nhist = min(it.n, w.pos - k0);  // rows written by earlier steps
  const KvView kv{a.kv_pool, nullptr, a.page_table, l, a.max_pages};
  it.kbase = kv_row(kv, w.seq, k0, 0) + it.g * kHeadDim;
  it.vbase = kv_row(kv, w.seq, k0, 1) + it.g * kHeadDim;
  return it;
}

__device__ __forceinline__ void attn_load_rows(AttnSmem& sm, const AttnItem& it, int r0, int r1, int tid) {
  for (int i = r0 * 32 + tid; i < r1 * 32; i += kWorkers) {
    const int rr = i >> 5, f = i & 31;
    cp_async16(&sm.ks[rr][kcol(4 * f)], it.kbase + (size_t)rr * kKvWidth + 4 * f);
    cp_async16(&sm.vs[rr][4 * f], it.vbase + (size_t)rr * kKvWidth + 4 * f);
  }
}

__device__ __forceinline__ int q_head(const AttnItem& it, int j) { return it.g * kGroups + it.hp * kHalf + j; }

struct QkvConst {
  float qs[kHalf], qb[kHalf];
  float ks, kb, vs, vb;
  float rc, rs;
};

__device__ __forceinline__ void qkv_const(const Args& a, const Worker& w, int l, const AttnItem& it, QkvConst& k) {
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
  const size_t ri = (size_t)w.pos * 64 + (d & 63);
  k.rc = __ldg(a.rope_cos + ri);
  k.rs = __ldg(a.rope_sin + ri);
}

// rotate-half RoPE of dim d given its partner dim d ^ 64
__device__ __forceinline__ float rope(float mine, float other, int d, float c, float sn) {
  return d < 64 ? __fsub_rn(__fmul_rn(mine, c), __fmul_rn(other, sn)) : __fadd_rn(__fmul_rn(mine, c), __fmul_rn(other, sn));
}

// The merge of one group's chunk partials (three heads), in two phases.
//   1. warp j (< 3) = head j, lane = chunk: each lane reads its chunk's (m, l) words, a warp prefix-max scan
//      gives the running maxima M_c = max(M_(c-1), m_c) (M_(-1) = -inf), and each lane forms its chunk's
//      rescale factors sa_c = e^(M_(c-1) - M_c), sb_c = e^(m_c - M_c) (shared memory, with l_c);
//   2. thread = head tid / 32, dims 4 lane .. +3: o = o sa_c + acc_c sb_c and L = L sa_c + l_c sb_c over the
//      chunks in order; out = o / L.
// The values and their order are those of merging chunk by chunk with the running max (the formula of the
// other decode kernels); phase 1 only computes every exponential at once. Partials are read as tagged words,
// waiting on the data.
__device__ void merge_group(const Args& a, float* sab, const Worker& w, int l, int h0, int nch, float (&out)[4]) {
  const unsigned tag = tag_of(w.epoch, l);
  const int j = w.warp, lane = w.lane;
  if (j < kHalf) {
    float carry = -INFINITY;
    for (int c0 = 0; c0 < nch; c0 += 32) {
      const int c = c0 + lane;
      unsigned long long mw = 0, lw = 0;
      if (c < nch) {
        const unsigned long long* pc = part_ptr(a, l, h0 + j, c);
        Spin sp;
        while (true) {
          ld_word2(pc, mw, lw);
          if ((tag_ok(mw, tag) && tag_ok(lw, tag)) || !sp.keep_going(w.abort_flag)) break;
        }
      }
      const float mc = c < nch ? word_value(mw) : -INFINITY;
      float x = mc;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x = fmaxf(x, y);
      }
      const float Mc = fmaxf(carry, x);
      float Mp = __shfl_up_sync(0xffffffffu, Mc, 1);
      if (lane == 0) Mp = carry;
      if (c < nch) {
        float* e = sab + ((size_t)j * a.max_chunks + c) * 3;
        e[0] = expf(Mp - Mc);
        e[1] = expf(mc - Mc);
        e[2] = word_value(lw);
      }
      carry = __shfl_sync(0xffffffffu, Mc, 31);
    }
  }
  named_sync(kBarW, kWorkers);
  if (j >= kHalf) return;
  const int d0 = 4 * lane;
  float L = 0.f, o[4] = {0.f, 0.f, 0.f, 0.f};
  for (int c0 = 0; c0 < nch; c0 += kMergeBatch) {
    unsigned long long dw[kMergeBatch][4];
    Spin sp;
    while (true) {
#pragma unroll
      for (int k = 0; k < kMergeBatch; ++k) {
        if (c0 + k < nch) {
          const unsigned long long* pc = part_ptr(a, l, h0 + j, c0 + k);
          ld_word2(pc + 4 + d0, dw[k][0], dw[k][1]);
          ld_word2(pc + 6 + d0, dw[k][2], dw[k][3]);
        }
      }
      bool ok = true;
#pragma unroll
      for (int k = 0; k < kMergeBatch; ++k)
        if (c0 + k < nch)
          ok = ok && tag_ok(dw[k][0], tag) && tag_ok(dw[k][1], tag) && tag_ok(dw[k][2], tag) && tag_ok(dw[k][3], tag);
      if (ok || !sp.keep_going(w.abort_flag)) break;
    }
#pragma unroll
    for (int k = 0; k < kMergeBatch; ++k) {
      if (c0 + k < nch) {
        const float* e = sab + ((size_t)j * a.max_chunks + c0 + k) * 3;
        const float sa = e[0], sb = e[1];
#pragma unroll
        for (int q = 0; q < 4; ++q) o[q] = __fadd_rn(__fmul_rn(o[q], sa), __fmul_rn(word_value(dw[k][q]), sb));
        L = __fadd_rn(__fmul_rn(L, sa), __fmul_rn(e[2], sb));
      }
    }
  }
  const float inv = L > 0.0f ? 1.0f / L : 0.0f;
#pragma unroll
  for (int q = 0; q < 4; ++q) out[q] = o[q] * inv;
}

__device__ void attn_item(const Args& a, AttnSmem& sm, Ctrl& cs, const Worker& w, int l, int nch,
                          const AttnItem& it, const QkvConst& qc) {
  const int tid = w.tid, warp = w.warp, lane = w.lane, n = it.n;
  const unsigned tag = tag_of(w.epoch, l);
  unsigned long long* acc_l = acc_layer(a, w.par, l);
  {
    // q (three heads) and, in the chunk that holds it, the new token's K/V row: bias + scale * (step * total)
    const int d = tid;
    const bool has_new = it.nhist < n;  // the new token is row nhist of this chunk
    unsigned long long wq[kHalf], wk = 0, wv = 0, sq;
    Spin sp;
    while (true) {
#pragma unroll
      for (int j = 0; j < kHalf; ++j) wq[j] = ld_word(acc_l + q_head(it, j) * kHeadDim + d);
      if (has_new) {
        wk = ld_word(acc_l + kHidden + it.g * kHeadDim + d);
        wv = ld_word(acc_l + kHidden + kKvWidth + it.g * kHeadDim + d);
      }
      sq = ld_word(a.buf.steps + (size_t)l * 4 + kQkv);
      bool ok = tag_ok(sq, tag);
#pragma unroll
      for (int j = 0; j < kHalf; ++j) ok = ok && count_ok(wq[j], nseg(kQkv));
      if (has_new) ok = ok && count_ok(wk, nseg(kQkv)) && count_ok(wv, nseg(kQkv));
      if (ok || !sp.keep_going(w.abort_flag)) break;
    }
    const float st = word_value(sq);
    float qv[kHalf], kv = 0.f, vv = 0.f;
#pragma unroll
    for (int j = 0; j < kHalf; ++j)
      qv[j] = __fmaf_rn(qc.qs[j], (float)((double)packed_total(wq[j], nseg(kQkv)) * (double)st), qc.qb[j]);
    if (has_new) {
      kv = __fmaf_rn(qc.ks, (float)((double)packed_total(wk, nseg(kQkv)) * (double)st), qc.kb);
      vv = __fmaf_rn(qc.vs, (float)((double)packed_total(wv, nseg(kQkv)) * (double)st), qc.vb);
    }
#pragma unroll
    for (int j = 0; j < kHalf; ++j) sm.qs[j][kcol(d)] = qv[j];
    if (has_new) sm.ks[it.nhist][kcol(d)] = kv;
    named_sync(kBarW, kWorkers);
    float qr[kHalf], kr = 0.f;
#pragma unroll
    for (int j = 0; j < kHalf; ++j) qr[j] = rope(qv[j], sm.qs[j][kcol(d ^ 64)], d, qc.rc, qc.rs);
    if (has_new) kr = rope(kv, sm.ks[it.nhist][kcol(d ^ 64)], d, qc.rc, qc.rs);
    named_sync(kBarW, kWorkers);
#pragma unroll
    for (int j = 0; j < kHalf; ++j) sm.qs[j][kcol(d)] = qr[j];
    if (has_new) {
      sm.ks[it.nhist][kcol(d)] = kr;
      sm.vs[it.nhist][d] = vv;
      if (it.hp == 0) {  // the cache row of this step, for later steps
        float* krow = w.kvrow + ((size_t)l * 2) * kPage * kKvWidth + it.g * kHeadDim + d;
        krow[0] = kr;
        krow[kPage * kKvWidth] = vv;
      }
    }
  }
  cp_async_wait_all();
  named_sync(kBarW, kWorkers);
  if (tid == 0) stamp(a, l, stack::kTraceAttnQ);
  const float scaling = kAttentionScaling;
  {
    // thread = (key, half of the head dims): three heads over 64 dims, the two halves added
    const int key = tid >> 1, c0 = (tid & 1) * kHalfCol;
    float s0 = 0.f, s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int f = 0; f < 16; ++f) {
      const float4 kk = *reinterpret_cast<const float4*>(&sm.ks[key][c0 + 4 * f]);
      const float4 x0 = *reinterpret_cast<const float4*>(&sm.qs[0][c0 + 4 * f]);
      const float4 x1 = *reinterpret_cast<const float4*>(&sm.qs[1][c0 + 4 * f]);
      const float4 x2 = *reinterpret_cast<const float4*>(&sm.qs[2][c0 + 4 * f]);
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
#pragma unroll 8
  for (int key = 0; key < n; ++key) {
    const float vv = sm.vs[key][tid];
    const float4 e = *reinterpret_cast<const float4*>(&sm.es[key][0]);
    acc[0] = fmaf(e.x, vv, acc[0]);
    acc[1] = fmaf(e.y, vv, acc[1]);
    acc[2] = fmaf(e.z, vv, acc[2]);
  }
#pragma unroll
  for (int j = 0; j < kHalf; ++j) st_word(part_ptr(a, l, q_head(it, j), it.c) + 4 + tid, tagged(tag, acc[j]));
  if (tid < 2 * kHalf) {
    const int j = tid >> 1;
    st_word(part_ptr(a, l, q_head(it, j), it.c) + (tid & 1), tagged(tag, (tid & 1) ? sm.ls[j] : sm.ms[j]));
  }
  if (tid == 0) stamp(a, l, stack::kTraceAttnPart);
  // the item of the group's last chunk merges the group: it reads the other chunks' partials as tagged
  // words, waiting on the data itself
  if (it.c != nch - 1) return;
  const int group = it.g * 2 + it.hp;
  named_sync(kBarW, kWorkers);  // this item's own partial is written
  // thread = 4 dims of one of the three heads (96 threads); the context and the group's max |ctx| as tagged
  // words. The chunk rows in shared memory are free now: they hold the rescale factors.
  float m = 0.0f;
  float out[4];
  merge_group(a, &sm.ks[0][0], w, l, q_head(it, 0), nch, out);
  if (tid < kHalf * 32) {
    const int j = tid >> 5, d0 = 4 * lane, h = q_head(it, j);
    unsigned long long* cw = a.buf.ctx + (size_t)(l & 1) * kHidden + h * kHeadDim + d0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      st_word(cw + e, tagged(tag, out[e]));
      m = fmaxf(m, fabsf(out[e]));
    }
  }
  m = warp_max(m);
  if (lane == 0) cs.redf[warp] = m;
  named_sync(kBarW, kWorkers);
  if (tid == 0) {
    st_word(a.buf.cmax + (size_t)(l & 1) * kMergeGroups + group,
            tagged(tag, fmaxf(fmaxf(cs.redf[0], cs.redf[1]), cs.redf[2])));
    stamp(a, l, stack::kTraceAttnMerge);
  }
}

// This CTA's first attention item of layer l (items blockIdx.x, + gridDim.x, ...): its history rows and
// constants do not depend on the layer's q|k|v, so they are requested before the q|k|v stage.
struct AttnPlan {
  bool active;
  int nch, total;
};

__device__ void attention_prefetch(const Args& a, AttnSmem& sm, const Worker& w, int l, AttnPlan& p) {
  p.nch = (w.pos + 1 + kChunk - 1) / kChunk;
  p.total = kMergeGroups * p.nch;
  p.active = (int)blockIdx.x < p.total;
  if (!p.active) return;
  named_sync(kBarW, kWorkers);  // the attention buffers are free (the previous layer's items are done)
  const AttnItem it = attn_decode(a, w, l, blockIdx.x, p.nch);
  attn_load_rows(sm, it, 0, it.nhist, w.tid);
}

__device__ void attention_stage(const Args& a, AttnSmem& sm, Ctrl& cs, const Worker& w, int l, const AttnPlan& p) {
  if (!p.active) return;
  AttnItem it = attn_decode(a, w, l, blockIdx.x, p.nch);
  QkvConst qc;
  qkv_const(a, w, l, it, qc);
  if (w.tid == 0) stamp(a, l, stack::kTraceWait + 1);
  for (int i = blockIdx.x;;) {
    attn_item(a, sm, cs, w, l, p.nch, it, qc);
    i += gridDim.x;
    if (i >= p.total) break;
    const AttnItem nx = attn_decode(a, w, l, i, p.nch);
    if (nx.g != it.g || nx.hp != it.hp) qkv_const(a, w, l, nx, qc);
    it = nx;
    named_sync(kBarW, kWorkers);  // previous chunk done with the shared buffers
    attn_load_rows(sm, it, 0, it.nhist, w.tid);
  }
  if (w.tid == 0) stamp(a, l, stack::kTraceDone + 1);
}

// ---------------------------------------------------------------------------------------------------
// the worker loop
// ---------------------------------------------------------------------------------------------------
__device__ void workers(const Args& a, uint8_t* ring, uint8_t* attn, uint8_t* dig, Ctrl& cs, uint32_t i0,
                        uint32_t i1, unsigned epoch, unsigned* abort_flag) {
  Worker w;
  w.tid = threadIdx.x - 32;
  w.lane = threadIdx.x & 31;
  w.warp = w.tid >> 5;
  w.epoch = epoch;
  w.par = epoch & 1u;
  w.s = 0;
  w.ph = 0;
  w.abort_flag = abort_flag;
  w.pos = __ldcg(&a.pos[0]);
  w.seq = __ldcg(&a.seq[0]);
  {
    const KvView kv0{a.kv_pool, nullptr, a.page_table, 0, a.max_pages};
    w.kvrow = kv_row(kv0, w.seq, w.pos, 0);
  }
  int si[kNumProj];  // this CTA's item of each projection, or -1
  for (int s = 0; s < kNumProj; ++s) si[s] = -1;
  for (uint32_t i = i0; i < i1; ++i) si[a.items[i].stage] = (int)i;
  AttnSmem& asm_ = *reinterpret_cast<AttnSmem*>(attn);
  // The CTA holding q|k|v tile 0, segment 0 writes each layer's output y (read by the LM head and the
  // hidden-state dump).
  const bool y_writer = si[kQkv] >= 0 && a.items[si[kQkv]].tile == 0 && a.items[si[kQkv]].seg == 0;
  const bool tr = w.tid == 0;
  for (int l = 0; l < kLayers; ++l) {
    const LayerDev& L = a.layers[l];
    const unsigned tag = tag_of(epoch, l);
    unsigned long long* acc = acc_layer(a, w.par, l);
    float4 wv[3];
    AttnPlan plan;
    attention_prefetch(a, asm_, w, l, plan);
    // ---- q|k|v: input = previous layer's output (or the token's embedding row) -----------------------
    if (si[kQkv] >= 0) {
      const Item it = a.items[si[kQkv]];
      load_vec(L.input_ln, w.tid, wv);
      float v[3][4];
      if (l == 0) {
        const int tok = __ldcg(&a.tokens[0]);
        const __half* row = reinterpret_cast<const __half*>(a.embed) + (size_t)tok * kHidden;
#pragma unroll
        for (int j = 0; j < 3; ++j) {
          const uint2 u = __ldg(reinterpret_cast<const uint2*>(row + 512 * j + 4 * w.tid));
          const __half2 h0 = *reinterpret_cast<const __half2*>(&u.x), h1 = *reinterpret_cast<const __half2*>(&u.y);
          v[j][0] = __low2float(h0);
          v[j][1] = __high2float(h0);
          v[j][2] = __low2float(h1);
          v[j][3] = __high2float(h1);
        }
      } else {
        const LayerDev& P = a.layers[l - 1];
        float4 os[3], ds[3];
        load_vec(P.o_s, w.tid, os);
        load_vec(P.down_s, w.tid, ds);
        load_y(a, w, l - 1, os, ds, si[kGu] >= 0 ? cs.av : nullptr, v);
        if (y_writer) {
          float* yw = ((l - 1) & 1) ? a.y1 : a.y0;
          float* dw = a.dump ? a.dump + (size_t)(l - 1) * kHidden : nullptr;
#pragma unroll
          for (int j = 0; j < 3; ++j) {
            const float4 yv = make_float4(v[j][0], v[j][1], v[j][2], v[j][3]);
            *reinterpret_cast<float4*>(yw + 512 * j + 4 * w.tid) = yv;
            if (dw) *reinterpret_cast<float4*>(dw + 512 * j + 4 * w.tid) = yv;
          }
        }
      }
      if (tr) stamp(a, l, stack::kTraceWait + 0);
      const float step = norm_and_step(cs, v, true, wv, w);
      if (w.tid == 0) st_word(a.buf.steps + (size_t)l * 4 + kQkv, tagged(tag, step));
      row_digits(dig, v, umma::digit_recip(step), it.kb0, it.kb1, w.tid);
      named_sync(kBarW, kWorkers);
      if (tr) stamp(a, l, stack::kTraceBuilt + 0);
      const long long tot = gemv_units(w, cs, a, ring, dig, it.kb1 - it.kb0);
      red_word(acc + acc_row(kQkv) + it.tile * 128 + w.tid, packed(tot));
      if (tr) stamp(a, l, stack::kTraceDone + 0);
    }
    // ---- attention chunks --------------------------------------------------------------------------
    attention_stage(a, asm_, cs, w, l, plan);
    // ---- o_proj: the merged context of this item's three heads; the step from every group's max ------
    if (si[kO] >= 0) {
      const Item it = a.items[si[kO]];
      if (tr) stamp(a, l, stack::kTraceWait + 2);
      const unsigned long long* cm = a.buf.cmax + (size_t)(l & 1) * kMergeGroups;
      const int nel = (it.kb1 - it.kb0) * kKBlock;  // this item's context elements, 4 per thread
      const unsigned long long* cw = a.buf.ctx + (size_t)(l & 1) * kHidden + it.kb0 * kKBlock + 4 * w.tid;
      unsigned long long x[4] = {0, 0, 0, 0}, mw[kMergeGroups];
      Spin sp;
      while (true) {
        if (4 * w.tid < nel) {
          ld_word2(cw, x[0], x[1]);
          ld_word2(cw + 2, x[2], x[3]);
        }
#pragma unroll
        for (int gi = 0; gi < kMergeGroups; ++gi) mw[gi] = ld_word(cm + gi);
        bool ok = true;
#pragma unroll
        for (int gi = 0; gi < kMergeGroups; ++gi) ok = ok && tag_ok(mw[gi], tag);
        if (4 * w.tid < nel) ok = ok && tag_ok(x[0], tag) && tag_ok(x[1], tag) && tag_ok(x[2], tag) && tag_ok(x[3], tag);
        if (ok || !sp.keep_going(abort_flag)) break;
      }
      float mx = 0.0f;
#pragma unroll
      for (int gi = 0; gi < kMergeGroups; ++gi) mx = fmaxf(mx, word_value(mw[gi]));
      const float step = mx > 0.0f ? mx / umma::kDigitRange : 1.0f;
      if (w.tid == 0) st_word(a.buf.steps + (size_t)l * 4 + kO, tagged(tag, step));
      if (4 * w.tid < nel) {
        const float v[4] = {word_value(x[0]), word_value(x[1]), word_value(x[2]), word_value(x[3])};
        put_digits(dig, 4 * w.tid, v, umma::digit_recip(step));
      }
      named_sync(kBarW, kWorkers);
      if (tr) stamp(a, l, stack::kTraceBuilt + 2);
      const long long tot = gemv_units(w, cs, a, ring, dig, it.kb1 - it.kb0);
      red_word(acc + acc_row(kO) + it.tile * 128 + w.tid, packed(tot));
      if (tr) stamp(a, l, stack::kTraceDone + 2);
    }
    // ---- gate|up: input = RMSNorm(a); h = SiLU(gate) * up for this tile's 64 columns -----------------
    if (si[kGu] >= 0) {
      const Item it = a.items[si[kGu]];
      load_vec(L.post_ln, w.tid, wv);
      float4 os[3];
      load_vec(L.o_s, w.tid, os);
      const int row = w.tid < 64 ? it.tile * 64 + w.tid : kInter + it.tile * 64 + (w.tid - 64);
      const float gsc = __ldg(L.gu_s + row);
      float v[3][4];
      load_a(a, w, l, os, v);
#pragma unroll
      for (int j = 0; j < 3; ++j)  // a, for this CTA's load of the layer output y (same thread, same elements)
        *reinterpret_cast<float4*>(cs.av + 512 * j + 4 * w.tid) = make_float4(v[j][0], v[j][1], v[j][2], v[j][3]);
      if (tr) stamp(a, l, stack::kTraceWait + 3);
      const float step = norm_and_step(cs, v, true, wv, w);
      row_digits(dig, v, umma::digit_recip(step), 0, nkb(kGu), w.tid);
      named_sync(kBarW, kWorkers);
      if (tr) stamp(a, l, stack::kTraceBuilt + 3);
      const long long tot = gemv_units(w, cs, a, ring, dig, it.kb1 - it.kb0, l);
      cs.ys[w.tid] = gsc * (float)((double)tot * (double)step);
      named_sync(kBarW, kWorkers);
      if (w.tid < 64) {  // warps 0 and 1: gate row tid pairs with up row 64 + tid
        const float gv = cs.ys[w.tid], uv = cs.ys[w.tid + 64];
        const float silu = __fdiv_rn(gv, __fadd_rn(1.0f, expf(-gv)));
        const float hv = __fmul_rn(silu, uv);
        st_word(a.buf.h + (size_t)(l & 1) * kInter + it.tile * 64 + w.tid, tagged(tag, hv));
        const float m = warp_max(fabsf(hv));
        if (w.lane == 0) cs.redf[w.warp] = m;
      }
      named_sync(kBarW, kWorkers);
      if (w.tid == 0)
        st_word(a.buf.hmax + (size_t)(l & 1) * kGuItems + it.tile, tagged(tag, fmaxf(cs.redf[0], cs.redf[1])));
      if (tr) stamp(a, l, stack::kTraceDone + 3);
    }
    // ---- down: input = h, step from the max |h| of every gate|up item ---------------------------------
    if (si[kDown] >= 0) {
      const Item it = a.items[si[kDown]];
      const unsigned long long* hm = a.buf.hmax + (size_t)(l & 1) * kGuItems;
      // every gate|up item's max |h| (for the step) and this thread's h values (at most 2 x 4 per thread),
      // read together until all are current
      const int n4 = (it.kb1 - it.kb0) * (kKBlock / 4);
      static_assert(seg_len(stack::kDown) * (kKBlock / 4) <= 2 * kWorkers, "two h quads per thread");
      const unsigned long long* hp = a.buf.h + (size_t)(l & 1) * kInter + it.kb0 * kKBlock;
      const bool has1 = w.tid + kWorkers < kGuItems, f0 = w.tid < n4, f1 = w.tid + kWorkers < n4;
      unsigned long long x0 = 0, x1 = 0, hx[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
      {
        Spin sp;
        while (true) {
          x0 = ld_word(hm + w.tid);
          if (has1) x1 = ld_word(hm + w.tid + kWorkers);
          if (f0) {
            ld_word2(hp + 4 * w.tid, hx[0][0], hx[0][1]);
            ld_word2(hp + 4 * w.tid + 2, hx[0][2], hx[0][3]);
          }
          if (f1) {
            ld_word2(hp + 4 * (w.tid + kWorkers), hx[1][0], hx[1][1]);
            ld_word2(hp + 4 * (w.tid + kWorkers) + 2, hx[1][2], hx[1][3]);
          }
          bool ok = tag_ok(x0, tag) && (!has1 || tag_ok(x1, tag));
#pragma unroll
          for (int e = 0; e < 4; ++e) ok = ok && (!f0 || tag_ok(hx[0][e], tag)) && (!f1 || tag_ok(hx[1][e], tag));
          if (ok || !sp.keep_going(abort_flag)) break;
        }
      }
      if (tr) stamp(a, l, stack::kTraceWait + 4);
      const float mx = block_max(cs, fmaxf(word_value(x0), has1 ? word_value(x1) : 0.0f), w);
      const float step = mx > 0.0f ? mx / umma::kDigitRange : 1.0f;
      if (w.tid == 0) st_word(a.buf.steps + (size_t)l * 4 + kDown, tagged(tag, step));
      const double rstep = umma::digit_recip(step);
#pragma unroll
      for (int b = 0; b < 2; ++b) {
        if (b == 0 ? f0 : f1) {
          const float hv[4] = {word_value(hx[b][0]), word_value(hx[b][1]), word_value(hx[b][2]), word_value(hx[b][3])};
          put_digits(dig, 4 * (w.tid + b * kWorkers), hv, rstep);
        }
      }
      named_sync(kBarW, kWorkers);
      if (tr) stamp(a, l, stack::kTraceBuilt + 4);
      const long long tot = gemv_units(w, cs, a, ring, dig, it.kb1 - it.kb0);
      red_word(acc + acc_row(kDown) + it.tile * 128 + w.tid, packed(tot));
      if (tr) stamp(a, l, stack::kTraceDone + 4);
    }
  }
  // the last layer's output, for the LM head (and the dump)
  if (y_writer) {
    const int l = kLayers - 1;
    float4 os[3], ds[3];
    load_vec(a.layers[l].o_s, w.tid, os);
    load_vec(a.layers[l].down_s, w.tid, ds);
    float v[3][4];
    load_y(a, w, l, os, ds, si[kGu] >= 0 ? cs.av : nullptr, v);
    float* yw = (l & 1) ? a.y1 : a.y0;
    float* dw = a.dump ? a.dump + (size_t)l * kHidden : nullptr;
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      const float4 yv = make_float4(v[j][0], v[j][1], v[j][2], v[j][3]);
      *reinterpret_cast<float4*>(yw + 512 * j + 4 * w.tid) = yv;
      if (dw) *reinterpret_cast<float4*>(dw + 512 * j + 4 * w.tid) = yv;
    }
  }
}

__global__ void __launch_bounds__(kThreads, 1) decode_bs1_kernel(const __grid_constant__ Args a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = align_smem_1024(smem_raw);
  uint8_t* ring = base;
  uint8_t* attn = base + (size_t)kRing * kUnitBytes;
  uint8_t* dig = attn + kAttnBytes;
  Ctrl& cs = *reinterpret_cast<Ctrl*>(dig + kDigitBytes);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t i0 = a.item_off[blockIdx.x], i1 = a.item_off[blockIdx.x + 1];
  unsigned* abort_flag = &a.sync->abort_flag.v;
  const unsigned epoch = __ldcg(&a.sync->epoch.v);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kRing; ++s) {
      mbar_init(&cs.full[s], 1);
      mbar_init(&cs.empty[s], kWorkers / 32);
    }
    mbar_fence_init();
  }
  __syncthreads();

  if (warp == 0) {
    if (lane == 0) producer(a, ring, cs, i0, i1, abort_flag);
    else clear_other_parity(a, epoch & 1u);
  } else {
    workers(a, ring, attn, dig, cs, i0, i1, epoch, abort_flag);
  }

  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned prev = atomicAdd(&a.sync->exit_cnt.v, 1u);
    if (prev == gridDim.x - 1) {  // every CTA is past its last wait: reset for the next launch
      __threadfence();
      a.sync->exit_cnt.v = 0u;
      a.sync->abort_flag.v = 0u;
      a.sync->epoch.v = epoch + 1u;
      __threadfence();
    }
  }
}

}  // namespace

stack::Schedule build_schedule(int ctas) {
  struct Cand {
    int stage, tile, seg, kb0, kb1;
  };
  std::vector<Cand> all;
  for (int s = 0; s < kNumProj; ++s)
    for (int tile = 0; tile < tiles(s); ++tile)
      for (int seg = 0; seg < nseg(s); ++seg) {
        const int kb0 = seg * seg_len(s), kb1 = std::min(nkb(s), kb0 + seg_len(s));
        if (kb0 < kb1) all.push_back({s, tile, seg, kb0, kb1});
      }
  // Largest items first onto the least-loaded CTA (load = 16 KB units streamed per layer) among those
  // without an item of the same projection. Ties go to the highest-numbered CTA for o_proj (the attention
  // items occupy the lowest-numbered CTAs just before it), to the lowest otherwise.
  std::stable_sort(all.begin(), all.end(), [](const Cand& x, const Cand& y) { return x.kb1 - x.kb0 > y.kb1 - y.kb0; });
  std::vector<int> load(ctas, 0);
  std::vector<std::vector<char>> has(kNumProj, std::vector<char>(ctas, 0));
  std::vector<std::vector<Cand>> per(ctas);
  stack::Schedule sc;
  for (const Cand& c : all) {
    int best = -1;
    for (int i = 0; i < ctas; ++i) {
      const int k = c.stage == kO ? ctas - 1 - i : i;
      if (has[c.stage][k]) continue;
      if (best < 0 || load[k] < load[best]) best = k;
    }
    if (best < 0) return sc;  // more items of one projection than CTAs: no schedule
    per[best].push_back(c);
    load[best] += c.kb1 - c.kb0;
    has[c.stage][best] = 1;
  }
  sc.off.push_back(0);
  for (int k = 0; k < ctas; ++k) {
    std::sort(per[k].begin(), per[k].end(), [](const Cand& x, const Cand& y) { return x.stage < y.stage; });
    for (const Cand& c : per[k]) {
      Item it;
      it.tile = (uint16_t)c.tile;
      it.stage = (uint8_t)c.stage;
      it.kb0 = (uint8_t)c.kb0;
      it.kb1 = (uint8_t)c.kb1;
      it.dslot = 0;
      it.seg = (uint16_t)c.seg;
      sc.items.push_back(it);
    }
    sc.off.push_back((uint32_t)sc.items.size());
    sc.max_units = std::max(sc.max_units, load[k]);
  }
  return sc;
}

size_t decode_bs1_smem() { return kSmemBytes; }

cudaError_t launch_decode_bs1(const Args& a, int ctas, cudaStream_t s) {
  cudaError_t e = ensure_smem_attr((const void*)decode_bs1_kernel, kSmemBytes);
  if (e != cudaSuccess) return e;
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
  return cudaLaunchKernelEx(&cfg, decode_bs1_kernel, a);
}

unsigned decode_bs1_kernel_error(bool reset) {
  unsigned v = 0;
  if (cudaMemcpyFromSymbol(&v, g_kernel_error, sizeof(v)) != cudaSuccess) return 0xFFFFFFFFu;
  if (reset && v) {
    const unsigned z = 0;
    cudaMemcpyToSymbol(g_kernel_error, &z, sizeof(z));
  }
  return v;
}

}  // namespace bs1
}  // namespace qb
