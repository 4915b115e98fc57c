// Shared constants, the reference's DDR layout, and the device-side restatement of the reference's
// elementwise operators with identical IEEE rounding.
//
// Model constants: hls/common/qwen2_model_config.h:7-52. Layout: hls/common/llm_memory_layout.h:55-149.
// Approximate operators: hls/prefill_only/qwen_prefill_attention_kernel.cpp:47-143 (host variant, not the
// __SYNTHESIS__ one). Every float operation in those operators is written with an explicit _rn intrinsic so
// nvcc cannot fuse a multiply and an add into an FMA: the reference's x86-64 -O2 build never fuses, and a
// fused operation rounds once where the reference rounds twice.
#pragma once

#include <cstdint>
#include <cstddef>

#ifdef __CUDACC__
#define QB_HD __host__ __device__ __forceinline__
#else
#define QB_HD inline
#endif

namespace qb {

constexpr int kHidden = 1536;
constexpr int kInter = 8960;
constexpr int kLayers = 28;
constexpr int kHeads = 12;
constexpr int kKvHeads = 2;
constexpr int kHeadDim = 128;
constexpr int kKvWidth = kKvHeads * kHeadDim;  // 256
constexpr int kGroups = kHeads / kKvHeads;     // 6 query heads share one KV head
constexpr int kQkvRows = kHidden + 2 * kKvWidth;  // 2048: q | k | v rows, contiguous in the layout
constexpr int kVocab = 151936;
constexpr int kMaxSeq = 32768;
constexpr float kEps = 1.0e-6f;
constexpr float kRopeTheta = 1000000.0f;

// Reference status codes (qwen_decode_top_wrapper.cpp:11-12, qwen_prefill_top_core.h:7-9).
constexpr int kStatusOk = 0;
constexpr int kStatusInvalid = 1;
constexpr int kStatusCapacity = 2;
constexpr int kStatusDecodeDescriptor = 10;
constexpr int kStatusDecodePort = 11;
constexpr int kStatusPrefillDescriptor = 20;
constexpr int kStatusPrefillPort = 21;
constexpr int kStatusPrefillWindow = 22;
// Codes that exist only in this implementation (the reference runs on the host and cannot fail this way).
constexpr int kStatusCuda = 30;      // a CUDA call failed; the message is in qwen_b200_last_error()
constexpr int kStatusNoDevice = 31;  // no CUDA device / extension unusable

// ------------------------------------------------------------------------------------------------
// Layer parameter layout. wbits = 4 is the reference layout (two nibbles per byte); wbits = 8 keeps
// the same field order with one byte per weight (the W8 track).
// ------------------------------------------------------------------------------------------------
struct LayerLayout {
  uint64_t input_ln, q_w, k_w, v_w, o_w, post_ln, gate_w, up_w, down_w;
  uint64_t q_b, k_b, v_b;
  uint64_t q_s, k_s, v_s, o_s, gate_s, up_s, down_s;
  uint64_t total;
};

QB_HD uint64_t weight_bytes(uint64_t out_dim, uint64_t in_dim, int wbits) { return out_dim * in_dim * wbits / 8; }

QB_HD LayerLayout layer_layout(int wbits) {
  LayerLayout l{};
  uint64_t off = 0;
  l.input_ln = off; off += kHidden * 4;
  l.q_w = off; off += weight_bytes(kHidden, kHidden, wbits);
  l.k_w = off; off += weight_bytes(kKvWidth, kHidden, wbits);
  l.v_w = off; off += weight_bytes(kKvWidth, kHidden, wbits);
  l.o_w = off; off += weight_bytes(kHidden, kHidden, wbits);
  l.post_ln = off; off += kHidden * 4;
  l.gate_w = off; off += weight_bytes(kInter, kHidden, wbits);
  l.up_w = off; off += weight_bytes(kInter, kHidden, wbits);
  l.down_w = off; off += weight_bytes(kHidden, kInter, wbits);
  l.q_b = off; off += kHidden * 4;
  l.k_b = off; off += kKvWidth * 4;
  l.v_b = off; off += kKvWidth * 4;
  l.q_s = off; off += kHidden * 4;
  l.k_s = off; off += kKvWidth * 4;
  l.v_s = off; off += kKvWidth * 4;
  l.o_s = off; off += kHidden * 4;
  l.gate_s = off; off += kInter * 4;
  l.up_s = off; off += kInter * 4;
  l.down_s = off; off += kHidden * 4;
  l.total = off;
  return l;
}

// Device view of one layer's parameters (all device pointers).
struct LayerDev {
  const uint8_t* qkv_w;   // [2048 rows][1536] codes: q | k | v contiguous
  const uint8_t* o_w;     // [1536][1536]
  const uint8_t* gu_w;    // [2 * 8960][1536]: gate | up contiguous
  const uint8_t* down_w;  // [1536][8960]
  const float* input_ln;  // [1536]
  const float* post_ln;   // [1536]
  const float* qkv_b;     // [2048]
  const float* qkv_s;     // [2048]
  const float* o_s;       // [1536]
  const float* gu_s;      // [2 * 8960]
  const float* down_s;    // [1536]
};

QB_HD LayerDev layer_dev_from_ddr(const uint8_t* weight_base, const float* scale_base, int wbits) {
  const LayerLayout l = layer_layout(wbits);
  LayerDev d;
  d.qkv_w = weight_base + l.q_w;
  d.o_w = weight_base + l.o_w;
  d.gu_w = weight_base + l.gate_w;
  d.down_w = weight_base + l.down_w;
  d.input_ln = scale_base + l.input_ln / 4;
  d.post_ln = scale_base + l.post_ln / 4;
  d.qkv_b = scale_base + l.q_b / 4;
  d.qkv_s = scale_base + l.q_s / 4;
  d.o_s = scale_base + l.o_s / 4;
  d.gu_s = scale_base + l.gate_s / 4;
  d.down_s = scale_base + l.down_s / 4;
  return d;
}

// ------------------------------------------------------------------------------------------------
// KV cache view: flat (the reference's token-major [t][kv_head][128] fp32, separate K and V bases)
// or paged (page table per sequence; a page holds kPage tokens of every layer's K and V).
// ------------------------------------------------------------------------------------------------
constexpr int kPage = 64;

struct KvView {
  float* k;                // flat: K base of this sequence/layer. paged: pool base
  float* v;                // flat: V base. paged: unused
  const int* page_table;   // nullptr => flat
  int layer;               // paged only
  int max_pages;           // paged only: row length of the page table
  int pool_pages = 0;      // paged only: pages in the pool (the extent of the decode attention's tensor maps)
};

// Floats per page: [layer][K|V][kPage][256].
constexpr uint64_t kPageFloats = (uint64_t)kLayers * 2ull * kPage * kKvWidth;

QB_HD float* kv_row(const KvView& kv, int seq, int token, int which /*0=K,1=V*/) {
  if (kv.page_table == nullptr) {
    return (which ? kv.v : kv.k) + (uint64_t)token * kKvWidth;
  }
  const int page = kv.page_table[seq * kv.max_pages + token / kPage];
  return kv.k + (uint64_t)page * kPageFloats + ((uint64_t)kv.layer * 2 + which) * kPage * kKvWidth +
         (uint64_t)(token % kPage) * kKvWidth;
}

// ------------------------------------------------------------------------------------------------
// Deterministic synthetic parameters (bit-identical to the oracle's generator): SplitMix64 finalizer
// and a 12-term Irwin-Hall sum of 16-bit uniforms.
// ------------------------------------------------------------------------------------------------
QB_HD uint64_t mix64(uint64_t x) {
  x ^= x >> 30;
  x *= 0xBF58476D1CE4E5B9ull;
  x ^= x >> 27;
  x *= 0x94D049BB133111EBull;
  x ^= x >> 31;
  return x;
}

QB_HD uint64_t synth_key(uint64_t seed, uint64_t stream) { return mix64(seed ^ mix64(stream + 0x9E3779B97F4A7C15ull)); }

#ifdef __CUDACC__
__device__ __forceinline__ float synth_normal_dev(uint64_t key, uint64_t index, float mean, float sigma) {
  long long sum = 0;
#pragma unroll
  for (uint64_t j = 0; j < 3; ++j) {
    const uint64_t h = mix64(key + index * 3ull + j);
    sum += (long long)(h & 0xFFFF) + (long long)((h >> 16) & 0xFFFF) + (long long)((h >> 32) & 0xFFFF) +
           (long long)((h >> 48) & 0xFFFF);
  }
  const float z = __fmul_rn(__ll2float_rn(2 * sum - 12 * 65535), 1.0f / 131072.0f);
  return __fadd_rn(__fmul_rn(z, sigma), mean);
}

// ------------------------------------------------------------------------------------------------
// Prefill approximations, bit-identical to the reference host code.
// ------------------------------------------------------------------------------------------------
constexpr float kPi = 3.14159265358979323846f;
constexpr float kTwoPi = 6.28318530717958647692f;
constexpr float kHalfPi = 1.57079632679489661923f;
constexpr float kAttentionScaling = 0.08838834764831845f;  // qwen_prefill_attention_kernel.cpp:28
constexpr float kRopeFreqStep = 0.8058421877614801f;      // qwen_prefill_attention_kernel.cpp:29

// qwen_prefill_attention_kernel.cpp:47-57
__device__ __forceinline__ float approx_sqrt(float value) {
  if (value <= 0.0f) return 0.0f;
  float guess = value > 1.0f ? value : 1.0f;
#pragma unroll
  for (int i = 0; i < 6; ++i) guess = __fmul_rn(0.5f, __fadd_rn(guess, __fdiv_rn(value, guess)));
  return guess;
}

// qwen_prefill_attention_kernel.cpp:59-85
__device__ __forceinline__ void approx_sincos(float angle, float* s, float* c) {
  float r = angle;
  while (r > kPi) r = __fsub_rn(r, kTwoPi);
  while (r < -kPi) r = __fadd_rn(r, kTwoPi);
  float cos_sign = 1.0f;
  if (r > kHalfPi) {
    r = __fsub_rn(kPi, r);
    cos_sign = -1.0f;
  } else if (r < -kHalfPi) {
    r = __fsub_rn(-kPi, r);
    cos_sign = -1.0f;
  }
  const float c6 = -1.0f / 5040.0f, c4 = 1.0f / 120.0f, c2 = -1.0f / 6.0f;
  const float d6 = -1.0f / 720.0f, d4 = 1.0f / 24.0f;
  const float x2 = __fmul_rn(r, r);
  float t = __fmul_rn(x2, c6);
  t = __fadd_rn(c4, t);
  t = __fmul_rn(x2, t);
  t = __fadd_rn(c2, t);
  t = __fmul_rn(x2, t);
  t = __fadd_rn(1.0f, t);
  *s = __fmul_rn(r, t);
  float u = __fmul_rn(x2, d6);
  u = __fadd_rn(d4, u);
  u = __fmul_rn(x2, u);
  u = __fadd_rn(-0.5f, u);
  u = __fmul_rn(x2, u);
  *c = __fmul_rn(cos_sign, __fadd_rn(1.0f, u));
}

// qwen_prefill_attention_kernel.cpp:87-110. Below -1 the argument is halved until it is >= -1 and
// the degree-6 Taylor value is squared back; above -1 there is no range reduction (so large positive
// arguments are far from exp, exactly as in the reference).
__device__ __forceinline__ float approx_exp(float value) {
  if (value <= -16.0f) return 0.0f;
  int half_steps = 0;
  float scaled = value;
  while (scaled < -1.0f) {
    scaled = __fmul_rn(scaled, 0.5f);
    ++half_steps;
  }
  float term = 1.0f, series = 1.0f;
#pragma unroll
  for (int degree = 1; degree <= 6; ++degree) {
    term = __fmul_rn(term, __fdiv_rn(scaled, (float)degree));
    series = __fadd_rn(series, term);
  }
  for (int i = 0; i < half_steps; ++i) series = __fmul_rn(series, series);
  return series > 0.0f ? series : 0.0f;
}

// Correctly rounded x / 3 and x / 5 without a division instruction: q = RN(x * RN(1/d)), the remainder
// x - d q is exact under one FMA, and RN(q + r * RN(1/d)) is the correctly rounded quotient (Markstein's
// correction step, P. Markstein, IBM J. Res. Dev. 34(1), 1990). Checked exhaustively against IEEE division
// over every finite fp32 x: identical except x = -0, which returns +0.
__device__ __forceinline__ float div_by_3_rn(float x) {
  const float c = 0x1.555556p-2f;  // RN(1/3)
  const float q = __fmul_rn(x, c);
  return __fmaf_rn(__fmaf_rn(-q, 3.0f, x), c, q);
}
__device__ __forceinline__ float div_by_5_rn(float x) {
  const float c = 0x1.99999ap-3f;  // RN(1/5)
  const float q = __fmul_rn(x, c);
  return __fmaf_rn(__fmaf_rn(-q, 5.0f, x), c, q);
}

// p ? a : b as one predicated select (a chain of ?: on data-dependent conditions can compile to branches).
__device__ __forceinline__ float select_f32(bool p, float a, float b) {
  float r;
  asm("{\n.reg .pred q;\nsetp.ne.u32 q, %3, 0;\nselp.f32 %0, %1, %2, q;\n}" : "=f"(r) : "f"(a), "f"(b), "r"((unsigned)p));
  return r;
}

// Two fp32 values in one 64-bit register, operated on by the paired fp32 instructions of sm_100
// (add / fma .rn .f32x2: each lane rounds exactly as the scalar instruction does).
struct F2 {
  unsigned long long v;
};
__device__ __forceinline__ F2 f2(float a, float b) {
  F2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r.v) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float f2_lo(F2 x) {
  float a;
  asm("{\n.reg .f32 u;\nmov.b64 {%0, u}, %1;\n}" : "=f"(a) : "l"(x.v));
  return a;
}
__device__ __forceinline__ float f2_hi(F2 x) {
  float b;
  asm("{\n.reg .f32 u;\nmov.b64 {u, %0}, %1;\n}" : "=f"(b) : "l"(x.v));
  return b;
}
__device__ __forceinline__ F2 add2(F2 a, F2 b) {
  F2 r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r.v) : "l"(a.v), "l"(b.v));
  return r;
}
__device__ __forceinline__ F2 fma2(F2 a, F2 b, F2 c) {
  F2 r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r.v) : "l"(a.v), "l"(b.v), "l"(c.v));
  return r;
}
// -0 pair read from constant memory, so that the code generator does not know its value (below).
static __constant__ float c_f2_negzero[2] = {-0.0f, -0.0f};
__device__ __forceinline__ F2 f2_negzero() { return f2(c_f2_negzero[0], c_f2_negzero[1]); }
// Paired product a b, rounded once: fma(a, b, -0) = RN(a b) for every a, b. The code generator was measured
// (B200) to merge mul.rn.f32x2 followed by add.rn.f32x2 into one fused multiply-add, and to fold an fma
// with a literal -0 addend the same way, either of which drops a rounding; an addend it cannot see through
// keeps the product rounded on its own.
__device__ __forceinline__ F2 mul2(F2 a, F2 b, F2 nz) { return fma2(a, b, nz); }
// RN(x / d) for d = 3 or 5 (correction step above), two lanes at once.
__device__ __forceinline__ F2 div_const2(F2 x, float d, float rcp, F2 nz) {
  const F2 c = f2(rcp, rcp), q = mul2(x, c, nz);
  return fma2(fma2(q, f2(-d, -d), x), c, q);
}

// approx_exp in straight-line form (no loops, no branches), two values at a time on the paired fp32 pipe:
// - the halving loop runs while scaled < -1, i.e. h = [v < -1] + [v < -2] + [v < -4] + [v < -8] times for
//   v > -16, and each halving is exact (|scaled| >= 1 before it), so scaled = v * 2^-h in one exact multiply;
// - the six divisions by the term degree: /1 and the power-of-two degrees are exact multiplications, /3 and
//   /5 use the correction step above, and /6 = (x * 0.5) / 3 (x * 0.5 is exact unless |x| < 2^-125, where
//   the sixth term underflows to zero in both forms);
// - the h squarings are the same chain of products, selected by the same comparisons.
// Same result as approx_exp for every input: finite ones (the zero sign of a quotient cannot reach the series,
// whose first term is 1), -inf and nan (0), and +inf (the series diverges to +inf; the correction steps
// would give nan, so it is selected explicitly). nz = f2_negzero().
__device__ __forceinline__ void approx_exp_fast2(float v0, float v1, float& r0, float& r1, F2 nz) {
  const bool a1 = v0 < -1.0f, a2 = v0 < -2.0f, a4 = v0 < -4.0f, a8 = v0 < -8.0f;
  const bool b1 = v1 < -1.0f, b2 = v1 < -2.0f, b4 = v1 < -4.0f, b8 = v1 < -8.0f;
  const int h0 = (int)a1 + (int)a2 + (int)a4 + (int)a8, h1 = (int)b1 + (int)b2 + (int)b4 + (int)b8;
  const F2 scaled = mul2(f2(v0, v1), f2(__int_as_float((127 - h0) << 23), __int_as_float((127 - h1) << 23)), nz);
  const F2 half = mul2(scaled, f2(0.5f, 0.5f), nz);
  const F2 q3 = div_const2(scaled, 3.0f, 0x1.555556p-2f, nz), q4 = mul2(scaled, f2(0.25f, 0.25f), nz);
  const F2 q5 = div_const2(scaled, 5.0f, 0x1.99999ap-3f, nz), q6 = div_const2(half, 3.0f, 0x1.555556p-2f, nz);
  F2 term = scaled, series = add2(f2(1.0f, 1.0f), scaled);
  term = mul2(term, half, nz);
  series = add2(series, term);
  term = mul2(term, q3, nz);
  series = add2(series, term);
  term = mul2(term, q4, nz);
  series = add2(series, term);
  term = mul2(term, q5, nz);
  series = add2(series, term);
  term = mul2(term, q6, nz);
  series = add2(series, term);
  const F2 s2 = mul2(series, series, nz), s4 = mul2(s2, s2, nz), s8 = mul2(s4, s4, nz), s16 = mul2(s8, s8, nz);
  float x = f2_lo(series), y = f2_hi(series);
  x = a1 ? f2_lo(s2) : x;
  y = b1 ? f2_hi(s2) : y;
  x = a2 ? f2_lo(s4) : x;
  y = b2 ? f2_hi(s4) : y;
  x = a4 ? f2_lo(s8) : x;
  y = b4 ? f2_hi(s8) : y;
  x = a8 ? f2_lo(s16) : x;
  y = b8 ? f2_hi(s16) : y;
  x = (v0 <= -16.0f || !(x > 0.0f)) ? 0.0f : x;
  y = (v1 <= -16.0f || !(y > 0.0f)) ? 0.0f : y;
  r0 = v0 > 3.402823466e38f ? v0 : x;
  r1 = v1 > 3.402823466e38f ? v1 : y;
}

// One value (the paired form with both lanes on it).
__device__ __forceinline__ float approx_exp_fast(float value) {
  float r, same;
  approx_exp_fast2(value, value, r, same, f2_negzero());
  return r;
}

// Round-to-nearest-even to bf16, kept in fp32 (verification/reference_wrapper_backend.py:40-46).
__device__ __forceinline__ float round_bf16(float x) {
  uint32_t b = __float_as_uint(x);
  b += 0x7FFFu + ((b >> 16) & 1u);
  return __uint_as_float(b & 0xFFFF0000u);
}

// Programmatic dependent launch: wait for the preceding kernel's writes / let the next kernel start.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" :::); }
#endif  // __CUDACC__

}  // namespace qb
