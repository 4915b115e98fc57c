// Host runtime behind the drop-in C-ABI: device context, staging of the caller's (host) buffers into
// HBM, the RoPE tables, and the per-call kernel sequences for decode and prefill.
//
// The reference ABI passes host arrays on every call and keeps no state (hls/decode_only/
// qwen_decode_host_wrapper.cpp, hls/prefill_only/qwen_prefill_host_wrapper.cpp). This runtime copies
// exactly the bytes the reference reads, runs the kernels on one stream, copies back exactly the bytes
// the reference writes, and synchronises before returning. Device buffers are allocated once and grown
// on demand; calls are serialised by a mutex (the reference is re-entrant; callers here are
// single-threaded ctypes loops).
#include <cuda_runtime.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "attention_tc.h"
#include "layer0_ref.h"
#include "decode_bs1.h"
#include "decode_stack.h"
#include "qgemm.h"
#include "lmhead.h"
#include "tgemm.h"
#include "qwen_kernels.cuh"
#include "runtime.h"

namespace qb {

namespace {
thread_local std::string g_error;
int g_prefill_capacity = 0;

struct Buf {
  void* p = nullptr;
  size_t bytes = 0;
};

cudaError_t ensure(Buf& b, size_t bytes) {
  if (b.bytes >= bytes) return cudaSuccess;
  if (b.p) cudaFree(b.p);
  b.p = nullptr;
  b.bytes = 0;
  size_t want = bytes + bytes / 4 + 4096;
  cudaError_t e = cudaMalloc(&b.p, want);
  if (e != cudaSuccess) return e;
  b.bytes = want;
  return cudaSuccess;
}

struct Ctx {
  int device = -1;
  cudaStream_t stream = nullptr;
  Buf wimg, simg;          // device DDR images of one layer (weights / scale-space floats)
  Buf x, q, ctx, a, h, out, kc, vc, attn_part, counters;
  Buf dpos, dseq;
  Buf rope_dec_cos, rope_dec_sin, rope_pre_cos, rope_pre_sin;
  int rope_dec_len = 0, rope_pre_len = 0;
  std::vector<float> host_cos, host_sin;
  bool counters_zeroed = false;
  size_t counters_bytes = 0;
  // int8 tensor-core projections (wbits 8): split-K scratch (decode), digit planes and steps (prefill)
  QgemmScratch qsc{nullptr, nullptr};
  Buf planes, psteps;
  Buf attn;     // tensor-core prefill attention scratch
  Buf qkv_raw;  // W8 prefill: biased q|k|v rows before RoPE
  // layer0 reference layers: fp32 weights and activations
  Buf l0w, l0a;
  // zero-weight layer for the stub entry points
  Buf zw, zs;
  LayerPtrs zero{};
  bool zero_ready = false;
};

std::mutex g_mu;
Ctx g_ctx;

#define QB_TRY(expr)                                                                      \
  do {                                                                                    \
    cudaError_t _e = (expr);                                                              \
    if (_e != cudaSuccess) {                                                              \
      set_error("%s failed: %s (%s:%d)", #expr, cudaGetErrorString(_e), __FILE__, __LINE__); \
      return kStatusCuda;                                                                 \
    }                                                                                     \
  } while (0)

int init_ctx(Ctx& c) {
  int dev = 0;
  if (const char* env = std::getenv("QWEN_B200_DEVICE")) dev = std::atoi(env);
  if (c.device == dev) return 0;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0) {
    set_error("no CUDA device is visible: the B200 extension cannot run here");
    return kStatusNoDevice;
  }
  QB_TRY(cudaSetDevice(dev));
  QB_TRY(cudaStreamCreateWithFlags(&c.stream, cudaStreamNonBlocking));
  c.device = dev;
  return 0;
}

// Decode RoPE cos/sin for positions [0, need): double pow/cos/sin on the host, cast to float, exactly as
// hls/decode_only/qwen_decode_attention_kernel.cpp:29-34; uploaded to a device table.
int ensure_decode_rope(Ctx& c, int need) {
  if (need <= c.rope_dec_len) return 0;
  int len = c.rope_dec_len ? c.rope_dec_len : 256;
  while (len < need) len *= 2;
  if (len > kMaxSeq + 1) len = kMaxSeq + 1;
  const int old = (int)(c.host_cos.size() / 64);
  c.host_cos.resize((size_t)len * 64);
  c.host_sin.resize((size_t)len * 64);
  for (int pos = old; pos < len; ++pos) {
    for (int pair = 0; pair < 64; ++pair) {
      const double angle =
          (double)pos * std::pow((double)kRopeTheta, -2.0 * (double)pair / (double)kHeadDim);
      c.host_cos[(size_t)pos * 64 + pair] = (float)std::cos(angle);
      c.host_sin[(size_t)pos * 64 + pair] = (float)std::sin(angle);
    }
  }
  QB_TRY(ensure(c.rope_dec_cos, (size_t)len * 64 * 4));
  QB_TRY(ensure(c.rope_dec_sin, (size_t)len * 64 * 4));
  QB_TRY(cudaMemcpyAsync(c.rope_dec_cos.p, c.host_cos.data(), (size_t)len * 64 * 4, cudaMemcpyHostToDevice, c.stream));
  QB_TRY(cudaMemcpyAsync(c.rope_dec_sin.p, c.host_sin.data(), (size_t)len * 64 * 4, cudaMemcpyHostToDevice, c.stream));
  QB_TRY(cudaStreamSynchronize(c.stream));
  c.rope_dec_len = len;
  return 0;
}

int ensure_prefill_rope(Ctx& c, int need) {
  if (need <= c.rope_pre_len) return 0;
  int len = c.rope_pre_len ? c.rope_pre_len : 128;
  while (len < need) len *= 2;
  QB_TRY(ensure(c.rope_pre_cos, (size_t)len * 64 * 4));
  QB_TRY(ensure(c.rope_pre_sin, (size_t)len * 64 * 4));
  QB_TRY(launch_prefill_rope_table(len, (float*)c.rope_pre_cos.p, (float*)c.rope_pre_sin.p, c.stream));
  c.rope_pre_len = len;
  return 0;
}

// Copy the tensors a half-layer needs into the device DDR images at the layout offsets of `wbits`.
int stage_layer(Ctx& c, int wbits, const LayerPtrs& L, bool attention, bool mlp, LayerDev* out) {
  const LayerLayout l = layer_layout(wbits);
  QB_TRY(ensure(c.wimg, l.total));
  QB_TRY(ensure(c.simg, l.total + 16));
  uint8_t* w = (uint8_t*)c.wimg.p;
  float* s = (float*)c.simg.p;
  auto cpw = [&](uint64_t off, const uint8_t* src, uint64_t n) {
    return cudaMemcpyAsync(w + off, src, n, cudaMemcpyDefault, c.stream);
  };
  auto cpf = [&](uint64_t off, const float* src, uint64_t n) {
    return cudaMemcpyAsync(s + off / 4, src, n * 4, cudaMemcpyDefault, c.stream);
  };
  if (attention) {
    QB_TRY(cpw(l.q_w, L.q_w, weight_bytes(kHidden, kHidden, wbits)));
    QB_TRY(cpw(l.k_w, L.k_w, weight_bytes(kKvWidth, kHidden, wbits)));
    QB_TRY(cpw(l.v_w, L.v_w, weight_bytes(kKvWidth, kHidden, wbits)));
    QB_TRY(cpw(l.o_w, L.o_w, weight_bytes(kHidden, kHidden, wbits)));
    QB_TRY(cpf(l.input_ln, L.input_ln, kHidden));
    QB_TRY(cpf(l.q_b, L.q_b, kHidden));
    QB_TRY(cpf(l.k_b, L.k_b, kKvWidth));
    QB_TRY(cpf(l.v_b, L.v_b, kKvWidth));
    QB_TRY(cpf(l.q_s, L.q_s, kHidden));
    QB_TRY(cpf(l.k_s, L.k_s, kKvWidth));
    QB_TRY(cpf(l.v_s, L.v_s, kKvWidth));
    QB_TRY(cpf(l.o_s, L.o_s, kHidden));
  }
  if (mlp) {
    QB_TRY(cpw(l.gate_w, L.gate_w, weight_bytes(kInter, kHidden, wbits)));
    QB_TRY(cpw(l.up_w, L.up_w, weight_bytes(kInter, kHidden, wbits)));
    QB_TRY(cpw(l.down_w, L.down_w, weight_bytes(kHidden, kInter, wbits)));
    QB_TRY(cpf(l.post_ln, L.post_ln, kHidden));
    QB_TRY(cpf(l.gate_s, L.gate_s, kInter));
    QB_TRY(cpf(l.up_s, L.up_s, kInter));
    QB_TRY(cpf(l.down_s, L.down_s, kHidden));
  }
  *out = layer_dev_from_ddr(w, s, wbits);
  return 0;
}

}  // namespace

void set_error(const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_error = buf;
}

int prefill_seq_capacity() {
  if (g_prefill_capacity == 0) {
    int cap = 128;
    if (const char* env = std::getenv("QWEN_B200_PREFILL_SEQ_CAPACITY")) {
      const int v = std::atoi(env);
      if (v > 0 && v <= kMaxSeq) cap = v;
    }
    g_prefill_capacity = cap;
  }
  return g_prefill_capacity;
}

LayerPtrs layer_ptrs_from_ddr(const uint8_t* weight_ddr, uint64_t wb, const float* scale_ddr, uint64_t sb,
                              int wbits) {
  const LayerLayout l = layer_layout(wbits);
  LayerPtrs p;
  p.q_w = weight_ddr + wb + l.q_w;
  p.k_w = weight_ddr + wb + l.k_w;
  p.v_w = weight_ddr + wb + l.v_w;
  p.o_w = weight_ddr + wb + l.o_w;
  p.gate_w = weight_ddr + wb + l.gate_w;
  p.up_w = weight_ddr + wb + l.up_w;
  p.down_w = weight_ddr + wb + l.down_w;
  auto f = [&](uint64_t off) { return scale_ddr + (sb + off) / 4; };
  p.input_ln = f(l.input_ln);
  p.post_ln = f(l.post_ln);
  p.q_b = f(l.q_b);
  p.k_b = f(l.k_b);
  p.v_b = f(l.v_b);
  p.q_s = f(l.q_s);
  p.k_s = f(l.k_s);
  p.v_s = f(l.v_s);
  p.o_s = f(l.o_s);
  p.gate_s = f(l.gate_s);
  p.up_s = f(l.up_s);
  p.down_s = f(l.down_s);
  return p;
}

// W8 layers run their projections on the int8 tensor cores: TMA descriptors of the staged image.
int ensure_qgemm(Ctx& c, const LayerDev& D, QgemmLayerMaps* maps) {
  if (c.qsc.acc == nullptr) {
    QB_TRY(cudaMalloc(&c.qsc.acc, qgemm_acc_ints() * 4));
    QB_TRY(cudaMalloc(&c.qsc.cnt, qgemm_counter_count() * 4));
    QB_TRY(cudaMemset(c.qsc.acc, 0, qgemm_acc_ints() * 4));
    QB_TRY(cudaMemset(c.qsc.cnt, 0, qgemm_counter_count() * 4));
  }
  if (!qgemm_make_layer_maps(maps, D)) {
    set_error("cuTensorMapEncodeTiled failed");
    return kStatusCuda;
  }
  return 0;
}

int run_decode(int wbits, const LayerPtrs& L, bool attention, bool mlp, const float* x, int past, float* k_cache,
               float* v_cache, float* attn_out, float* out) {
  std::lock_guard<std::mutex> lock(g_mu);
  Ctx& c = g_ctx;
  if (int st = init_ctx(c)) return st;
  LayerDev D;
  if (int st = stage_layer(c, wbits, L, attention, mlp, &D)) return st;
  QgemmLayerMaps maps;
  const bool tc = wbits == 8;
  if (tc) {
    if (int st = ensure_qgemm(c, D, &maps)) return st;
  }
  const size_t H = (size_t)kHidden * 4;
  QB_TRY(ensure(c.x, H));
  QB_TRY(ensure(c.a, H));
  QB_TRY(ensure(c.out, H));
  QB_TRY(cudaMemcpyAsync(c.x.p, x, H, cudaMemcpyDefault, c.stream));
  float* a_dev = (float*)c.x.p;
  if (attention) {
    const int len = past + 1;
    if (int st = ensure_decode_rope(c, len)) return st;
    const size_t kvb = (size_t)len * kKvWidth * 4;
    QB_TRY(ensure(c.kc, kvb));
    QB_TRY(ensure(c.vc, kvb));
    QB_TRY(ensure(c.q, H));
    QB_TRY(ensure(c.ctx, H));
    QB_TRY(ensure(c.attn_part, attn_partial_floats(1, len) * 4));
    if (!c.counters_zeroed || c.counters_bytes < 64) {
      QB_TRY(ensure(c.counters, 64));
      QB_TRY(cudaMemsetAsync(c.counters.p, 0, 64, c.stream));
      c.counters_zeroed = true;
      c.counters_bytes = 64;
    }
    QB_TRY(ensure(c.dpos, 8));
    QB_TRY(ensure(c.dseq, 8));
    const int zero = 0;
    QB_TRY(cudaMemcpyAsync(c.dpos.p, &past, 4, cudaMemcpyHostToDevice, c.stream));
    QB_TRY(cudaMemcpyAsync(c.dseq.p, &zero, 4, cudaMemcpyHostToDevice, c.stream));
    if (past > 0) {
      QB_TRY(cudaMemcpyAsync(c.kc.p, k_cache, (size_t)past * kKvWidth * 4, cudaMemcpyDefault, c.stream));
      QB_TRY(cudaMemcpyAsync(c.vc.p, v_cache, (size_t)past * kKvWidth * 4, cudaMemcpyDefault, c.stream));
    }
    DecodeTokens tok{(const int*)c.dpos.p, (const int*)c.dseq.p, 1};
    KvView kv{(float*)c.kc.p, (float*)c.vc.p, nullptr, 0, 0};
    XSource src{(const float*)c.x.p, nullptr, nullptr};
    if (tc) {
      QB_TRY(qgemm_qkv(maps, D, src, tok, (const float*)c.rope_dec_cos.p, (const float*)c.rope_dec_sin.p,
                       (float*)c.q.p, kv, c.qsc, c.stream, false));
    } else {
      QB_TRY(launch_decode_qkv(wbits, D, src, tok, (const float*)c.rope_dec_cos.p, (const float*)c.rope_dec_sin.p,
                               (float*)c.q.p, kv, c.stream, false));
    }
    QB_TRY(launch_decode_attention((const float*)c.q.p, kv, tok, len, (float*)c.ctx.p, (float*)c.attn_part.p,
                                   (unsigned*)c.counters.p, c.stream, false));
    if (tc) {
      QB_TRY(qgemm_o(maps, D, (const float*)c.ctx.p, 1, (float*)c.a.p, c.qsc, c.stream, false));
    } else {
      QB_TRY(launch_decode_o(wbits, D, (const float*)c.ctx.p, 1, (float*)c.a.p, c.stream, false));
    }
    a_dev = (float*)c.a.p;
    const size_t row = (size_t)past * kKvWidth;
    QB_TRY(cudaMemcpyAsync(k_cache + row, (float*)c.kc.p + row, kKvWidth * 4, cudaMemcpyDefault, c.stream));
    QB_TRY(cudaMemcpyAsync(v_cache + row, (float*)c.vc.p + row, kKvWidth * 4, cudaMemcpyDefault, c.stream));
    if (attn_out) QB_TRY(cudaMemcpyAsync(attn_out, c.a.p, H, cudaMemcpyDefault, c.stream));
  }
  if (mlp) {
    QB_TRY(ensure(c.h, (size_t)kInter * 4));
    if (tc) {
      QB_TRY(qgemm_gateup(maps, D, a_dev, 1, (float*)c.h.p, c.qsc, c.stream, false));
      QB_TRY(qgemm_down(maps, D, (const float*)c.h.p, a_dev, 1, (float*)c.out.p, false, c.qsc, c.stream, false));
    } else {
      QB_TRY(launch_decode_gateup(wbits, D, a_dev, 1, (float*)c.h.p, c.stream, false));
      QB_TRY(launch_decode_down(wbits, D, (const float*)c.h.p, a_dev, 1, (float*)c.out.p, false, c.stream, false));
    }
    QB_TRY(cudaMemcpyAsync(out, c.out.p, H, cudaMemcpyDefault, c.stream));
  }
  QB_TRY(cudaStreamSynchronize(c.stream));
  return 0;
}

int run_prefill(int wbits, const LayerPtrs& L, bool attention, bool mlp, const float* x, int S, float* k_cache,
                float* v_cache, float* attn_out, float* out) {
  std::lock_guard<std::mutex> lock(g_mu);
  Ctx& c = g_ctx;
  if (int st = init_ctx(c)) return st;
  LayerDev D;
  if (int st = stage_layer(c, wbits, L, attention, mlp, &D)) return st;
  const size_t SH = (size_t)S * kHidden * 4;
  QB_TRY(ensure(c.x, SH));
  QB_TRY(ensure(c.a, SH));
  QB_TRY(ensure(c.q, SH));
  QB_TRY(ensure(c.out, SH));
  QB_TRY(cudaMemcpyAsync(c.x.p, x, SH, cudaMemcpyDefault, c.stream));
  float* a_dev = (float*)c.x.p;
  // W8: projections on the int8 tensor cores, inputs as digit planes
  const bool tc = wbits == 8;
  DigitPlanes dp{}, dph{};
  if (tc) {
    QB_TRY(ensure(c.planes, tgemm_plane_bytes(S, kInter)));
    QB_TRY(ensure(c.psteps, (size_t)tgemm_pad(S) * 4));
    dp = DigitPlanes{(int8_t*)c.planes.p, (float*)c.psteps.p, S, tgemm_pad(S), kHidden};
    dph = dp;
    dph.K = kInter;
  }
  if (attention) {
    if (int st = ensure_prefill_rope(c, S)) return st;
    const size_t kvb = (size_t)S * kKvWidth * 4;
    QB_TRY(ensure(c.kc, kvb));
    QB_TRY(ensure(c.vc, kvb));
    QB_TRY(ensure(c.ctx, SH));
    if (tc) {
      QB_TRY(tgemm_prefill_rmsnorm_digitize((const float*)c.x.p, D.input_ln, dp, c.stream));
      QB_TRY(ensure(c.qkv_raw, (size_t)S * kQkvRows * 4));
      QB_TRY(tgemm_qkv(D, dp, (const float*)c.rope_pre_cos.p, (const float*)c.rope_pre_sin.p, (float*)c.q.p,
                       (float*)c.kc.p, (float*)c.vc.p, (float*)c.qkv_raw.p, c.stream));
    } else {
      // xn reuses `out` as scratch
      QB_TRY(launch_prefill_rmsnorm((const float*)c.x.p, D.input_ln, S, (float*)c.out.p, c.stream));
      QB_TRY(launch_prefill_qkv(wbits, D, (const float*)c.out.p, S, (const float*)c.rope_pre_cos.p,
                                (const float*)c.rope_pre_sin.p, (float*)c.q.p, (float*)c.kc.p, (float*)c.vc.p,
                                c.stream));
    }
    const size_t ab = prefill_attn_tc_scratch_bytes(S);
    QB_TRY(ensure(c.attn, ab));
    QB_TRY(launch_prefill_attention_tc((const float*)c.q.p, (const float*)c.kc.p, (const float*)c.vc.p, S,
                                       (float*)c.ctx.p, c.attn.p, ab, c.stream));
    if (tc) {
      QB_TRY(tgemm_digitize((const float*)c.ctx.p, dp, c.stream));
      QB_TRY(tgemm_o(D, dp, (float*)c.a.p, c.stream));
    } else {
      QB_TRY(launch_prefill_o(wbits, D, (const float*)c.ctx.p, S, (float*)c.a.p, c.stream));
    }
    a_dev = (float*)c.a.p;
    QB_TRY(cudaMemcpyAsync(k_cache, c.kc.p, kvb, cudaMemcpyDefault, c.stream));
    QB_TRY(cudaMemcpyAsync(v_cache, c.vc.p, kvb, cudaMemcpyDefault, c.stream));
    if (attn_out) QB_TRY(cudaMemcpyAsync(attn_out, c.a.p, SH, cudaMemcpyDefault, c.stream));
  }
  if (mlp) {
    QB_TRY(ensure(c.h, (size_t)S * kInter * 4));
    if (tc) {
      QB_TRY(tgemm_prefill_rmsnorm_digitize(a_dev, D.post_ln, dp, c.stream));
      QB_TRY(tgemm_gateup(D, dp, (float*)c.h.p, c.stream));
      QB_TRY(tgemm_digitize((const float*)c.h.p, dph, c.stream));
      QB_TRY(tgemm_down(D, dph, a_dev, (float*)c.out.p, false, c.stream));
    } else {
      QB_TRY(launch_prefill_rmsnorm(a_dev, D.post_ln, S, (float*)c.q.p, c.stream));
      QB_TRY(launch_prefill_gateup(wbits, D, (const float*)c.q.p, S, (float*)c.h.p, c.stream));
      QB_TRY(launch_prefill_down(wbits, D, (const float*)c.h.p, a_dev, S, (float*)c.out.p, false, c.stream));
    }
    QB_TRY(cudaMemcpyAsync(out, c.out.p, SH, cudaMemcpyDefault, c.stream));
  }
  QB_TRY(cudaStreamSynchronize(c.stream));
  return 0;
}

namespace {

// Device copies of one layer0 layer's fp32 weights (offsets in floats; biases absent when null).
struct L0Dev {
  const float *in_ln, *q_w, *q_b, *k_w, *k_b, *v_w, *v_b, *o_w, *o_b;
  const float *post_ln, *gate_w, *gate_b, *up_w, *up_b, *down_w, *down_b;
};

int stage_layer0(Ctx& c, const Layer0Ptrs& W, L0Dev* d) {
  const size_t H = kHidden, KV = kKvWidth, I = kInter;
  struct Part {
    const float* src;
    size_t n;
    const float** dst;
  } parts[] = {{W.input_ln, H, &d->in_ln},      {W.q_w, H * H, &d->q_w},       {W.q_b, H, &d->q_b},
               {W.k_w, KV * H, &d->k_w},        {W.k_b, KV, &d->k_b},          {W.v_w, KV * H, &d->v_w},
               {W.v_b, KV, &d->v_b},            {W.o_w, H * H, &d->o_w},       {W.o_b, H, &d->o_b},
               {W.post_ln, H, &d->post_ln},     {W.gate_w, I * H, &d->gate_w}, {W.gate_b, I, &d->gate_b},
               {W.up_w, I * H, &d->up_w},       {W.up_b, I, &d->up_b},         {W.down_w, H * I, &d->down_w},
               {W.down_b, H, &d->down_b}};
  size_t total = 0;
  for (const Part& p : parts) total += (p.n + 3) / 4 * 4;  // every part 16-byte aligned
  QB_TRY(ensure(c.l0w, total * 4));
  float* base = (float*)c.l0w.p;
  size_t off = 0;
  for (const Part& p : parts) {
    if (p.src) {
      QB_TRY(cudaMemcpyAsync(base + off, p.src, p.n * 4, cudaMemcpyDefault, c.stream));
      *p.dst = base + off;
    } else {
      *p.dst = nullptr;
    }
    off += (p.n + 3) / 4 * 4;
  }
  return 0;
}

// Activation buffers of n tokens (decode: n = 1 plus the assembled head-major caches of `total` rows).
struct L0Act {
  float *x, *xn, *q, *k, *v, *ctx, *o, *resid, *post, *gate, *up, *h, *down, *out, *kc, *vc;
};

int stage_act0(Ctx& c, int n, int cache_rows, L0Act* a) {
  const size_t H = (size_t)n * kHidden, KV = (size_t)n * kKvWidth, I = (size_t)n * kInter;
  const size_t C = (size_t)kKvHeads * cache_rows * kHeadDim;
  const size_t sizes[] = {H, H, H, KV, KV, H, H, H, H, I, I, I, H, H, C, C};
  float** dst[] = {&a->x, &a->xn, &a->q, &a->k, &a->v, &a->ctx, &a->o, &a->resid, &a->post, &a->gate, &a->up,
                   &a->h, &a->down, &a->out, &a->kc, &a->vc};
  size_t total = 0;
  for (size_t z : sizes) total += (z + 3) / 4 * 4;
  QB_TRY(ensure(c.l0a, total * 4));
  float* base = (float*)c.l0a.p;
  size_t off = 0;
  for (int i = 0; i < 16; ++i) {
    *dst[i] = base + off;
    off += (sizes[i] + 3) / 4 * 4;
  }
  return 0;
}

// Attention output -> residual -> post-attention norm -> SwiGLU MLP -> output, for n tokens.
int layer0_tail(Ctx& c, const L0Dev& d, const L0Act& a, int n, float eps, bool decode_form) {
  const long long H = (long long)n * kHidden, I = (long long)n * kInter;
  QB_TRY(l0::linear(a.ctx, n, kHidden, d.o_w, d.o_b, kHidden, a.o, c.stream));
  QB_TRY(l0::add(a.x, a.o, H, a.resid, c.stream));
  QB_TRY(l0::rmsnorm(a.resid, d.post_ln, n, eps, decode_form, a.post, c.stream));
  QB_TRY(l0::linear(a.post, n, kHidden, d.gate_w, d.gate_b, kInter, a.gate, c.stream));
  QB_TRY(l0::linear(a.post, n, kHidden, d.up_w, d.up_b, kInter, a.up, c.stream));
  QB_TRY(l0::silu_mul(a.gate, a.up, I, a.h, c.stream));
  QB_TRY(l0::linear(a.h, n, kInter, d.down_w, d.down_b, kHidden, a.down, c.stream));
  QB_TRY(l0::add(a.resid, a.down, H, a.out, c.stream));
  return 0;
}

}  // namespace

int run_layer0_decode(const Layer0Ptrs& W, const float* x, int past, const float* past_k, const float* past_v,
                      float eps, float* out, float* next_k, float* next_v) {
  std::lock_guard<std::mutex> lock(g_mu);
  Ctx& c = g_ctx;
  if (int st = init_ctx(c)) return st;
  const int total = past + 1;
  if (int st = ensure_decode_rope(c, total)) return st;
  L0Dev d;
  L0Act a;
  if (int st = stage_layer0(c, W, &d)) return st;
  if (int st = stage_act0(c, 1, total, &a)) return st;
  QB_TRY(cudaMemcpyAsync(a.x, x, (size_t)kHidden * 4, cudaMemcpyDefault, c.stream));
  QB_TRY(l0::rmsnorm(a.x, d.in_ln, 1, eps, true, a.xn, c.stream));
  QB_TRY(l0::linear(a.xn, 1, kHidden, d.q_w, d.q_b, kHidden, a.q, c.stream));
  QB_TRY(l0::linear(a.xn, 1, kHidden, d.k_w, d.k_b, kKvWidth, a.k, c.stream));
  QB_TRY(l0::linear(a.xn, 1, kHidden, d.v_w, d.v_b, kKvWidth, a.v, c.stream));
  QB_TRY(l0::rope(a.q, a.k, 1, past, (const float*)c.rope_dec_cos.p, (const float*)c.rope_dec_sin.p, false, c.stream));
  // next caches [2][total][128]: the caller's history rows, then this token's K (post-RoPE) and V
  const size_t row = (size_t)kHeadDim * 4;
  for (int h = 0; h < kKvHeads; ++h) {
    if (past > 0) {
      QB_TRY(cudaMemcpyAsync(a.kc + (size_t)h * total * kHeadDim, past_k + (size_t)h * past * kHeadDim, past * row,
                             cudaMemcpyDefault, c.stream));
      QB_TRY(cudaMemcpyAsync(a.vc + (size_t)h * total * kHeadDim, past_v + (size_t)h * past * kHeadDim, past * row,
                             cudaMemcpyDefault, c.stream));
    }
    QB_TRY(cudaMemcpyAsync(a.kc + ((size_t)h * total + past) * kHeadDim, a.k + (size_t)h * kHeadDim, row,
                           cudaMemcpyDeviceToDevice, c.stream));
    QB_TRY(cudaMemcpyAsync(a.vc + ((size_t)h * total + past) * kHeadDim, a.v + (size_t)h * kHeadDim, row,
                           cudaMemcpyDeviceToDevice, c.stream));
  }
  QB_TRY(l0::attention(a.q, 1, past, a.kc, a.vc, (long long)total * kHeadDim, kHeadDim, a.ctx, c.stream));
  if (int st = layer0_tail(c, d, a, 1, eps, true)) return st;
  QB_TRY(cudaMemcpyAsync(out, a.out, (size_t)kHidden * 4, cudaMemcpyDefault, c.stream));
  QB_TRY(cudaMemcpyAsync(next_k, a.kc, (size_t)kKvHeads * total * row, cudaMemcpyDefault, c.stream));
  QB_TRY(cudaMemcpyAsync(next_v, a.vc, (size_t)kKvHeads * total * row, cudaMemcpyDefault, c.stream));
  QB_TRY(cudaStreamSynchronize(c.stream));
  return 0;
}

int run_layer0_prefill(const Layer0Ptrs& W, const float* x, int S, float eps, float* out, float* k_cache,
                       float* v_cache) {
  std::lock_guard<std::mutex> lock(g_mu);
  Ctx& c = g_ctx;
  if (int st = init_ctx(c)) return st;
  if (int st = ensure_decode_rope(c, S)) return st;  // same float(cos(double angle)) table, bf16-rounded in use
  L0Dev d;
  L0Act a;
  if (int st = stage_layer0(c, W, &d)) return st;
  if (int st = stage_act0(c, S, S, &a)) return st;
  QB_TRY(cudaMemcpyAsync(a.x, x, (size_t)S * kHidden * 4, cudaMemcpyDefault, c.stream));
  QB_TRY(l0::rmsnorm(a.x, d.in_ln, S, eps, false, a.xn, c.stream));
  QB_TRY(l0::linear(a.xn, S, kHidden, d.q_w, d.q_b, kHidden, a.q, c.stream));
  QB_TRY(l0::linear(a.xn, S, kHidden, d.k_w, d.k_b, kKvWidth, a.k, c.stream));
  QB_TRY(l0::linear(a.xn, S, kHidden, d.v_w, d.v_b, kKvWidth, a.v, c.stream));
  QB_TRY(l0::rope(a.q, a.k, S, 0, (const float*)c.rope_dec_cos.p, (const float*)c.rope_dec_sin.p, true, c.stream));
  if (k_cache != nullptr) {
    QB_TRY(l0::to_head_major(a.k, S, true, a.kc, c.stream));
    QB_TRY(l0::to_head_major(a.v, S, true, a.vc, c.stream));
  }
  // attention reads the token-major rows [S][256] (unrounded, as the reference's k_proj_out / v_proj_out)
  QB_TRY(l0::attention(a.q, S, 0, a.k, a.v, kHeadDim, kKvWidth, a.ctx, c.stream));
  if (int st = layer0_tail(c, d, a, S, eps, false)) return st;
  QB_TRY(cudaMemcpyAsync(out, a.out, (size_t)S * kHidden * 4, cudaMemcpyDefault, c.stream));
  if (k_cache != nullptr) {
    const size_t bytes = (size_t)kKvHeads * S * kHeadDim * 4;
    QB_TRY(cudaMemcpyAsync(k_cache, a.kc, bytes, cudaMemcpyDefault, c.stream));
    QB_TRY(cudaMemcpyAsync(v_cache, a.vc, bytes, cudaMemcpyDefault, c.stream));
  }
  QB_TRY(cudaStreamSynchronize(c.stream));
  return 0;
}

const LayerPtrs& zero_layer_device() {
  std::lock_guard<std::mutex> lock(g_mu);
  Ctx& c = g_ctx;
  if (!c.zero_ready && init_ctx(c) == 0) {
    // one int4-sized image is enough for either width: codes are all zero
    const LayerLayout l = layer_layout(8);
    if (ensure(c.zw, l.total) == cudaSuccess && ensure(c.zs, l.total) == cudaSuccess) {
      cudaMemset(c.zw.p, 0, l.total);
      std::vector<float> ones(kInter, 1.0f);
      float* s = (float*)c.zs.p;
      cudaMemset(s, 0, l.total);
      // scales and norm weights 1, biases 0 (qwen_decode_host_wrapper.cpp:23-34)
      const uint64_t ones_at[] = {l.input_ln, l.post_ln, l.q_s, l.k_s, l.v_s, l.o_s, l.gate_s, l.up_s, l.down_s};
      const uint64_t ones_n[] = {kHidden, kHidden, kHidden, kKvWidth, kKvWidth, kHidden, kInter, kInter, kHidden};
      for (int i = 0; i < 9; ++i) cudaMemcpy(s + ones_at[i] / 4, ones.data(), ones_n[i] * 4, cudaMemcpyHostToDevice);
      c.zero = layer_ptrs_from_ddr((const uint8_t*)c.zw.p, 0, s, 0, 8);
      // weight pointers of the 4-bit view start at the same zero bytes
      c.zero_ready = cudaDeviceSynchronize() == cudaSuccess;
    }
  }
  return c.zero;
}

}  // namespace qb

extern "C" {

const char* qwen_b200_last_error(void) { return qb::g_error.c_str(); }

int qwen_b200_prefill_seq_capacity(void) { return qb::prefill_seq_capacity(); }

int qwen_b200_set_prefill_seq_capacity(int capacity) {
  if (capacity <= 0 || capacity > qb::kMaxSeq) return qb::kStatusInvalid;
  qb::prefill_seq_capacity();
  qb::g_prefill_capacity = capacity;
  return 0;
}

unsigned qwen_b200_kernel_error(int reset) {
  return qb::gemv_kernel_error(reset != 0) | qb::qgemm_kernel_error(reset != 0) |
         qb::stack::decode_stack_kernel_error(reset != 0) | qb::bs1::decode_bs1_kernel_error(reset != 0) |
         qb::tgemm_kernel_error(reset != 0) |
         qb::lm_head_kernel_error(reset != 0) | qb::attn_tc_kernel_error(reset != 0) |
         qb::decode_attn_kernel_error(reset != 0);
}

int qwen_b200_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
  return n;
}

}  // extern "C"
