// Device-resident Qwen2.5-1.5B engine: weights, paged KV cache and activations stay in HBM; a decode step
// is one CUDA-graph launch of 5 kernels per layer plus the LM head (programmatic dependent launch lets
// each kernel's CTAs be scheduled while the previous one drains).
//
// Per-layer flow matches the reference's top wrappers (hls/decode_only/qwen_decode_top_wrapper.cpp:79-112,
// hls/prefill_only/qwen_prefill_top_core.cpp:158-182) followed by the caller's bf16 rounding
// (verification/real_host_top_backend.py:260, 334); the final norm / LM head / argmax stand in for the
// caller's Hugging Face modules (:138-146) as defined in oracle/qwen_oracle.c (`oracle_lm_head_argmax`).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <dlfcn.h>
#include <nccl.h>  // types and the unique-id layout; the library itself is opened at run time

#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/qwen_b200_engine.h"
#include "attention_tc.h"
#include "decode_bs1.h"
#include "decode_stack.h"
#include "qgemm.h"
#include "lmhead.h"
#include "tgemm.h"
#include "qwen_kernels.cuh"
#include "runtime.h"

#include "exact.h"

namespace qb {
namespace {

__global__ void embed_gather_kernel(const uint16_t* __restrict__ embed, const int* __restrict__ tokens, int n,
                                    float* __restrict__ x) {
  const int t = blockIdx.x;
  if (t >= n) return;
  const __half* row = reinterpret_cast<const __half*>(embed) + (size_t)tokens[t] * kHidden;
  for (int d = threadIdx.x; d < kHidden; d += blockDim.x) x[(size_t)t * kHidden + d] = __half2float(row[d]);
}

// flat [n][256] K and V of one layer <-> paged rows pos0 .. pos0 + n - 1 of one slot
__global__ void kv_scatter_kernel(const float* __restrict__ kf, const float* __restrict__ vf, int n, KvView kv,
                                  int slot, int to_pages, int pos0) {
  griddep_wait();  // inputs come from the preceding kernel (programmatic dependent launch)
  griddep_launch();
  const int t = blockIdx.x;
  if (t >= n) return;
  float* kd = kv_row(kv, slot, pos0 + t, 0);
  float* vd = kv_row(kv, slot, pos0 + t, 1);
  for (int d = threadIdx.x; d < kKvWidth; d += blockDim.x) {
    if (to_pages) {
      kd[d] = kf[(size_t)t * kKvWidth + d];
      vd[d] = vf[(size_t)t * kKvWidth + d];
    } else {
      const_cast<float*>(kf)[(size_t)t * kKvWidth + d] = kd[d];
      const_cast<float*>(vf)[(size_t)t * kKvWidth + d] = vd[d];
    }
  }
}

// Paged rows of one layer of a slot <-> the Hugging Face cache layout [kv_head][token][128] (head-major), the
// layout the reference caller converts to and from (verification/real_host_top_backend.py:199-206).
__global__ void kv_hf_kernel(KvView kv, int slot, int n, float* __restrict__ kh, float* __restrict__ vh, int to_pages) {
  const int t = blockIdx.x;
  if (t >= n) return;
  float* kr = kv_row(kv, slot, t, 0);
  float* vr = kv_row(kv, slot, t, 1);
  for (int i = threadIdx.x; i < kKvWidth; i += blockDim.x) {
    const size_t o = ((size_t)(i >> 7) * n + t) * kHeadDim + (i & 127);
    if (to_pages) {
      kr[i] = kh[o];
      vr[i] = vh[o];
    } else {
      kh[o] = kr[i];
      vh[o] = vr[i];
    }
  }
}

__global__ void advance_pos_kernel(int* __restrict__ pos, int n) {
  griddep_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) pos[i] += 1;
}

// end of a device-resident decode step: next input token = argmax, position + 1
__global__ void advance_kernel(int* __restrict__ tokens, const int* __restrict__ next, int* __restrict__ pos, int n) {
  griddep_wait();
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t < n) {
    tokens[t] = next[t];
    pos[t] += 1;
  }
}

#define E_TRY(expr)                                                                                 \
  do {                                                                                              \
    cudaError_t _e = (expr);                                                                        \
    if (_e != cudaSuccess) {                                                                        \
      set_error("%s failed: %s (%s:%d)", #expr, cudaGetErrorString(_e), __FILE__, __LINE__);        \
      return kStatusCuda;                                                                           \
    }                                                                                               \
  } while (0)

// NCCL entry points, resolved from libnccl.so.2 on first use: the process's already-loaded copy when one is
// (e.g. PyTorch's), otherwise the system library. The core library keeps no link-time dependency on NCCL.
struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  std::string load_error;
};

const NcclApi* nccl_api() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      const char* why = dlerror();
      api.load_error = why ? why : "dlopen(libnccl.so.2) failed";
      return;
    }
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
    if (!api.get_unique_id || !api.comm_init_rank || !api.all_gather || !api.comm_destroy || !api.error_string)
      api.load_error = "libnccl.so.2 lacks an NCCL entry point";
  });
  return api.load_error.empty() ? &api : nullptr;
}

#define N_TRY(api, expr)                                                                              \
  do {                                                                                              \
    ncclResult_t _r = (expr);                                                                       \
    if (_r != ncclSuccess) {                                                                        \
      set_error("%s failed: %s", #expr, (api)->error_string(_r));                                   \
      return kStatusCuda;                                                                           \
    }                                                                                               \
  } while (0)

template <typename T>
cudaError_t dalloc(T** p, size_t count) {
  return cudaMalloc(reinterpret_cast<void**>(p), count * sizeof(T));
}

}  // namespace
}  // namespace qb

using namespace qb;

struct qwen_engine {
  int device = 0, wbits = 8, max_seqs = 1, max_len = 1, max_pages = 1;
  cudaStream_t stream = nullptr;
  // parameters
  uint8_t* wimg = nullptr;
  float* simg = nullptr;
  uint64_t layer_bytes = 0;
  LayerDev layers[kLayers];
  uint16_t* embed = nullptr;
  float* final_norm = nullptr;
  // KV pages
  float* kv_pool = nullptr;
  int n_pages = 0;
  int* d_page_table = nullptr;
  std::vector<int> page_table;   // [max_seqs][max_pages], -1 = unassigned
  std::vector<int> free_pages;
  std::vector<int> seq_len;
  // decode state (up to kGemvMaxTokens tokens per group)
  int *d_tokens = nullptr, *d_pos = nullptr, *d_seq = nullptr, *d_next = nullptr;
  int* h_io = nullptr;  // pinned: [4 tokens][4 pos][4 seq][4 next]
  int* hb_io = nullptr;  // pinned, batched path: [tokens][pos][seq][next], batch_cap each
  int batch_cap = 4;
  bool use_batched = true;
  float *x = nullptr, *q = nullptr, *ctx = nullptr, *a = nullptr, *h = nullptr, *y0 = nullptr, *y1 = nullptr;
  float* attn_part = nullptr;
  unsigned* attn_cnt = nullptr;
  float* lm_part = nullptr;
  unsigned* lm_cnt = nullptr;
  float* dump = nullptr;
  float* logits = nullptr;
  int last_rows = 0;
  // rope tables
  float *rope_dec_cos = nullptr, *rope_dec_sin = nullptr, *rope_pre_cos = nullptr, *rope_pre_sin = nullptr;
  int rope_dec_len = 0, rope_pre_len = 0;
  // prefill buffers
  int pre_cap = 0;
  float *p_x = nullptr, *p_xn = nullptr, *p_q = nullptr, *p_ctx = nullptr, *p_a = nullptr, *p_h = nullptr,
        *p_k = nullptr, *p_v = nullptr;
  float* p_qkv = nullptr;  // W8: biased q|k|v rows before RoPE [cap][2048]
  int* p_tokens = nullptr;
  int8_t* p_planes = nullptr;  // W8 prefill: digit planes [3][Spad][8960] and steps [Spad]
  float* p_steps = nullptr;
  void* p_attn = nullptr;      // tensor-core prefill attention scratch (fp16 operand planes)
  size_t p_attn_bytes = 0;
  bool use_attn_tc = true;
  int attn_ctas = 0;  // option "attn_ctas": cap on the decode attention grid (0 = one CTA per SM)
  // options
  bool use_graphs = true, use_pdl = true, dump_hidden = false, keep_logits = false, prefetch = true;
  std::map<long long, cudaGraphExec_t> graphs;
  std::vector<int> dev_slots;  // slots whose positions are current in d_pos / d_seq (decode_device path)
  // int8 tensor-core projections (wbits == 8)
  bool use_qgemm = true;
  QgemmLayerMaps maps[kLayers];
  QgemmScratch qsc{nullptr, nullptr};
  // persistent whole-step kernel (wbits == 8): tiled weights, schedule, synchronisation words
  bool use_stack = true;
  bool tiles_dirty = true;
  uint8_t* wtiles = nullptr;
  LayerDev* d_layers = nullptr;
  stack::SyncWords* sync = nullptr;
  int* stack_acc = nullptr;
  float* stack_steps = nullptr;
  uint32_t* d_item_off = nullptr;
  stack::Item* d_items = nullptr;
  int stack_ctas = 0;
  int attn_max_chunks = 0;
  unsigned long long* trace = nullptr;  // optional timeline of the persistent kernel
  int stack_ring = 9;                   // weight stages in flight per CTA
  // persistent batch-1 step on the CUDA cores (wbits == 8, one sequence per step): its schedule and words
  bool use_bs1 = true;
  int bs1_ctas = 0;  // CTAs of the batch-1 kernel (option "bs1_ctas"; default: bs1::kMinCtas)
  bool bs1_poison = false;  // test hook (option "bs1_poison"): the next batch-1 launch finds impossible counts
  bs1::Sync* bs1_sync = nullptr;
  bs1::Buffers bs1_buf{nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr};
  uint32_t* d_item_off1 = nullptr;
  stack::Item* d_items1 = nullptr;
  cudaEvent_t kev[3] = {nullptr, nullptr, nullptr};  // per-kernel timing (profile_decode)
  bool time_kernels = false;
  // per-category timing of the batched step (profile_batched): events around each kernel group
  std::vector<cudaEvent_t> bev;
  std::vector<int> bev_cat;  // category of the group each event opens
  int bev_used = 0;
  bool time_batched = false;
  // tensor-core LM head
  bool use_lm_tc = true;
  LmScratch lm{nullptr, nullptr, nullptr};
  // token exchange of a multi-GPU run (qwen_engine_nccl_init)
  ncclComm_t nccl = nullptr;
  int nccl_ranks = 0, nccl_rank = 0;
  // asynchronous token gathers (qwen_engine_gather_tokens_async): a side stream and the completion events of
  // the last two gathers
  cudaStream_t gather_stream = nullptr;
  cudaEvent_t gather_ready = nullptr, gather_done[2] = {nullptr, nullptr};
  long long gather_n = 0;
  // option "exact": every layer and the LM head in the reference's arithmetic order (exact.h)
  bool exact = false;
  int ex_cap = 0;                                              // token rows of the buffers below
  float *ex_xn = nullptr, *ex_qkv = nullptr, *ex_gu = nullptr;  // [cap][1536], [cap][2048], [cap][17920]
};

namespace {

int ensure_rope_dec(qwen_engine* e, int need) {
  if (need <= e->rope_dec_len) return 0;
  int len = std::max(1024, e->rope_dec_len);
  while (len < need) len *= 2;
  std::vector<float> c((size_t)len * 64), s((size_t)len * 64);
  for (int pos = 0; pos < len; ++pos)
    for (int pair = 0; pair < 64; ++pair) {
      const double angle = (double)pos * std::pow((double)kRopeTheta, -2.0 * (double)pair / (double)kHeadDim);
      c[(size_t)pos * 64 + pair] = (float)std::cos(angle);
      s[(size_t)pos * 64 + pair] = (float)std::sin(angle);
    }
  cudaFree(e->rope_dec_cos);
  cudaFree(e->rope_dec_sin);
  E_TRY(dalloc(&e->rope_dec_cos, (size_t)len * 64));
  E_TRY(dalloc(&e->rope_dec_sin, (size_t)len * 64));
  E_TRY(cudaMemcpy(e->rope_dec_cos, c.data(), c.size() * 4, cudaMemcpyHostToDevice));
  E_TRY(cudaMemcpy(e->rope_dec_sin, s.data(), s.size() * 4, cudaMemcpyHostToDevice));
  e->rope_dec_len = len;
  return 0;
}

int ensure_rope_pre(qwen_engine* e, int need) {
  if (need <= e->rope_pre_len) return 0;
  int len = std::max(128, e->rope_pre_len);
  while (len < need) len *= 2;
  cudaFree(e->rope_pre_cos);
  cudaFree(e->rope_pre_sin);
  E_TRY(dalloc(&e->rope_pre_cos, (size_t)len * 64));
  E_TRY(dalloc(&e->rope_pre_sin, (size_t)len * 64));
  E_TRY(launch_prefill_rope_table(len, e->rope_pre_cos, e->rope_pre_sin, e->stream));
  e->rope_pre_len = len;
  return 0;
}

KvView paged_view(qwen_engine* e, int layer) {
  KvView kv;
  kv.k = e->kv_pool;
  kv.v = nullptr;
  kv.page_table = e->d_page_table;
  kv.layer = layer;
  kv.max_pages = e->max_pages;
  kv.pool_pages = e->n_pages;
  return kv;
}

// make sure slot has pages for positions [0, len)
int ensure_pages(qwen_engine* e, int slot, int len) {
  const int need = (len + kPage - 1) / kPage;
  if (need > e->max_pages) {
    set_error("sequence length %d exceeds the engine's max_len %d", len, e->max_len);
    return kStatusInvalid;
  }
  bool changed = false;
  for (int p = 0; p < need; ++p) {
    int& entry = e->page_table[(size_t)slot * e->max_pages + p];
    if (entry < 0) {
      if (e->free_pages.empty()) {
        set_error("KV page pool exhausted");
        return kStatusInvalid;
      }
      entry = e->free_pages.back();
      e->free_pages.pop_back();
      changed = true;
    }
  }
  if (changed) {
    E_TRY(cudaMemcpyAsync(e->d_page_table + (size_t)slot * e->max_pages,
                          e->page_table.data() + (size_t)slot * e->max_pages, (size_t)e->max_pages * 4,
                          cudaMemcpyHostToDevice, e->stream));
  }
  return 0;
}

int ensure_prefill_buffers(qwen_engine* e, int n) {
  if (n <= e->pre_cap) return 0;
  int cap = std::max(128, e->pre_cap);
  while (cap < n) cap *= 2;
  float** bufs[] = {&e->p_x, &e->p_xn, &e->p_q, &e->p_ctx, &e->p_a};
  for (float** b : bufs) {
    cudaFree(*b);
    E_TRY(dalloc(b, (size_t)cap * kHidden));
  }
  cudaFree(e->p_h);
  E_TRY(dalloc(&e->p_h, (size_t)cap * kInter));
  cudaFree(e->p_k);
  cudaFree(e->p_v);
  E_TRY(dalloc(&e->p_k, (size_t)cap * kKvWidth));
  E_TRY(dalloc(&e->p_v, (size_t)cap * kKvWidth));
  cudaFree(e->p_tokens);
  E_TRY(dalloc(&e->p_tokens, (size_t)cap));
  cudaFree(e->p_attn);
  e->p_attn = nullptr;
  e->p_attn_bytes = prefill_attn_tc_scratch_bytes(cap);
  E_TRY(cudaMalloc(&e->p_attn, e->p_attn_bytes));
  if (e->wbits == 8) {
    cudaFree(e->p_qkv);
    E_TRY(dalloc(&e->p_qkv, (size_t)cap * kQkvRows));
    cudaFree(e->p_planes);
    cudaFree(e->p_steps);
    E_TRY(dalloc(&e->p_planes, tgemm_plane_bytes(cap, kInter)));
    E_TRY(dalloc(&e->p_steps, (size_t)tgemm_pad(cap)));
  }
  e->pre_cap = cap;
  return 0;
}

// Rebuild the tiled copy of the int8 weights after they changed (outside any stream capture).
int ensure_tiles(qwen_engine* e) {
  if (e->wbits != 8 || !e->tiles_dirty) return 0;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  E_TRY(cudaStreamIsCapturing(e->stream, &cap));
  if (cap != cudaStreamCaptureStatusNone) {
    set_error("weights changed during stream capture");
    return kStatusCuda;
  }
  for (int l = 0; l < kLayers; ++l)
    E_TRY(stack::launch_tile_layer(e->layers[l], e->wtiles + (size_t)l * stack::kLayerTileBytes, e->stream));
  e->tiles_dirty = false;
  return 0;
}

// Buffers of the reference-order path for up to n token rows (allocated on first use, outside capture).
int ensure_exact(qwen_engine* e, int n) {
  n = std::max(n, e->batch_cap);
  if (n <= e->ex_cap) return 0;
  int cap = std::max(128, e->ex_cap);
  while (cap < n) cap *= 2;
  cudaFree(e->ex_xn);
  cudaFree(e->ex_qkv);
  cudaFree(e->ex_gu);
  e->ex_xn = e->ex_qkv = e->ex_gu = nullptr;
  E_TRY(dalloc(&e->ex_xn, (size_t)cap * kHidden));
  E_TRY(dalloc(&e->ex_qkv, (size_t)cap * kQkvRows));
  E_TRY(dalloc(&e->ex_gu, (size_t)cap * 2 * kInter));
  e->ex_cap = cap;
  return 0;
}

// One decode step in the reference's arithmetic (qwen_decode_attention_kernel.cpp:168-218,
// qwen_decode_mlp_kernel.cpp:87-122, the caller's bf16 rounding between layers and its final norm + LM head):
// bit-identical to the reference host library's decode layers, token for token.
int enqueue_decode_exact(qwen_engine* e, int nt, bool advance) {
  cudaStream_t s = e->stream;
  const int wb = e->wbits;
  const float scaling = (float)(1.0 / std::sqrt((double)kHeadDim));  // qwen_decode_attention_kernel.cpp:118
  embed_gather_kernel<<<nt, 256, 0, s>>>(e->embed, e->d_tokens, nt, e->x);
  E_TRY(cudaGetLastError());
  const float* xin = e->x;
  for (int l = 0; l < kLayers; ++l) {
    const LayerDev& L = e->layers[l];
    const KvView kv = paged_view(e, l);
    float* yout = (l & 1) ? e->y1 : e->y0;
    E_TRY(exact::launch_rmsnorm_dec(xin, L.input_ln, nt, e->ex_xn, s));
    E_TRY(exact::launch_project(wb, e->ex_xn, nt, kHidden, L.qkv_w, L.qkv_b, L.qkv_s, kQkvRows, e->ex_qkv, nullptr,
                                false, s));
    E_TRY(exact::launch_rope_store(e->ex_qkv, nt, e->d_pos, 0, e->rope_dec_cos, e->rope_dec_sin, e->q, kv, e->d_seq,
                                   0, s));
    E_TRY(exact::launch_attention_dec(e->q, kv, e->d_pos, e->d_seq, nt, scaling, e->ctx, s));
    E_TRY(exact::launch_project(wb, e->ctx, nt, kHidden, L.o_w, nullptr, L.o_s, kHidden, e->a, nullptr, false, s));
    E_TRY(exact::launch_rmsnorm_dec(e->a, L.post_ln, nt, e->ex_xn, s));
    E_TRY(exact::launch_project(wb, e->ex_xn, nt, kHidden, L.gu_w, nullptr, L.gu_s, 2 * kInter, e->ex_gu, nullptr,
                                false, s));
    E_TRY(exact::launch_silu_mul(e->ex_gu, nt, false, e->h, s));
    E_TRY(exact::launch_project(wb, e->h, nt, kInter, L.down_w, nullptr, L.down_s, kHidden, yout, e->a, true, s));
    if (e->dump_hidden) {
      E_TRY(cudaMemcpyAsync(e->dump + (size_t)l * nt * kHidden, yout, (size_t)nt * kHidden * 4,
                            cudaMemcpyDeviceToDevice, s));
    }
    xin = yout;
  }
  E_TRY(exact::launch_lm_head(e->embed, e->final_norm, xin, nt, e->ex_xn, e->logits, e->d_next, s));
  if (advance) {
    E_TRY(launch_k(advance_kernel, dim3(1), dim3(32), 0, s, false, e->d_tokens, (const int*)e->d_next, e->d_pos, nt));
  }
  return 0;
}

// A prefill chunk after `past` cached tokens: the slot's K/V rows [0, past) of layer l into the flat rows
// [0, past) that the chunk's attention reads (its own rows follow at [past, past + n)).
int gather_history(qwen_engine* e, int slot, int l, int past, bool pdl) {
  if (past <= 0) return 0;
  E_TRY(launch_k(kv_scatter_kernel, dim3(past), dim3(256), 0, e->stream, pdl, static_cast<const float*>(e->p_k),
                 static_cast<const float*>(e->p_v), past, paged_view(e, l), slot, 0, 0));
  return 0;
}

// Prefill in the reference's arithmetic (qwen_prefill_attention_kernel.cpp:2232-2367,
// qwen_prefill_mlp_kernel.cpp:264-337): K/V of every token first, then each query's causal context. With
// past > 0 the n tokens continue a slot that holds `past` tokens (positions past .. past + n - 1).
int enqueue_prefill_exact(qwen_engine* e, int slot, int n, int past) {
  cudaStream_t s = e->stream;
  const int wb = e->wbits;
  embed_gather_kernel<<<n, 256, 0, s>>>(e->embed, e->p_tokens, n, e->p_x);
  E_TRY(cudaGetLastError());
  KvView flat{};
  flat.k = e->p_k;
  flat.v = e->p_v;
  flat.page_table = nullptr;
  for (int l = 0; l < kLayers; ++l) {
    const LayerDev& L = e->layers[l];
    E_TRY(launch_prefill_rmsnorm(e->p_x, L.input_ln, n, e->p_xn, s));
    E_TRY(exact::launch_project(wb, e->p_xn, n, kHidden, L.qkv_w, L.qkv_b, L.qkv_s, kQkvRows, e->ex_qkv, nullptr,
                                false, s));
    if (int st = gather_history(e, slot, l, past, false)) return st;
    E_TRY(exact::launch_rope_store(e->ex_qkv, n, nullptr, past, e->rope_pre_cos, e->rope_pre_sin, e->p_q, flat,
                                   nullptr, 0, s));
    E_TRY(exact::launch_attention_pre(e->p_q, e->p_k, e->p_v, n, e->p_ctx, s, past));
    E_TRY(exact::launch_project(wb, e->p_ctx, n, kHidden, L.o_w, nullptr, L.o_s, kHidden, e->p_a, nullptr, false, s));
    E_TRY(launch_k(kv_scatter_kernel, dim3(n), dim3(256), 0, s, false,
                   static_cast<const float*>(e->p_k + (size_t)past * kKvWidth),
                   static_cast<const float*>(e->p_v + (size_t)past * kKvWidth), n, paged_view(e, l), slot, 1, past));
    E_TRY(launch_prefill_rmsnorm(e->p_a, L.post_ln, n, e->p_xn, s));
    E_TRY(exact::launch_project(wb, e->p_xn, n, kHidden, L.gu_w, nullptr, L.gu_s, 2 * kInter, e->ex_gu, nullptr,
                                false, s));
    E_TRY(exact::launch_silu_mul(e->ex_gu, n, true, e->p_h, s));
    E_TRY(exact::launch_project(wb, e->p_h, n, kInter, L.down_w, nullptr, L.down_s, kHidden, e->p_x, e->p_a, true, s));
    if (e->dump_hidden) {
      E_TRY(cudaMemcpyAsync(e->dump + (size_t)l * kHidden, e->p_x + (size_t)(n - 1) * kHidden, kHidden * 4,
                            cudaMemcpyDeviceToDevice, s));
    }
  }
  E_TRY(exact::launch_lm_head(e->embed, e->final_norm, e->p_x + (size_t)(n - 1) * kHidden, 1, e->ex_xn, e->logits,
                              e->d_next, s));
  return 0;
}

bool stack_enabled(const qwen_engine* e) { return e->wbits == 8 && e->use_stack && e->wtiles != nullptr; }
bool bs1_enabled(const qwen_engine* e, int nt) { return nt == 1 && e->use_bs1 && e->d_items1 != nullptr; }

// Final norm + LM head + argmax of n rows of x into d_next (logits kept when requested).
int enqueue_lm_head(qwen_engine* e, const float* x, int n, int* next, float* logits, bool pdl) {
  if (e->use_lm_tc && e->lm.planes != nullptr) {
    E_TRY(lm_head_tc(e->embed, e->final_norm, x, n, logits, next, e->lm, e->stream));
    return 0;
  }
  for (int g = 0; g < n; g += kGemvMaxTokens) {
    const int m = std::min(kGemvMaxTokens, n - g);
    E_TRY(launch_lm_head_argmax(e->embed, e->final_norm, x + (size_t)g * kHidden, m,
                                logits ? logits + (size_t)g * kVocab : nullptr, e->lm_part, e->lm_cnt, next + g,
                                e->stream, pdl && g == 0));
  }
  return 0;
}

// Enqueue one decode step for nt tokens whose ids/positions/slots are already in d_tokens/d_pos/d_seq.
// max_len bounds the attention grid (positions + 1 of every token must be <= max_len).
int enqueue_decode(qwen_engine* e, int nt, int max_len, bool advance) {
  if (e->exact) return enqueue_decode_exact(e, nt, advance);
  const bool pdl = e->use_pdl;
  DecodeTokens tok{e->d_pos, e->d_seq, nt};
  float* xin = nullptr;
  const uint64_t wb = (uint64_t)e->wbits;
  const size_t o_bytes = (size_t)kHidden * kHidden * wb / 8;
  const size_t gu_bytes = (size_t)2 * kInter * kHidden * wb / 8;
  const size_t down_bytes = (size_t)kInter * kHidden * wb / 8;
  const size_t qkv_bytes = (size_t)kQkvRows * kHidden * wb / 8;
  const size_t lm_head_prefetch = (size_t)32 << 20;
  if (e->time_kernels) E_TRY(cudaEventRecord(e->kev[0], e->stream));
  if (stack_enabled(e) && bs1_enabled(e, nt)) {
    if (int st = ensure_tiles(e)) return st;
    bs1::Args a{};
    a.wtiles = e->wtiles;
    a.layers = e->d_layers;
    a.embed = e->embed;
    a.tokens = e->d_tokens;
    a.pos = e->d_pos;
    a.seq = e->d_seq;
    a.rope_cos = e->rope_dec_cos;
    a.rope_sin = e->rope_dec_sin;
    a.kv_pool = e->kv_pool;
    a.page_table = e->d_page_table;
    a.max_pages = e->max_pages;
    a.y0 = e->y0;
    a.y1 = e->y1;
    a.dump = e->dump_hidden ? e->dump : nullptr;
    a.buf = e->bs1_buf;
    a.max_chunks = e->attn_max_chunks;
    a.sync = e->bs1_sync;
    a.item_off = e->d_item_off1;
    a.items = e->d_items1;
    a.trace = e->trace;
    a.ring = e->stack_ring;
    if (e->bs1_poison) {
      // both launch halves of the packed split-K words get counts no producer can complete (bytes 0x40: count
      // field 0x4040, value field far below a carry into it): the launch's consumers wait out their bounded
      // waits (~1 s), raise the abort flag and set the kernel error flag; the launch zeroes the other half as
      // usual, so the launch after it is clean
      E_TRY(cudaMemsetAsync(e->bs1_buf.acc, 0x40, bs1::acc_words() * 8, e->stream));
      e->bs1_poison = false;
    }
    E_TRY(bs1::launch_decode_bs1(a, e->bs1_ctas, e->stream));
    xin = ((kLayers - 1) & 1) ? e->y1 : e->y0;
  } else if (stack_enabled(e)) {
    if (int st = ensure_tiles(e)) return st;
    stack::Args a{};
    a.wtiles = e->wtiles;
    a.layers = e->d_layers;
    a.embed = e->embed;
    a.tokens = e->d_tokens;
    a.pos = e->d_pos;
    a.seq = e->d_seq;
    a.nt = nt;
    a.rope_cos = e->rope_dec_cos;
    a.rope_sin = e->rope_dec_sin;
    a.kv_pool = e->kv_pool;
    a.page_table = e->d_page_table;
    a.max_pages = e->max_pages;
    a.y0 = e->y0;
    a.y1 = e->y1;
    a.q = e->q;
    a.ctx = e->ctx;
    a.a = e->a;
    a.h = e->h;
    a.dump = e->dump_hidden ? e->dump : nullptr;
    a.attn_part = e->attn_part;
    a.attn_max_chunks = e->attn_max_chunks;
    a.acc = e->stack_acc;
    a.steps = e->stack_steps;
    a.sync = e->sync;
    a.item_off = e->d_item_off;
    a.items = e->d_items;
    a.trace = e->trace;
    a.ring = e->stack_ring;
    E_TRY(stack::launch_decode_stack(a, e->stack_ctas, e->stream));
    xin = ((kLayers - 1) & 1) ? e->y1 : e->y0;
  }
  for (int l = 0; l < kLayers && !stack_enabled(e); ++l) {
    const LayerDev& L = e->layers[l];
    XSource src{xin, e->embed, e->d_tokens};
    KvView kv = paged_view(e, l);
    // Each kernel streams the next kernels' weights into L2 while it runs (the weights are independent
    // of the activations), so HBM stays busy through the latency-bound kernels and launch gaps.
    const bool last = l + 1 == kLayers;
    const void* next_qkv = last ? (const void*)e->embed : (const void*)e->layers[l + 1].qkv_w;
    const size_t next_qkv_bytes = last ? lm_head_prefetch : qkv_bytes;
    float* yout = (l & 1) ? e->y1 : e->y0;
    if (e->wbits == 8 && e->use_qgemm) {
      // int8 tensor cores; each kernel's TMA producer starts streaming its weights before it waits
      const QgemmLayerMaps& M = e->maps[l];
      E_TRY(qgemm_qkv(M, L, src, tok, e->rope_dec_cos, e->rope_dec_sin, e->q, kv, e->qsc, e->stream, pdl && l > 0));
      E_TRY(launch_decode_attention(e->q, kv, tok, max_len, e->ctx, e->attn_part, e->attn_cnt, e->stream, pdl,
                                    e->prefetch ? L.gu_w : nullptr, gu_bytes, e->attn_ctas));
      E_TRY(qgemm_o(M, L, e->ctx, nt, e->a, e->qsc, e->stream, pdl));
      E_TRY(qgemm_gateup(M, L, e->a, nt, e->h, e->qsc, e->stream, pdl));
      E_TRY(qgemm_down(M, L, e->h, e->a, nt, yout, true, e->qsc, e->stream, pdl));
    } else {
      E_TRY(launch_decode_qkv(e->wbits, L, src, tok, e->rope_dec_cos, e->rope_dec_sin, e->q, kv, e->stream,
                              pdl && l > 0, e->prefetch ? L.o_w : nullptr, o_bytes));
      E_TRY(launch_decode_attention(e->q, kv, tok, max_len, e->ctx, e->attn_part, e->attn_cnt, e->stream, pdl,
                                    e->prefetch ? L.gu_w : nullptr, gu_bytes, e->attn_ctas));
      E_TRY(launch_decode_o(e->wbits, L, e->ctx, nt, e->a, e->stream, pdl, e->prefetch ? L.down_w : nullptr,
                            down_bytes));
      E_TRY(launch_decode_gateup(e->wbits, L, e->a, nt, e->h, e->stream, pdl, e->prefetch ? next_qkv : nullptr,
                                 next_qkv_bytes));
      E_TRY(launch_decode_down(e->wbits, L, e->h, e->a, nt, yout, true, e->stream, pdl));
    }
    if (e->dump_hidden) {
      E_TRY(cudaMemcpyAsync(e->dump + (size_t)l * nt * kHidden, yout, (size_t)nt * kHidden * 4,
                            cudaMemcpyDeviceToDevice, e->stream));
    }
    xin = yout;
  }
  if (e->time_kernels) E_TRY(cudaEventRecord(e->kev[1], e->stream));
  if (int st = enqueue_lm_head(e, xin, nt, e->d_next, e->keep_logits ? e->logits : nullptr,
                               pdl && !e->dump_hidden && !stack_enabled(e) && !e->time_kernels))
    return st;
  if (e->time_kernels) E_TRY(cudaEventRecord(e->kev[2], e->stream));
  if (advance) {
    E_TRY(launch_k(advance_kernel, dim3(1), dim3(32), 0, e->stream, pdl, e->d_tokens, (const int*)e->d_next,
                   e->d_pos, nt));
  }
  return 0;
}

bool batched_ok(const qwen_engine* e, int n) {
  return e->wbits == 8 && e->use_batched && !e->exact && n > kGemvMaxTokens && n <= e->batch_cap;
}

// One greedy decode step of n > 4 tokens (W8): every projection of all tokens in one many-token tensor-core
// GEMM per layer (weights read once per step), paged-KV attention over all tokens, LM head in groups of 4.
// Tokens / positions / slots are in d_tokens / d_pos / d_seq. Eager launches (no graph).
// Timing categories of the batched step (profile_batched).
enum BatchedCat { kBcNorm = 0, kBcDigits, kBcQkv, kBcAttn, kBcO, kBcGateUp, kBcDown, kBcHead, kBcCats };

int enqueue_decode_batched(qwen_engine* e, int n, int max_len, bool advance) {
  cudaStream_t s = e->stream;
  if (int st = ensure_tiles(e)) return st;
  // optional timing: an event before each kernel group, tagged with its category
  if (e->time_batched) {
    e->bev_used = 0;
    e->bev_cat.clear();
  }
  auto mark = [&](int cat) -> cudaError_t {
    if (!e->time_batched) return cudaSuccess;
    if (e->bev_used == (int)e->bev.size()) {
      cudaEvent_t ev;
      cudaError_t err = cudaEventCreate(&ev);
      if (err != cudaSuccess) return err;
      e->bev.push_back(ev);
    }
    e->bev_cat.push_back(cat);
    return cudaEventRecord(e->bev[e->bev_used++], s);
  };
  embed_gather_kernel<<<n, 256, 0, s>>>(e->embed, e->d_tokens, n, e->p_x);
  E_TRY(cudaGetLastError());
  const DigitPlanes dp{e->p_planes, e->p_steps, n, tgemm_pad(n), kHidden};
  const DigitPlanes dph{e->p_planes, e->p_steps, n, tgemm_pad(n), kInter};
  const DecodeTokens tok{e->d_pos, e->d_seq, n};
  for (int l = 0; l < kLayers; ++l) {
    const LayerDev& L = e->layers[l];
    const KvView kv = paged_view(e, l);
    E_TRY(mark(kBcDigits));
    E_TRY(tgemm_rmsnorm_digitize(e->p_x, L.input_ln, dp, s));
    E_TRY(mark(kBcQkv));
    E_TRY(tgemm_qkv_decode(L, dp, e->d_pos, e->d_seq, kv, e->rope_dec_cos, e->rope_dec_sin, e->p_q, e->p_qkv, s));
    E_TRY(mark(kBcAttn));
    E_TRY(launch_decode_attention(e->p_q, kv, tok, max_len, e->p_ctx, e->attn_part, e->attn_cnt, s, true,
                                  nullptr, 0, e->attn_ctas));
    E_TRY(mark(kBcDigits));
    E_TRY(tgemm_digitize(e->p_ctx, dp, s));
    E_TRY(mark(kBcO));
    E_TRY(tgemm_o(L, dp, e->p_a, s));
    E_TRY(mark(kBcDigits));
    E_TRY(tgemm_rmsnorm_digitize(e->p_a, L.post_ln, dp, s));
    E_TRY(mark(kBcGateUp));
    E_TRY(tgemm_gateup_decode(L, dp, e->p_h, s));
    E_TRY(mark(kBcDigits));
    E_TRY(tgemm_digitize(e->p_h, dph, s));
    E_TRY(mark(kBcDown));
    E_TRY(tgemm_down(L, dph, e->p_a, e->p_x, true, s));
    if (e->dump_hidden)
      E_TRY(cudaMemcpyAsync(e->dump + (size_t)l * n * kHidden, e->p_x, (size_t)n * kHidden * 4,
                            cudaMemcpyDeviceToDevice, s));
  }
  E_TRY(mark(kBcHead));
  if (int st = enqueue_lm_head(e, e->p_x, n, e->d_next, e->keep_logits ? e->logits : nullptr, false)) return st;
  E_TRY(mark(kBcCats));  // end marker
  if (advance) {
    advance_kernel<<<(n + 127) / 128, 128, 0, s>>>(e->d_tokens, e->d_next, e->d_pos, n);
    E_TRY(cudaGetLastError());
  }
  return 0;
}

// Batched step through a CUDA graph per (token count, 512-position bucket): removes the host cost of the
// ~340 launches (tensor-map encoding included) from the step.
int run_decode_step_batched(qwen_engine* e, int n, int max_len, bool advance) {
  const int chunks = (max_len + 63) / 64;
  const int bucket = ((chunks + 7) / 8) * 8;
  const int grid_len = bucket * 64;
  if (!e->use_graphs || e->dump_hidden || e->keep_logits || e->time_batched)
    return enqueue_decode_batched(e, n, grid_len, advance);
  const long long key = (1ll << 62) | ((long long)n << 40) | ((long long)advance << 39) | bucket;
  auto it = e->graphs.find(key);
  if (it == e->graphs.end()) {
    // one eager pass first (same positions: it writes exactly what the graph will rewrite), so that every
    // kernel's one-time set-up happens outside stream capture
    if (int st = enqueue_decode_batched(e, n, grid_len, false)) return st;
    cudaGraph_t g;
    E_TRY(cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal));
    const int st = enqueue_decode_batched(e, n, grid_len, advance);
    cudaError_t ce = cudaStreamEndCapture(e->stream, &g);
    if (st) return st;
    E_TRY(ce);
    cudaGraphExec_t exec;
    E_TRY(cudaGraphInstantiate(&exec, g, 0));
    cudaGraphDestroy(g);
    it = e->graphs.emplace(key, exec).first;
  }
  E_TRY(cudaGraphLaunch(it->second, e->stream));
  return 0;
}

int run_decode_step(qwen_engine* e, int nt, int max_len, bool advance) {
  if (int st = ensure_tiles(e)) return st;
  const int chunks = (max_len + 63) / 64;
  const int bucket = ((chunks + 7) / 8) * 8;  // re-capture every 512 positions
  const int grid_len = bucket * 64;
  if (!e->use_graphs || e->dump_hidden || e->keep_logits) return enqueue_decode(e, nt, grid_len, advance);
  const long long key = ((long long)nt << 40) | ((long long)advance << 39) | bucket;
  auto it = e->graphs.find(key);
  if (it == e->graphs.end()) {
    // one eager pass first (same positions: it writes exactly what the graph will rewrite), so every
    // kernel's one-time attribute setup happens outside stream capture
    if (int st = enqueue_decode(e, nt, grid_len, false)) return st;
    cudaGraph_t g;
    E_TRY(cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal));
    const int st = enqueue_decode(e, nt, grid_len, advance);
    cudaError_t ce = cudaStreamEndCapture(e->stream, &g);
    if (st) return st;
    E_TRY(ce);
    cudaGraphExec_t exec;
    E_TRY(cudaGraphInstantiate(&exec, g, 0));
    cudaGraphDestroy(g);
    it = e->graphs.emplace(key, exec).first;
  }
  E_TRY(cudaGraphLaunch(it->second, e->stream));
  return 0;
}

// The device work of one prefill (tokens already in p_tokens): embedding gather, 28 layers, LM head of the
// last token into d_next. past > 0: a chunk continuing a slot that holds `past` tokens (chunked prefill):
// the chunk's rows take positions past .. past + n - 1 (RoPE rows and flat K/V rows offset by past), the
// slot's cached rows are gathered in front of them, and the attention runs with that query offset.
int enqueue_prefill(qwen_engine* e, int slot, int n, int past) {
  if (e->exact) return enqueue_prefill_exact(e, slot, n, past);
  cudaStream_t s = e->stream;
  float* kf = e->p_k + (size_t)past * kKvWidth;  // this chunk's K / V rows in the flat buffers
  float* vf = e->p_v + (size_t)past * kKvWidth;
  const float* rc = e->rope_pre_cos + (size_t)past * 64;
  const float* rs = e->rope_pre_sin + (size_t)past * 64;
  embed_gather_kernel<<<n, 256, 0, s>>>(e->embed, e->p_tokens, n, e->p_x);
  E_TRY(cudaGetLastError());
  const bool tc = e->wbits == 8;
  const DigitPlanes dp{e->p_planes, e->p_steps, n, tgemm_pad(n), kHidden};
  const DigitPlanes dph{e->p_planes, e->p_steps, n, tgemm_pad(n), kInter};
  for (int l = 0; l < kLayers; ++l) {
    const LayerDev& L = e->layers[l];
    if (tc) {  // W8: projections on the int8 tensor cores
      E_TRY(tgemm_prefill_rmsnorm_digitize(e->p_x, L.input_ln, dp, s));
      E_TRY(tgemm_qkv(L, dp, rc, rs, e->p_q, kf, vf, e->p_qkv, s));
    } else {
      E_TRY(launch_prefill_rmsnorm(e->p_x, L.input_ln, n, e->p_xn, s));
      E_TRY(launch_prefill_qkv(e->wbits, L, e->p_xn, n, rc, rs, e->p_q, kf, vf, s));
    }
    if (int st = gather_history(e, slot, l, past, true)) return st;
    if (e->use_attn_tc) {
      E_TRY(launch_prefill_attention_tc(e->p_q, e->p_k, e->p_v, n, e->p_ctx, e->p_attn, e->p_attn_bytes, s, past));
    } else {
      E_TRY(launch_prefill_attention(e->p_q, e->p_k, e->p_v, n, e->p_ctx, s, past));
    }
    if (tc) {
      E_TRY(tgemm_digitize(e->p_ctx, dp, s));
      E_TRY(tgemm_o(L, dp, e->p_a, s));
    } else {
      E_TRY(launch_prefill_o(e->wbits, L, e->p_ctx, n, e->p_a, s));
    }
    E_TRY(launch_k(kv_scatter_kernel, dim3(n), dim3(256), 0, s, true, static_cast<const float*>(kf),
                   static_cast<const float*>(vf), n, paged_view(e, l), slot, 1, past));
    if (tc) {
      E_TRY(tgemm_prefill_rmsnorm_digitize(e->p_a, L.post_ln, dp, s));
      E_TRY(tgemm_gateup(L, dp, e->p_h, s));
      E_TRY(tgemm_digitize(e->p_h, dph, s));
      E_TRY(tgemm_down(L, dph, e->p_a, e->p_x, true, s));
    } else {
      E_TRY(launch_prefill_rmsnorm(e->p_a, L.post_ln, n, e->p_xn, s));
      E_TRY(launch_prefill_gateup(e->wbits, L, e->p_xn, n, e->p_h, s));
      E_TRY(launch_prefill_down(e->wbits, L, e->p_h, e->p_a, n, e->p_x, true, s));
    }
    if (e->dump_hidden) {
      // prefill keeps each layer's output row of the last prompt token
      E_TRY(cudaMemcpyAsync(e->dump + (size_t)l * kHidden, e->p_x + (size_t)(n - 1) * kHidden, kHidden * 4,
                            cudaMemcpyDeviceToDevice, s));
    }
  }
  if (int st = enqueue_lm_head(e, e->p_x + (size_t)(n - 1) * kHidden, 1, e->d_next,
                               e->keep_logits ? e->logits : nullptr, false))
    return st;
  return 0;
}

// Prefill through a CUDA graph per (token count, slot) once one eager pass has run (kernel set-up outside
// capture): the ~12 launches per layer of a short prompt otherwise cost host time comparable to the work.
int run_prefill(qwen_engine* e, int slot, int n, int past) {
  if (!e->use_graphs || e->dump_hidden || e->keep_logits) return enqueue_prefill(e, slot, n, past);
  const long long key = (2ll << 61) | ((long long)past << 36) | ((long long)n << 20) | slot;
  auto it = e->graphs.find(key);
  if (it == e->graphs.end()) {
    if (int st = enqueue_prefill(e, slot, n, past)) return st;
    cudaGraph_t g;
    E_TRY(cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal));
    const int st = enqueue_prefill(e, slot, n, past);
    cudaError_t ce = cudaStreamEndCapture(e->stream, &g);
    if (st) return st;
    E_TRY(ce);
    cudaGraphExec_t exec;
    E_TRY(cudaGraphInstantiate(&exec, g, 0));
    cudaGraphDestroy(g);
    e->graphs.emplace(key, exec);
    return 0;  // the eager pass produced this call's result
  }
  E_TRY(cudaGraphLaunch(it->second, e->stream));
  return 0;
}

}  // namespace

extern "C" {

int qwen_engine_create(int device, int wbits, int max_seqs, int max_len, qwen_engine** out) {
  if (!out || (wbits != 4 && wbits != 8) || max_seqs <= 0 || max_len <= 0 || max_len > kMaxSeq) return kStatusInvalid;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) {
    set_error("CUDA device %d is not available", device);
    return kStatusNoDevice;
  }
  qwen_engine* e = new qwen_engine();
  e->device = device;
  e->wbits = wbits;
  e->max_seqs = max_seqs;
  e->max_len = max_len;
  e->max_pages = (max_len + kPage - 1) / kPage;
  E_TRY(cudaSetDevice(device));
  E_TRY(cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking));
  const LayerLayout lay = layer_layout(wbits);
  e->layer_bytes = (lay.total + 255) / 256 * 256;
  E_TRY(dalloc(&e->wimg, e->layer_bytes * kLayers));
  E_TRY(dalloc(&e->simg, e->layer_bytes / 4 * kLayers));
  for (int l = 0; l < kLayers; ++l)
    e->layers[l] = layer_dev_from_ddr(e->wimg + e->layer_bytes * l, e->simg + e->layer_bytes / 4 * l, wbits);
  if (wbits == 8) {
    for (int l = 0; l < kLayers; ++l)
      if (!qgemm_make_layer_maps(&e->maps[l], e->layers[l])) {
        set_error("cuTensorMapEncodeTiled failed for layer %d", l);
        return kStatusCuda;
      }
    E_TRY(dalloc(&e->qsc.acc, qgemm_acc_ints()));
    E_TRY(dalloc(&e->qsc.cnt, qgemm_counter_count()));
    E_TRY(cudaMemset(e->qsc.acc, 0, qgemm_acc_ints() * 4));
    E_TRY(cudaMemset(e->qsc.cnt, 0, qgemm_counter_count() * 4));
    int sms = 0;
    E_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
    int coop = 0;
    E_TRY(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, device));
    if (coop && stack::decode_stack_smem() <= (size_t)227 * 1024) {
      const stack::Schedule sc = stack::build_schedule(sms);
      e->stack_ctas = sms;
      E_TRY(dalloc(&e->wtiles, (size_t)kLayers * stack::kLayerTileBytes));
      E_TRY(dalloc(&e->d_layers, (size_t)kLayers));
      E_TRY(cudaMemcpy(e->d_layers, e->layers, sizeof(LayerDev) * kLayers, cudaMemcpyHostToDevice));
      E_TRY(cudaMalloc(&e->sync, sizeof(stack::SyncWords)));
      E_TRY(cudaMemset(e->sync, 0, sizeof(stack::SyncWords)));
      E_TRY(dalloc(&e->stack_acc, stack::kAccInts));
      E_TRY(cudaMemset(e->stack_acc, 0, stack::kAccInts * 4));
      E_TRY(dalloc(&e->stack_steps, (size_t)kLayers * 16));
      E_TRY(cudaMemset(e->stack_steps, 0, (size_t)kLayers * 16 * 4));
      E_TRY(dalloc(&e->d_item_off, sc.off.size()));
      E_TRY(cudaMemcpy(e->d_item_off, sc.off.data(), sc.off.size() * 4, cudaMemcpyHostToDevice));
      E_TRY(dalloc(&e->d_items, sc.items.size()));
      E_TRY(cudaMemcpy(e->d_items, sc.items.data(), sc.items.size() * sizeof(stack::Item), cudaMemcpyHostToDevice));
    }
  }
  E_TRY(dalloc(&e->embed, (size_t)kVocab * kHidden));
  E_TRY(dalloc(&e->final_norm, (size_t)kHidden));
  e->n_pages = max_seqs * e->max_pages;
  E_TRY(dalloc(&e->kv_pool, (size_t)e->n_pages * kPageFloats));
  E_TRY(dalloc(&e->d_page_table, (size_t)max_seqs * e->max_pages));
  e->page_table.assign((size_t)max_seqs * e->max_pages, -1);
  E_TRY(cudaMemcpy(e->d_page_table, e->page_table.data(), e->page_table.size() * 4, cudaMemcpyHostToDevice));
  for (int p = e->n_pages - 1; p >= 0; --p) e->free_pages.push_back(p);
  e->seq_len.assign(max_seqs, 0);
  // tokens per decode step: up to 4 in the persistent kernel, up to max_seqs in the batched W8 path
  const int T = std::max(kGemvMaxTokens, max_seqs);
  e->batch_cap = T;
  E_TRY(dalloc(&e->d_tokens, T));
  E_TRY(dalloc(&e->d_pos, T));
  E_TRY(dalloc(&e->d_seq, T));
  E_TRY(dalloc(&e->d_next, T));
  E_TRY(cudaMallocHost(&e->h_io, 16 * sizeof(int)));
  E_TRY(cudaMallocHost(&e->hb_io, (size_t)4 * T * sizeof(int)));
  E_TRY(dalloc(&e->x, (size_t)T * kHidden));
  E_TRY(dalloc(&e->q, (size_t)T * kHidden));
  E_TRY(dalloc(&e->ctx, (size_t)T * kHidden));
  E_TRY(dalloc(&e->a, (size_t)T * kHidden));
  E_TRY(dalloc(&e->y0, (size_t)T * kHidden));
  E_TRY(dalloc(&e->y1, (size_t)T * kHidden));
  E_TRY(dalloc(&e->h, (size_t)T * kInter));
  e->attn_max_chunks = (max_len + 512 + 64 + 63) / 64;
  E_TRY(dalloc(&e->attn_part, std::max(attn_partial_floats(T, max_len + 512 + 64),
                                       stack::attn_part_floats(T, e->attn_max_chunks))));
  if (e->stack_ctas > 0 && bs1::decode_bs1_smem() <= (size_t)227 * 1024) {
    const int ctas1 = std::min(e->stack_ctas, bs1::kMinCtas);
    const stack::Schedule s1 = bs1::build_schedule(ctas1);
    if (!s1.off.empty()) {
      bs1::Buffers& b = e->bs1_buf;
      const size_t words[7] = {bs1::acc_words(), bs1::part_words(e->attn_max_chunks), bs1::ctx_words(),
                               bs1::cmax_words(), bs1::h_words(), bs1::hmax_words(), bs1::step_words()};
      unsigned long long** ptrs[7] = {&b.acc, &b.part, &b.ctx, &b.cmax, &b.h, &b.hmax, &b.steps};
      for (int i = 0; i < 7; ++i) {
        E_TRY(dalloc(ptrs[i], words[i]));
        E_TRY(cudaMemset(*ptrs[i], 0, words[i] * 8));
      }
      E_TRY(cudaMalloc(&e->bs1_sync, sizeof(bs1::Sync)));
      E_TRY(cudaMemset(e->bs1_sync, 0, sizeof(bs1::Sync)));
      E_TRY(dalloc(&e->d_item_off1, (size_t)e->stack_ctas + 1));  // option "bs1_ctas" goes up to every SM
      E_TRY(cudaMemcpy(e->d_item_off1, s1.off.data(), s1.off.size() * 4, cudaMemcpyHostToDevice));
      e->bs1_ctas = ctas1;
      E_TRY(dalloc(&e->d_items1, s1.items.size()));
      E_TRY(cudaMemcpy(e->d_items1, s1.items.data(), s1.items.size() * sizeof(stack::Item), cudaMemcpyHostToDevice));
    }
  }
  E_TRY(dalloc(&e->attn_cnt, (size_t)T * kKvHeads));
  E_TRY(cudaMemset(e->attn_cnt, 0, (size_t)T * kKvHeads * 4));
  {
    uint8_t* lm = nullptr;
    E_TRY(cudaMalloc(&lm, lm_scratch_bytes()));
    E_TRY(cudaMemset(lm, 0, lm_scratch_bytes()));
    e->lm.planes = reinterpret_cast<__half*>(lm);
    e->lm.packed = reinterpret_cast<unsigned long long*>(lm + (size_t)2 * 128 * kHidden * 2);
    e->lm.counter = reinterpret_cast<unsigned*>(lm + (size_t)2 * 128 * kHidden * 2 + 128 * 8);
  }
  E_TRY(dalloc(&e->lm_part, (size_t)lm_head_partial_floats()));
  E_TRY(dalloc(&e->lm_cnt, 1));
  E_TRY(cudaMemset(e->lm_cnt, 0, 4));
  E_TRY(dalloc(&e->dump, (size_t)kLayers * T * kHidden));
  E_TRY(dalloc(&e->logits, (size_t)T * kVocab));
  if (int st = ensure_rope_dec(e, max_len + 1)) return st;
  *out = e;
  return 0;
}

void qwen_engine_destroy(qwen_engine* e) {
  if (!e) return;
  cudaSetDevice(e->device);
  if (e->gather_stream) {
    cudaStreamSynchronize(e->gather_stream);
    cudaStreamDestroy(e->gather_stream);
  }
  for (cudaEvent_t ev : {e->gather_ready, e->gather_done[0], e->gather_done[1]})
    if (ev) cudaEventDestroy(ev);
  if (e->nccl) {
    cudaStreamSynchronize(e->stream);
    if (const NcclApi* api = nccl_api()) api->comm_destroy(e->nccl);
    e->nccl = nullptr;
  }
  for (auto& kv : e->graphs) cudaGraphExecDestroy(kv.second);
  void* ptrs[] = {e->wimg, e->simg, e->embed, e->final_norm, e->kv_pool, e->d_page_table, e->d_tokens, e->d_pos,
                  e->d_seq, e->d_next, e->x, e->q, e->ctx, e->a, e->y0, e->y1, e->h, e->attn_part, e->attn_cnt,
                  e->lm_part, e->lm_cnt, e->dump, e->logits, e->rope_dec_cos, e->rope_dec_sin, e->rope_pre_cos,
                  e->rope_pre_sin, e->p_x, e->p_xn, e->p_q, e->p_ctx, e->p_a, e->p_h, e->p_k, e->p_v, e->p_tokens,
                  e->qsc.acc, e->qsc.cnt, e->wtiles, e->d_layers, e->sync, e->stack_acc, e->stack_steps,
                  e->d_item_off, e->d_items, e->bs1_buf.acc, e->bs1_buf.part, e->bs1_buf.ctx, e->bs1_buf.cmax,
                  e->bs1_buf.h, e->bs1_buf.hmax, e->bs1_buf.steps, e->bs1_sync, e->d_item_off1, e->d_items1};
  for (void* p : ptrs) cudaFree(p);
  cudaFree(e->trace);
  cudaFree(e->lm.planes);
  cudaFree(e->p_planes);
  cudaFree(e->p_steps);
  cudaFree(e->p_attn);
  cudaFree(e->p_qkv);
  cudaFree(e->ex_xn);
  cudaFree(e->ex_qkv);
  cudaFree(e->ex_gu);
  for (cudaEvent_t ev : e->kev)
    if (ev) cudaEventDestroy(ev);
  for (cudaEvent_t ev : e->bev) cudaEventDestroy(ev);
  if (e->h_io) cudaFreeHost(e->h_io);
  if (e->hb_io) cudaFreeHost(e->hb_io);
  if (e->stream) cudaStreamDestroy(e->stream);
  delete e;
}

int qwen_engine_init_synthetic(qwen_engine* e, uint64_t seed, float weight_sigma) {
  if (!e) return kStatusInvalid;
  E_TRY(cudaSetDevice(e->device));
  for (int l = 0; l < kLayers; ++l)
    E_TRY(launch_synth_layer(seed, l, e->wbits, weight_sigma, e->wimg + e->layer_bytes * l,
                             e->simg + e->layer_bytes / 4 * l, e->stream));
  E_TRY(launch_synth_embedding(seed, e->embed, e->stream));
  E_TRY(launch_synth_fill(seed, (1ull << 20) + 1, kHidden, 1.0f, 0.02f, e->final_norm, e->stream));
  e->tiles_dirty = true;
  if (int st = ensure_tiles(e)) return st;
  E_TRY(cudaStreamSynchronize(e->stream));
  return 0;
}

int qwen_engine_load_layer(qwen_engine* e, int layer, const uint8_t* weight_ddr, const float* scale_ddr) {
  if (!e || layer < 0 || layer >= kLayers || !weight_ddr || !scale_ddr) return kStatusInvalid;
  E_TRY(cudaSetDevice(e->device));
  const LayerLayout lay = layer_layout(e->wbits);
  E_TRY(cudaMemcpy(e->wimg + e->layer_bytes * layer, weight_ddr, lay.total, cudaMemcpyDefault));
  E_TRY(cudaMemcpy(e->simg + e->layer_bytes / 4 * layer, scale_ddr, lay.total / 4 * 4, cudaMemcpyDefault));
  e->tiles_dirty = true;
  return 0;
}

int qwen_engine_load_embedding(qwen_engine* e, const uint16_t* embed_f16, const float* final_norm) {
  if (!e || !embed_f16 || !final_norm) return kStatusInvalid;
  E_TRY(cudaSetDevice(e->device));
  E_TRY(cudaMemcpy(e->embed, embed_f16, (size_t)kVocab * kHidden * 2, cudaMemcpyDefault));
  E_TRY(cudaMemcpy(e->final_norm, final_norm, (size_t)kHidden * 4, cudaMemcpyDefault));
  return 0;
}

int qwen_engine_set_option(qwen_engine* e, const char* name, long long value) {
  if (!e || !name) return kStatusInvalid;
  const std::string n(name);
  if (n == "graphs") e->use_graphs = value != 0;
  else if (n == "pdl") {
    e->use_pdl = value != 0;
    for (auto& kv : e->graphs) cudaGraphExecDestroy(kv.second);
    e->graphs.clear();
  } else if (n == "prefetch") {
    e->prefetch = value != 0;
    for (auto& kv : e->graphs) cudaGraphExecDestroy(kv.second);
    e->graphs.clear();
  } else if (n == "trace") {
    if (value != 0 && e->trace == nullptr && e->stack_ctas > 0) {
      const size_t n_stamps = (size_t)e->stack_ctas * kLayers * stack::kTraceSlots;
      E_TRY(cudaMalloc(&e->trace, n_stamps * 8));
      E_TRY(cudaMemset(e->trace, 0, n_stamps * 8));
    } else if (value == 0 && e->trace != nullptr) {
      E_TRY(cudaFree(e->trace));
      e->trace = nullptr;
    }
    for (auto& kv : e->graphs) cudaGraphExecDestroy(kv.second);
    e->graphs.clear();
  } else if (n == "stack_ring") {
    if (value < 2 || value > 9) return kStatusInvalid;
    e->stack_ring = (int)value;
    for (auto& kv : e->graphs) cudaGraphExecDestroy(kv.second);
    e->graphs.clear();
  } else if (n == "lm_tc") {
    e->use_lm_tc = value != 0;
    for (auto& kv : e->graphs) cudaGraphExecDestroy(kv.second);
    e->graphs.clear();
  } else if (n == "prefill_attn_tc") {
    e->use_attn_tc = value != 0;
  } else if (n == "attn_ctas") {
    if (value < 0) return kStatusInvalid;
    e->attn_ctas = value;
    for (auto& kv : e->graphs) cudaGraphExecDestroy(kv.second);
    e->graphs.clear();
  } else if (n == "batched") {
    e->use_batched = value != 0;
  } else if (n == "stack") {
    e->use_stack = value != 0;
    for (auto& kv : e->graphs) cudaGraphExecDestroy(kv.second);
    e->graphs.clear();
  } else if (n == "bs1_ctas") {
    // the batch-1 kernel on fewer CTAs than SMs, leaving SMs free for kernels on other streams (the NCCL
    // gather of a multi-GPU run); the schedule needs at least as many CTAs as one projection has items
    if (e->d_items1 == nullptr || value < 1 || value > e->stack_ctas) return kStatusInvalid;
    const stack::Schedule s1 = bs1::build_schedule((int)value);
    if (s1.off.empty()) {
      set_error("bs1_ctas %lld: fewer CTAs than the items of one projection", value);
      return kStatusInvalid;
    }
    E_TRY(cudaSetDevice(e->device));
    E_TRY(cudaStreamSynchronize(e->stream));
    E_TRY(cudaMemcpy(e->d_item_off1, s1.off.data(), s1.off.size() * 4, cudaMemcpyHostToDevice));
    E_TRY(cudaMemcpy(e->d_items1, s1.items.data(), s1.items.size() * sizeof(stack::Item), cudaMemcpyHostToDevice));
    e->bs1_ctas = (int)value;
    for (auto& kv : e->graphs) cudaGraphExecDestroy(kv.second);
    e->graphs.clear();
  } else if (n == "bs1_poison") {
    e->bs1_poison = value != 0;
    for (auto& kv : e->graphs) cudaGraphExecDestroy(kv.second);
    e->graphs.clear();
  } else if (n == "bs1") {
    e->use_bs1 = value != 0;
    for (auto& kv : e->graphs) cudaGraphExecDestroy(kv.second);
    e->graphs.clear();
  } else if (n == "qgemm") {
    e->use_qgemm = value != 0;
    for (auto& kv : e->graphs) cudaGraphExecDestroy(kv.second);
    e->graphs.clear();
  } else if (n == "exact") {
    e->exact = value != 0;
    if (e->exact) {
      E_TRY(cudaSetDevice(e->device));
      if (int st = ensure_exact(e, e->pre_cap)) return st;
    }
    for (auto& kv : e->graphs) cudaGraphExecDestroy(kv.second);
    e->graphs.clear();
  } else if (n == "dump_hidden") e->dump_hidden = value != 0;
  else if (n == "logits") e->keep_logits = value != 0;
  else return kStatusInvalid;
  return 0;
}

namespace {

// n prompt tokens into `slot` after the `past` tokens it holds (0: a fresh prompt).
int prefill_at(qwen_engine* e, int slot, const int32_t* tokens, int n, int past, int32_t* next_token) {
  if (n <= 0 || past < 0 || past + n > e->max_len) {
    set_error("prefill of %d tokens after %d exceeds the engine's max_len %d", n, past, e->max_len);
    return kStatusInvalid;
  }
  for (int i = 0; i < n; ++i)
    if (tokens[i] < 0 || tokens[i] >= kVocab) return kStatusInvalid;
  E_TRY(cudaSetDevice(e->device));
  if (int st = ensure_prefill_buffers(e, past + n)) return st;  // flat K/V rows: history + chunk
  if (e->exact) {
    if (int st = ensure_exact(e, n)) return st;
  }
  if (int st = ensure_rope_pre(e, past + n)) return st;
  if (int st = ensure_pages(e, slot, past + n)) return st;
  cudaStream_t s = e->stream;
  E_TRY(cudaMemcpyAsync(e->p_tokens, tokens, (size_t)n * 4, cudaMemcpyHostToDevice, s));
  if (int st = run_prefill(e, slot, n, past)) return st;
  E_TRY(cudaMemcpyAsync(e->h_io + 12, e->d_next, 4, cudaMemcpyDeviceToHost, s));
  E_TRY(cudaStreamSynchronize(s));
  e->seq_len[slot] = past + n;
  e->last_rows = 1;
  e->dev_slots.clear();
  if (next_token) *next_token = e->h_io[12];
  return 0;
}

}  // namespace

int qwen_engine_prefill(qwen_engine* e, int slot, const int32_t* tokens, int n, int32_t* next_token) {
  if (!e || slot < 0 || slot >= e->max_seqs || !tokens || n <= 0 || n > e->max_len) return kStatusInvalid;
  if (e->seq_len[slot] != 0) {
    set_error("prefill into a non-empty slot %d (reset it first, or continue it with qwen_engine_prefill_chunk)",
              slot);
    return kStatusInvalid;
  }
  return prefill_at(e, slot, tokens, n, 0, next_token);
}

int qwen_engine_prefill_chunk(qwen_engine* e, int slot, const int32_t* tokens, int n, int32_t* next_token) {
  if (!e || slot < 0 || slot >= e->max_seqs || !tokens || n <= 0) return kStatusInvalid;
  return prefill_at(e, slot, tokens, n, e->seq_len[slot], next_token);
}

int qwen_engine_decode(qwen_engine* e, const int32_t* slots, const int32_t* tokens, int n, int32_t* next_tokens) {
  if (!e || !slots || !tokens || n <= 0) return kStatusInvalid;
  E_TRY(cudaSetDevice(e->device));
  if (batched_ok(e, n)) {
    int max_len = 0;
    std::vector<char> seen(e->max_seqs, 0);
    for (int i = 0; i < n; ++i) {
      const int slot = slots[i];
      if (slot < 0 || slot >= e->max_seqs || seen[slot] || tokens[i] < 0 || tokens[i] >= kVocab) return kStatusInvalid;
      seen[slot] = 1;
      const int pos = e->seq_len[slot];
      if (int st = ensure_pages(e, slot, pos + 1)) return st;
      e->hb_io[i] = tokens[i];
      e->hb_io[e->batch_cap + i] = pos;
      e->hb_io[2 * e->batch_cap + i] = slot;
      max_len = std::max(max_len, pos + 1);
    }
    if (int st = ensure_rope_dec(e, max_len)) return st;
    if (int st = ensure_prefill_buffers(e, n)) return st;
    e->dev_slots.clear();
    E_TRY(cudaMemcpyAsync(e->d_tokens, e->hb_io, n * 4, cudaMemcpyHostToDevice, e->stream));
    E_TRY(cudaMemcpyAsync(e->d_pos, e->hb_io + e->batch_cap, n * 4, cudaMemcpyHostToDevice, e->stream));
    E_TRY(cudaMemcpyAsync(e->d_seq, e->hb_io + 2 * e->batch_cap, n * 4, cudaMemcpyHostToDevice, e->stream));
    if (int st = run_decode_step_batched(e, n, max_len, false)) return st;
    E_TRY(cudaMemcpyAsync(e->hb_io + 3 * e->batch_cap, e->d_next, n * 4, cudaMemcpyDeviceToHost, e->stream));
    E_TRY(cudaStreamSynchronize(e->stream));
    for (int i = 0; i < n; ++i) {
      next_tokens[i] = e->hb_io[3 * e->batch_cap + i];
      e->seq_len[slots[i]] += 1;
    }
    e->last_rows = n;
    return 0;
  }
  for (int base = 0; base < n; base += kGemvMaxTokens) {
    const int nt = std::min(kGemvMaxTokens, n - base);
    int max_len = 0;
    for (int i = 0; i < nt; ++i) {
      const int slot = slots[base + i];
      if (slot < 0 || slot >= e->max_seqs || tokens[base + i] < 0 || tokens[base + i] >= kVocab) return kStatusInvalid;
      for (int j = 0; j < i; ++j)
        if (slots[base + j] == slot) return kStatusInvalid;
      const int pos = e->seq_len[slot];
      if (int st = ensure_pages(e, slot, pos + 1)) return st;
      e->h_io[i] = tokens[base + i];
      e->h_io[4 + i] = pos;
      e->h_io[8 + i] = slot;
      max_len = std::max(max_len, pos + 1);
    }
    if (int st = ensure_rope_dec(e, max_len)) return st;
    e->dev_slots.clear();
    E_TRY(cudaMemcpyAsync(e->d_tokens, e->h_io, nt * 4, cudaMemcpyHostToDevice, e->stream));
    E_TRY(cudaMemcpyAsync(e->d_pos, e->h_io + 4, nt * 4, cudaMemcpyHostToDevice, e->stream));
    E_TRY(cudaMemcpyAsync(e->d_seq, e->h_io + 8, nt * 4, cudaMemcpyHostToDevice, e->stream));
    if (int st = run_decode_step(e, nt, max_len, false)) return st;
    E_TRY(cudaMemcpyAsync(e->h_io + 12, e->d_next, nt * 4, cudaMemcpyDeviceToHost, e->stream));
    E_TRY(cudaStreamSynchronize(e->stream));
    for (int i = 0; i < nt; ++i) {
      next_tokens[base + i] = e->h_io[12 + i];
      e->seq_len[slots[base + i]] += 1;
    }
    e->last_rows = nt;
  }
  return 0;
}

int qwen_engine_bench_decode(qwen_engine* e, const int32_t* slots, const int32_t* first_tokens, int n, int steps,
                             int warmup, float* ms_per_step) {
  if (!e || !slots || !first_tokens || n <= 0 || steps <= 0 || warmup < 0) return kStatusInvalid;
  if (n > kGemvMaxTokens && !batched_ok(e, n)) return kStatusInvalid;
  E_TRY(cudaSetDevice(e->device));
  if (n > kGemvMaxTokens) {
    int max_end = 0;
    for (int i = 0; i < n; ++i) {
      const int slot = slots[i];
      if (slot < 0 || slot >= e->max_seqs) return kStatusInvalid;
      const int end = e->seq_len[slot] + warmup + steps;
      if (int st = ensure_pages(e, slot, end)) return st;
      e->hb_io[i] = first_tokens[i];
      e->hb_io[e->batch_cap + i] = e->seq_len[slot];
      e->hb_io[2 * e->batch_cap + i] = slot;
      max_end = std::max(max_end, end);
    }
    if (int st = ensure_rope_dec(e, max_end)) return st;
    if (int st = ensure_prefill_buffers(e, n)) return st;
    e->dev_slots.clear();
    E_TRY(cudaMemcpyAsync(e->d_tokens, e->hb_io, n * 4, cudaMemcpyHostToDevice, e->stream));
    E_TRY(cudaMemcpyAsync(e->d_pos, e->hb_io + e->batch_cap, n * 4, cudaMemcpyHostToDevice, e->stream));
    E_TRY(cudaMemcpyAsync(e->d_seq, e->hb_io + 2 * e->batch_cap, n * 4, cudaMemcpyHostToDevice, e->stream));
    for (int i = 0; i < warmup; ++i)
      if (int st = run_decode_step_batched(e, n, max_end, true)) return st;
    cudaEvent_t t0, t1;
    E_TRY(cudaEventCreate(&t0));
    E_TRY(cudaEventCreate(&t1));
    E_TRY(cudaStreamSynchronize(e->stream));
    E_TRY(cudaEventRecord(t0, e->stream));
    for (int i = 0; i < steps; ++i)
      if (int st = run_decode_step_batched(e, n, max_end, true)) return st;
    E_TRY(cudaEventRecord(t1, e->stream));
    E_TRY(cudaEventSynchronize(t1));
    float ms = 0.f;
    E_TRY(cudaEventElapsedTime(&ms, t0, t1));
    cudaEventDestroy(t0);
    cudaEventDestroy(t1);
    for (int i = 0; i < n; ++i) e->seq_len[slots[i]] += warmup + steps;
    if (ms_per_step) *ms_per_step = ms / steps;
    return 0;
  }
  int max_end = 0;
  for (int i = 0; i < n; ++i) {
    const int slot = slots[i];
    if (slot < 0 || slot >= e->max_seqs) return kStatusInvalid;
    const int end = e->seq_len[slot] + warmup + steps;
    if (int st = ensure_pages(e, slot, end)) return st;
    e->h_io[i] = first_tokens[i];
    e->h_io[4 + i] = e->seq_len[slot];
    e->h_io[8 + i] = slot;
    max_end = std::max(max_end, end);
  }
  if (int st = ensure_rope_dec(e, max_end)) return st;
  e->dev_slots.clear();
  E_TRY(cudaMemcpyAsync(e->d_tokens, e->h_io, n * 4, cudaMemcpyHostToDevice, e->stream));
  E_TRY(cudaMemcpyAsync(e->d_pos, e->h_io + 4, n * 4, cudaMemcpyHostToDevice, e->stream));
  E_TRY(cudaMemcpyAsync(e->d_seq, e->h_io + 8, n * 4, cudaMemcpyHostToDevice, e->stream));
  // the attention grid must cover every position reached in the run: one graph for the whole run
  for (int i = 0; i < warmup; ++i)
    if (int st = run_decode_step(e, n, max_end, true)) return st;
  cudaEvent_t t0, t1;
  E_TRY(cudaEventCreate(&t0));
  E_TRY(cudaEventCreate(&t1));
  E_TRY(cudaStreamSynchronize(e->stream));
  E_TRY(cudaEventRecord(t0, e->stream));
  for (int i = 0; i < steps; ++i)
    if (int st = run_decode_step(e, n, max_end, true)) return st;
  E_TRY(cudaEventRecord(t1, e->stream));
  E_TRY(cudaEventSynchronize(t1));
  float ms = 0.f;
  E_TRY(cudaEventElapsedTime(&ms, t0, t1));
  cudaEventDestroy(t0);
  cudaEventDestroy(t1);
  for (int i = 0; i < n; ++i) e->seq_len[slots[i]] += warmup + steps;
  if (ms_per_step) *ms_per_step = ms / steps;
  return 0;
}

int qwen_engine_profile_decode(qwen_engine* e, int slot, int first_token, int steps, float* ms_out) {
  if (!e || slot < 0 || slot >= e->max_seqs || steps <= 0 || !ms_out) return kStatusInvalid;
  E_TRY(cudaSetDevice(e->device));
  const int end = e->seq_len[slot] + steps;
  if (int st = ensure_pages(e, slot, end)) return st;
  if (int st = ensure_rope_dec(e, end)) return st;
  if (int st = ensure_tiles(e)) return st;
  for (int i = 0; i < 3; ++i)
    if (e->kev[i] == nullptr) E_TRY(cudaEventCreate(&e->kev[i]));
  e->h_io[0] = first_token;
  e->h_io[4] = e->seq_len[slot];
  e->h_io[8] = slot;
  e->dev_slots.clear();
  E_TRY(cudaMemcpyAsync(e->d_tokens, e->h_io, 4, cudaMemcpyHostToDevice, e->stream));
  E_TRY(cudaMemcpyAsync(e->d_pos, e->h_io + 4, 4, cudaMemcpyHostToDevice, e->stream));
  E_TRY(cudaMemcpyAsync(e->d_seq, e->h_io + 8, 4, cudaMemcpyHostToDevice, e->stream));
  double layers_ms = 0.0, head_ms = 0.0;
  e->time_kernels = true;
  int st = 0;
  for (int i = 0; i < steps && st == 0; ++i) {
    st = enqueue_decode(e, 1, ((end + 63) / 64) * 64, true);
    if (st == 0 && cudaEventSynchronize(e->kev[2]) != cudaSuccess) st = kStatusCuda;
    float a = 0.f, b = 0.f;
    if (st == 0 && (cudaEventElapsedTime(&a, e->kev[0], e->kev[1]) != cudaSuccess ||
                    cudaEventElapsedTime(&b, e->kev[1], e->kev[2]) != cudaSuccess))
      st = kStatusCuda;
    layers_ms += a;
    head_ms += b;
  }
  e->time_kernels = false;
  if (st) return st;
  E_TRY(cudaStreamSynchronize(e->stream));
  e->seq_len[slot] += steps;
  ms_out[0] = (float)(layers_ms / steps);
  ms_out[1] = (float)(head_ms / steps);
  return 0;
}

int qwen_engine_profile_batched(qwen_engine* e, const int32_t* slots, const int32_t* first_tokens, int n, int steps,
                                float* ms_out) {
  if (!e || !slots || !first_tokens || !ms_out || steps <= 0 || !batched_ok(e, n)) return kStatusInvalid;
  E_TRY(cudaSetDevice(e->device));
  int max_end = 0;
  for (int i = 0; i < n; ++i) {
    const int slot = slots[i];
    if (slot < 0 || slot >= e->max_seqs) return kStatusInvalid;
    const int end = e->seq_len[slot] + steps;
    if (int st = ensure_pages(e, slot, end)) return st;
    e->hb_io[i] = first_tokens[i];
    e->hb_io[e->batch_cap + i] = e->seq_len[slot];
    e->hb_io[2 * e->batch_cap + i] = slot;
    max_end = std::max(max_end, end);
  }
  if (int st = ensure_rope_dec(e, max_end)) return st;
  if (int st = ensure_prefill_buffers(e, n)) return st;
  e->dev_slots.clear();
  E_TRY(cudaMemcpyAsync(e->d_tokens, e->hb_io, n * 4, cudaMemcpyHostToDevice, e->stream));
  E_TRY(cudaMemcpyAsync(e->d_pos, e->hb_io + e->batch_cap, n * 4, cudaMemcpyHostToDevice, e->stream));
  E_TRY(cudaMemcpyAsync(e->d_seq, e->hb_io + 2 * e->batch_cap, n * 4, cudaMemcpyHostToDevice, e->stream));
  double acc[kBcCats] = {0};
  e->time_batched = true;
  int st = 0;
  for (int i = 0; i < steps && st == 0; ++i) {
    st = enqueue_decode_batched(e, n, ((max_end + 63) / 64) * 64, true);
    if (st == 0 && cudaStreamSynchronize(e->stream) != cudaSuccess) st = kStatusCuda;
    // event k opens the group of category bev_cat[k]; the last event closes the LM head
    for (int k = 0; st == 0 && k + 1 < e->bev_used; ++k) {
      float ms = 0.f;
      if (cudaEventElapsedTime(&ms, e->bev[k], e->bev[k + 1]) != cudaSuccess) st = kStatusCuda;
      acc[e->bev_cat[k]] += ms;
    }
  }
  e->time_batched = false;
  if (st) return st;
  for (int i = 0; i < n; ++i) e->seq_len[slots[i]] += steps;
  for (int c = 0; c < kBcCats; ++c) ms_out[c] = (float)(acc[c] / steps);
  return 0;
}

int qwen_engine_write_kv(qwen_engine* e, int slot, int layer, const float* k, const float* v, int n_tokens) {
  if (!e || slot < 0 || slot >= e->max_seqs || layer < 0 || layer >= kLayers || !k || !v || n_tokens <= 0)
    return kStatusInvalid;
  E_TRY(cudaSetDevice(e->device));
  if (int st = ensure_prefill_buffers(e, n_tokens)) return st;
  if (int st = ensure_pages(e, slot, n_tokens)) return st;
  E_TRY(cudaMemcpyAsync(e->p_k, k, (size_t)n_tokens * kKvWidth * 4, cudaMemcpyDefault, e->stream));
  E_TRY(cudaMemcpyAsync(e->p_v, v, (size_t)n_tokens * kKvWidth * 4, cudaMemcpyDefault, e->stream));
  kv_scatter_kernel<<<n_tokens, 256, 0, e->stream>>>(e->p_k, e->p_v, n_tokens, paged_view(e, layer), slot, 1, 0);
  E_TRY(cudaGetLastError());
  E_TRY(cudaStreamSynchronize(e->stream));
  if (layer == kLayers - 1) e->seq_len[slot] = n_tokens;
  e->dev_slots.clear();
  return 0;
}

int qwen_engine_read_kv(qwen_engine* e, int slot, int layer, float* k, float* v, int n_tokens) {
  if (!e || slot < 0 || slot >= e->max_seqs || layer < 0 || layer >= kLayers || !k || !v || n_tokens <= 0 ||
      n_tokens > e->seq_len[slot])
    return kStatusInvalid;
  E_TRY(cudaSetDevice(e->device));
  if (int st = ensure_prefill_buffers(e, n_tokens)) return st;
  kv_scatter_kernel<<<n_tokens, 256, 0, e->stream>>>(e->p_k, e->p_v, n_tokens, paged_view(e, layer), slot, 0, 0);
  E_TRY(cudaGetLastError());
  E_TRY(cudaMemcpyAsync(k, e->p_k, (size_t)n_tokens * kKvWidth * 4, cudaMemcpyDefault, e->stream));
  E_TRY(cudaMemcpyAsync(v, e->p_v, (size_t)n_tokens * kKvWidth * 4, cudaMemcpyDefault, e->stream));
  E_TRY(cudaStreamSynchronize(e->stream));
  return 0;
}

int qwen_engine_read_kv_hf(qwen_engine* e, int slot, int layer, float* k, float* v, int n_tokens) {
  if (!e || slot < 0 || slot >= e->max_seqs || layer < 0 || layer >= kLayers || !k || !v || n_tokens <= 0 ||
      n_tokens > e->seq_len[slot])
    return kStatusInvalid;
  E_TRY(cudaSetDevice(e->device));
  if (int st = ensure_prefill_buffers(e, n_tokens)) return st;
  kv_hf_kernel<<<n_tokens, 256, 0, e->stream>>>(paged_view(e, layer), slot, n_tokens, e->p_k, e->p_v, 0);
  E_TRY(cudaGetLastError());
  E_TRY(cudaMemcpyAsync(k, e->p_k, (size_t)n_tokens * kKvWidth * 4, cudaMemcpyDefault, e->stream));
  E_TRY(cudaMemcpyAsync(v, e->p_v, (size_t)n_tokens * kKvWidth * 4, cudaMemcpyDefault, e->stream));
  E_TRY(cudaStreamSynchronize(e->stream));
  return 0;
}

int qwen_engine_write_kv_hf(qwen_engine* e, int slot, int layer, const float* k, const float* v, int n_tokens) {
  if (!e || slot < 0 || slot >= e->max_seqs || layer < 0 || layer >= kLayers || !k || !v || n_tokens <= 0 ||
      n_tokens > e->max_len)
    return kStatusInvalid;
  E_TRY(cudaSetDevice(e->device));
  if (int st = ensure_prefill_buffers(e, n_tokens)) return st;
  if (int st = ensure_pages(e, slot, n_tokens)) return st;
  E_TRY(cudaMemcpyAsync(e->p_k, k, (size_t)n_tokens * kKvWidth * 4, cudaMemcpyDefault, e->stream));
  E_TRY(cudaMemcpyAsync(e->p_v, v, (size_t)n_tokens * kKvWidth * 4, cudaMemcpyDefault, e->stream));
  kv_hf_kernel<<<n_tokens, 256, 0, e->stream>>>(paged_view(e, layer), slot, n_tokens, e->p_k, e->p_v, 1);
  E_TRY(cudaGetLastError());
  E_TRY(cudaStreamSynchronize(e->stream));
  if (layer == kLayers - 1) e->seq_len[slot] = n_tokens;
  e->dev_slots.clear();
  return 0;
}

int qwen_engine_set_seq_len(qwen_engine* e, int slot, int len) {
  if (!e || slot < 0 || slot >= e->max_seqs || len < 0 || len > e->max_len) return kStatusInvalid;
  if (int st = ensure_pages(e, slot, len)) return st;
  e->seq_len[slot] = len;
  e->dev_slots.clear();
  return 0;
}

int qwen_engine_seq_len(qwen_engine* e, int slot) {
  if (!e || slot < 0 || slot >= e->max_seqs) return -1;
  return e->seq_len[slot];
}

int qwen_engine_reset(qwen_engine* e, int slot) {
  if (!e || slot < 0 || slot >= e->max_seqs) return kStatusInvalid;
  for (int p = 0; p < e->max_pages; ++p) {
    int& entry = e->page_table[(size_t)slot * e->max_pages + p];
    if (entry >= 0) e->free_pages.push_back(entry);
    entry = -1;
  }
  E_TRY(cudaSetDevice(e->device));
  E_TRY(cudaMemcpy(e->d_page_table + (size_t)slot * e->max_pages, e->page_table.data() + (size_t)slot * e->max_pages,
                   (size_t)e->max_pages * 4, cudaMemcpyHostToDevice));
  e->seq_len[slot] = 0;
  e->dev_slots.clear();
  return 0;
}

int qwen_engine_read_hidden(qwen_engine* e, float* out, long long n_floats) {
  if (!e || !out) return kStatusInvalid;
  const long long have = (long long)kLayers * e->last_rows * kHidden;
  if (n_floats < have) return kStatusInvalid;
  E_TRY(cudaMemcpy(out, e->dump, (size_t)have * 4, cudaMemcpyDeviceToHost));
  return 0;
}

int qwen_engine_read_trace(qwen_engine* e, unsigned long long* out, long long n, int* ctas, int* slots) {
  if (!e || !out || !ctas || !slots) return kStatusInvalid;
  *ctas = e->stack_ctas;
  *slots = stack::kTraceSlots;
  const long long have = (long long)e->stack_ctas * kLayers * stack::kTraceSlots;
  if (e->trace == nullptr || n < have) return kStatusInvalid;
  E_TRY(cudaMemcpy(out, e->trace, (size_t)have * 8, cudaMemcpyDeviceToHost));
  return 0;
}

int qwen_engine_read_logits(qwen_engine* e, float* out, long long n_floats) {
  if (!e || !out) return kStatusInvalid;
  const long long have = (long long)e->last_rows * kVocab;
  if (n_floats < have) return kStatusInvalid;
  E_TRY(cudaMemcpy(out, e->logits, (size_t)have * 4, cudaMemcpyDeviceToHost));
  return 0;
}

int qwen_engine_decode_device(qwen_engine* e, const int32_t* slots, const int32_t* d_tokens, int n,
                              int32_t* d_next) {
  if (!e || !slots || !d_tokens || !d_next || n <= 0) return kStatusInvalid;
  const bool batched = batched_ok(e, n);
  if (n > kGemvMaxTokens && !batched) return kStatusInvalid;
  E_TRY(cudaSetDevice(e->device));
  int max_len = 0;
  const std::vector<int> want(slots, slots + n);
  std::vector<char> seen(e->max_seqs, 0);
  for (int i = 0; i < n; ++i) {
    const int slot = slots[i];
    if (slot < 0 || slot >= e->max_seqs || seen[slot]) return kStatusInvalid;
    seen[slot] = 1;
    const int pos = e->seq_len[slot];
    if (int st = ensure_pages(e, slot, pos + 1)) return st;
    max_len = std::max(max_len, pos + 1);
  }
  if (int st = ensure_rope_dec(e, max_len)) return st;
  if (batched) {
    if (int st = ensure_prefill_buffers(e, n)) return st;
  }
  if (want != e->dev_slots) {
    // (re)upload positions and slots; steady-state calls keep them on the device and advance them there
    int* hio = batched ? e->hb_io : e->h_io;
    const int cap = batched ? e->batch_cap : kGemvMaxTokens;
    E_TRY(cudaStreamSynchronize(e->stream));
    for (int i = 0; i < n; ++i) {
      hio[cap + i] = e->seq_len[slots[i]];
      hio[2 * cap + i] = slots[i];
    }
    E_TRY(cudaMemcpyAsync(e->d_pos, hio + cap, n * 4, cudaMemcpyHostToDevice, e->stream));
    E_TRY(cudaMemcpyAsync(e->d_seq, hio + 2 * cap, n * 4, cudaMemcpyHostToDevice, e->stream));
    E_TRY(cudaStreamSynchronize(e->stream));
    e->dev_slots = want;
  }
  E_TRY(cudaMemcpyAsync(e->d_tokens, d_tokens, n * 4, cudaMemcpyDeviceToDevice, e->stream));
  if (batched) {
    if (int st = run_decode_step_batched(e, n, max_len, false)) return st;
  } else {
    if (int st = run_decode_step(e, n, max_len, false)) return st;
  }
  E_TRY(cudaMemcpyAsync(d_next, e->d_next, n * 4, cudaMemcpyDeviceToDevice, e->stream));
  advance_pos_kernel<<<(n + 255) / 256, 256, 0, e->stream>>>(e->d_pos, n);
  E_TRY(cudaGetLastError());
  for (int i = 0; i < n; ++i) e->seq_len[slots[i]] += 1;
  e->last_rows = n;
  return 0;
}

int qwen_engine_read_layer(qwen_engine* e, int layer, uint8_t* weight_ddr, float* scale_ddr) {
  if (!e || layer < 0 || layer >= kLayers || !weight_ddr || !scale_ddr) return kStatusInvalid;
  E_TRY(cudaSetDevice(e->device));
  const LayerLayout lay = layer_layout(e->wbits);
  E_TRY(cudaMemcpy(weight_ddr, e->wimg + e->layer_bytes * layer, lay.total, cudaMemcpyDeviceToHost));
  E_TRY(cudaMemcpy(scale_ddr, e->simg + e->layer_bytes / 4 * layer, lay.total / 4 * 4, cudaMemcpyDeviceToHost));
  return 0;
}

int qwen_engine_profile_kernels(qwen_engine* e, int n, int past, int iters, float* ms_out) {
  if (!e || n <= 0 || n > kGemvMaxTokens || past < 0 || past + 1 > e->max_len || iters <= 0 || !ms_out)
    return kStatusInvalid;
  E_TRY(cudaSetDevice(e->device));
  // scratch sequences: slots 0..n-1 hold `past` tokens (contents are whatever the pool holds)
  for (int i = 0; i < n; ++i) {
    if (int st = ensure_pages(e, i, past + 1)) return st;
    e->h_io[i] = 1000 + i;
    e->h_io[4 + i] = past;
    e->h_io[8 + i] = i;
  }
  if (int st = ensure_rope_dec(e, past + 1)) return st;
  e->dev_slots.clear();
  E_TRY(cudaMemcpyAsync(e->d_tokens, e->h_io, n * 4, cudaMemcpyHostToDevice, e->stream));
  E_TRY(cudaMemcpyAsync(e->d_pos, e->h_io + 4, n * 4, cudaMemcpyHostToDevice, e->stream));
  E_TRY(cudaMemcpyAsync(e->d_seq, e->h_io + 8, n * 4, cudaMemcpyHostToDevice, e->stream));
  E_TRY(cudaMemsetAsync(e->y0, 0, (size_t)n * kHidden * 4, e->stream));
  E_TRY(cudaMemsetAsync(e->ctx, 0, (size_t)n * kHidden * 4, e->stream));
  E_TRY(cudaMemsetAsync(e->a, 0, (size_t)n * kHidden * 4, e->stream));
  E_TRY(cudaMemsetAsync(e->h, 0, (size_t)n * kInter * 4, e->stream));
  DecodeTokens tok{e->d_pos, e->d_seq, n};
  cudaEvent_t t0, t1;
  E_TRY(cudaEventCreate(&t0));
  E_TRY(cudaEventCreate(&t1));
  for (int kind = 0; kind < 6; ++kind) {
    auto launch = [&](int l) -> cudaError_t {
      const LayerDev& L = e->layers[l];
      KvView kv = paged_view(e, l);
      if (e->wbits == 8 && e->use_qgemm && kind != 1 && kind != 5) {
        const QgemmLayerMaps& M = e->maps[l];
        switch (kind) {
          case 0: return qgemm_qkv(M, L, XSource{e->y0, e->embed, e->d_tokens}, tok, e->rope_dec_cos, e->rope_dec_sin,
                                   e->q, kv, e->qsc, e->stream, false);
          case 2: return qgemm_o(M, L, e->ctx, n, e->a, e->qsc, e->stream, false);
          case 3: return qgemm_gateup(M, L, e->a, n, e->h, e->qsc, e->stream, false);
          default: return qgemm_down(M, L, e->h, e->a, n, e->y1, true, e->qsc, e->stream, false);
        }
      }
      switch (kind) {
        case 0: return launch_decode_qkv(e->wbits, L, XSource{e->y0, e->embed, e->d_tokens}, tok, e->rope_dec_cos,
                                         e->rope_dec_sin, e->q, kv, e->stream, false);
        case 1: return launch_decode_attention(e->q, kv, tok, past + 1, e->ctx, e->attn_part, e->attn_cnt, e->stream,
                                               false);
        case 2: return launch_decode_o(e->wbits, L, e->ctx, n, e->a, e->stream, false);
        case 3: return launch_decode_gateup(e->wbits, L, e->a, n, e->h, e->stream, false);
        case 4: return launch_decode_down(e->wbits, L, e->h, e->a, n, e->y1, true, e->stream, false);
        default: return launch_lm_head_argmax(e->embed, e->final_norm, e->y0, n, nullptr, e->lm_part, e->lm_cnt,
                                              e->d_next, e->stream, false);
      }
    };
    for (int w = 0; w < 3; ++w) E_TRY(launch(w % kLayers));
    E_TRY(cudaEventRecord(t0, e->stream));
    for (int i = 0; i < iters; ++i) E_TRY(launch(i % kLayers));
    E_TRY(cudaEventRecord(t1, e->stream));
    E_TRY(cudaEventSynchronize(t1));
    float ms = 0.f;
    E_TRY(cudaEventElapsedTime(&ms, t0, t1));
    ms_out[kind] = ms / iters;
  }
  cudaEventDestroy(t0);
  cudaEventDestroy(t1);
  return 0;
}

int qwen_engine_nccl_unique_id(uint8_t* id_out) {
  if (!id_out) return kStatusInvalid;
  const NcclApi* api = nccl_api();
  if (!api) {
    set_error("NCCL unavailable: %s", "libnccl.so.2 could not be loaded");
    return kStatusCuda;
  }
  ncclUniqueId id;
  N_TRY(api, api->get_unique_id(&id));
  std::memcpy(id_out, id.internal, NCCL_UNIQUE_ID_BYTES);
  return 0;
}

int qwen_engine_nccl_init(qwen_engine* e, const uint8_t* id, int nranks, int rank) {
  if (!e || !id || nranks <= 0 || rank < 0 || rank >= nranks || e->nccl) return kStatusInvalid;
  const NcclApi* api = nccl_api();
  if (!api) {
    set_error("NCCL unavailable: %s", "libnccl.so.2 could not be loaded");
    return kStatusCuda;
  }
  E_TRY(cudaSetDevice(e->device));
  ncclUniqueId uid;
  std::memcpy(uid.internal, id, NCCL_UNIQUE_ID_BYTES);
  N_TRY(api, api->comm_init_rank(&e->nccl, nranks, uid, rank));
  e->nccl_ranks = nranks;
  e->nccl_rank = rank;
  return 0;
}

int qwen_engine_gather_tokens(qwen_engine* e, const int32_t* d_local, int n, int32_t* d_all) {
  if (!e || !d_local || !d_all || n <= 0) return kStatusInvalid;
  if (!e->nccl) {
    set_error("qwen_engine_gather_tokens: no communicator (call qwen_engine_nccl_init first)");
    return kStatusInvalid;
  }
  const NcclApi* api = nccl_api();
  N_TRY(api, api->all_gather(d_local, d_all, (size_t)n, ncclInt32, e->nccl, e->stream));
  return 0;
}

int qwen_engine_gather_tokens_async(qwen_engine* e, const int32_t* d_local, int n, int32_t* d_all) {
  if (!e || !d_local || !d_all || n <= 0) return kStatusInvalid;
  if (!e->nccl) {
    set_error("qwen_engine_gather_tokens_async: no communicator (call qwen_engine_nccl_init first)");
    return kStatusInvalid;
  }
  E_TRY(cudaSetDevice(e->device));
  if (!e->gather_stream) {
    E_TRY(cudaStreamCreateWithFlags(&e->gather_stream, cudaStreamNonBlocking));
    E_TRY(cudaEventCreateWithFlags(&e->gather_ready, cudaEventDisableTiming));
    for (cudaEvent_t& ev : e->gather_done) E_TRY(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
  }
  const NcclApi* api = nccl_api();
  // the gather starts after the engine stream's work so far (the step that wrote d_local) and runs beside
  // the following steps
  E_TRY(cudaEventRecord(e->gather_ready, e->stream));
  E_TRY(cudaStreamWaitEvent(e->gather_stream, e->gather_ready, 0));
  N_TRY(api, api->all_gather(d_local, d_all, (size_t)n, ncclInt32, e->nccl, e->gather_stream));
  const int k = (int)(e->gather_n & 1);
  E_TRY(cudaEventRecord(e->gather_done[k], e->gather_stream));
  // at most two gathers in flight: the engine stream's work after this call waits for the previous gather,
  // so a buffer that gather read may be rewritten from the step after next on
  if (e->gather_n > 0) E_TRY(cudaStreamWaitEvent(e->stream, e->gather_done[k ^ 1], 0));
  ++e->gather_n;
  return 0;
}

int qwen_engine_gather_join(qwen_engine* e) {
  if (!e) return kStatusInvalid;
  if (e->gather_n > 0) {
    E_TRY(cudaSetDevice(e->device));
    E_TRY(cudaStreamWaitEvent(e->stream, e->gather_done[(e->gather_n - 1) & 1], 0));
  }
  return 0;
}

void* qwen_engine_stream(qwen_engine* e) { return e ? (void*)e->stream : nullptr; }

int qwen_engine_kernels_per_decode_step(qwen_engine* e, int n) {
  const int groups = (n + kGemvMaxTokens - 1) / kGemvMaxTokens;
  if (e && stack_enabled(e)) return groups * 2;
  return groups * (kLayers * 5 + 1);
}

}  // extern "C"
