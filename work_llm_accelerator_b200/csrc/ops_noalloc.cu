// Allocation-free variant of the device-pointer decode attention operator (include/qwen_b200_ops.h).
//
// Who needs it: host programs that cannot call cudaMalloc at the point where they run attention -- for
// example a serving runtime that reserves all GPU memory in its own pool at start-up and forbids any
// other allocation afterwards, or a latency-critical decode loop where cudaMalloc/cudaFree would
// synchronise the device. qwen_b200_decode_attention allocates its split-history scratch on first use;
// this entry point instead uses a fixed scratch array compiled into the library.
//
// The scratch is `g_noalloc_scratch` below: a file-scope __device__ array of kNoAllocWords 32-bit words
// (about 0.8 MB), present on every GPU that loads the library until the process exits. It holds the
// per-chunk softmax partials for histories of up to kNoAllocMaxSeq = 8192 tokens, the two per-KV-head
// completion counters and the token position. Host code cannot use the array's name as a device address
// (it names a host-side shadow), so the device address is looked up once per device with
// cudaGetSymbolAddress, with that device current, on the first call made on it; that first call should
// therefore come before any stream capture. Every call on a device reuses the same array and it keeps the
// last call's contents: each call first clears the counters and writes its position with a one-thread
// kernel on the caller's stream. Calls whose execution overlaps on the GPU (different streams, no ordering
// between them) race on the array and give wrong results.
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/qwen_b200_ops.h"
#include "qwen_kernels.cuh"
#include "runtime.h"

namespace qb {
namespace {

constexpr int kNoAllocMaxSeq = 8192;
constexpr int kNoAllocHeaderWords = 256;  // [0,2) counters, [64,66) position and sequence slot
constexpr size_t kNoAllocPartFloats = 2 * (kNoAllocMaxSeq / 64) * 6 * (2 + 128);
constexpr size_t kNoAllocWords = kNoAllocHeaderWords + kNoAllocPartFloats;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned g_noalloc_scratch[kNoAllocWords];

std::mutex g_noalloc_mu;
unsigned* g_noalloc_ptr[kMaxDevices] = {};

// Clears the completion counters and records the token position; names the array directly.
__global__ void noalloc_prepare_kernel(int pos) {
  g_noalloc_scratch[0] = 0u;
  g_noalloc_scratch[1] = 0u;
  g_noalloc_scratch[64] = (unsigned)pos;
  g_noalloc_scratch[65] = 0u;
}

bool device_accessible(const void* p) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

}  // namespace
}  // namespace qb

extern "C" int qwen_b200_decode_attention_noalloc(const float* q, const float* k_cache, const float* v_cache,
                                                  int seq_len, float* context, void* stream) {
  using namespace qb;
  if (!q || !k_cache || !v_cache || !context || seq_len <= 0) {
    set_error("qwen_b200_decode_attention_noalloc: null buffer or seq_len %d <= 0", seq_len);
    return kStatusInvalid;
  }
  if (seq_len > kNoAllocMaxSeq || attn_partial_floats(1, seq_len) > kNoAllocPartFloats) {
    set_error("qwen_b200_decode_attention_noalloc: seq_len %d exceeds the fixed scratch limit of %d tokens "
              "(use qwen_b200_decode_attention for longer histories)",
              seq_len, kNoAllocMaxSeq);
    return kStatusInvalid;
  }
  if (!device_accessible(q) || !device_accessible(k_cache) || !device_accessible(v_cache) ||
      !device_accessible(context)) {
    set_error("qwen_b200_decode_attention_noalloc: every buffer must be device (or managed) memory");
    return kStatusInvalid;
  }
  auto aligned16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (!aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache) || !aligned16(context)) {
    set_error("qwen_b200_decode_attention_noalloc: %s is not 16-byte aligned (the kernel moves 16-byte vectors)",
              !aligned16(q) ? "q" : !aligned16(k_cache) ? "k_cache" : !aligned16(v_cache) ? "v_cache" : "context");
    return kStatusInvalid;
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    set_error("qwen_b200_decode_attention_noalloc: no current CUDA device");
    return kStatusNoDevice;
  }
  unsigned* base = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (g_noalloc_ptr[dev] == nullptr) {
      void* p = nullptr;
      const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      if (e != cudaSuccess || p == nullptr) {
        set_error("qwen_b200_decode_attention_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
        return kStatusCuda;
      }
      g_noalloc_ptr[dev] = static_cast<unsigned*>(p);
    }
    base = g_noalloc_ptr[dev];
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  noalloc_prepare_kernel<<<1, 1, 0, s>>>(seq_len - 1);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) {
    int* tok_words = reinterpret_cast<int*>(base + 64);
    DecodeTokens tok{tok_words, tok_words + 1, 1};
    KvView kv{const_cast<float*>(k_cache), const_cast<float*>(v_cache), nullptr, 0, 0};
    float* part = reinterpret_cast<float*>(base + kNoAllocHeaderWords);
    e = launch_decode_attention(q, kv, tok, seq_len, context, part, base, s, false);
  }
  if (e != cudaSuccess) {
    set_error("qwen_b200_decode_attention_noalloc: %s", cudaGetErrorString(e));
    return kStatusCuda;
  }
  return 0;
}
