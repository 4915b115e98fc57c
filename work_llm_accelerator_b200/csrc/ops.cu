// Device-pointer operator API (include/qwen_b200_ops.h): hot-path kernels on caller-owned GPU buffers.
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>

#include "../../include/qwen_b200_ops.h"
#include "attention_tc.h"
#include "exact.h"
#include "qgemm.h"
#include "tgemm.h"
#include "qwen_kernels.cuh"
#include "runtime.h"

namespace qb {
namespace {

constexpr int kMaxDevices = 64;

struct OpScratch {
  float* part = nullptr;
  size_t part_floats = 0;
  unsigned* counters = nullptr;  // 2 (one per KV head), zeroed at allocation
  int* tok = nullptr;            // [pos, seq]
  QgemmScratch qsc{nullptr, nullptr};
};

std::mutex g_ops_mu;
OpScratch g_ops[kMaxDevices];

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

bool device_accessible(const void* p) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

__global__ void set_token_kernel(int* tok, int pos) {
  tok[0] = pos;
  tok[1] = 0;
}

}  // namespace
}  // namespace qb

extern "C" int qwen_b200_decode_attention(const float* q, const float* k_cache, const float* v_cache, int seq_len,
                                          float* context, void* stream) {
  using namespace qb;
  if (!q || !k_cache || !v_cache || !context || seq_len <= 0 || seq_len > kMaxSeq) {
    set_error("qwen_b200_decode_attention: null buffer or seq_len %d outside 1..%d", seq_len, kMaxSeq);
    return kStatusInvalid;
  }
  if (!device_accessible(q) || !device_accessible(k_cache) || !device_accessible(v_cache) ||
      !device_accessible(context)) {
    set_error("qwen_b200_decode_attention: every buffer must be device (or managed) memory");
    return kStatusInvalid;
  }
  if (!aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache) || !aligned16(context)) {
    set_error("qwen_b200_decode_attention: %s is not 16-byte aligned (the kernel moves 16-byte vectors)",
              !aligned16(q) ? "q" : !aligned16(k_cache) ? "k_cache" : !aligned16(v_cache) ? "v_cache" : "context");
    return kStatusInvalid;
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    set_error("qwen_b200_decode_attention: no current CUDA device");
    return kStatusNoDevice;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  std::lock_guard<std::mutex> lock(g_ops_mu);
  OpScratch& o = g_ops[dev];
  const size_t need = attn_partial_floats(1, seq_len);
  cudaError_t e = cudaSuccess;
  if (o.counters == nullptr) {
    if ((e = cudaMalloc(&o.counters, 2 * sizeof(unsigned))) == cudaSuccess &&
        (e = cudaMalloc(&o.tok, 2 * sizeof(int))) == cudaSuccess) {
      e = cudaMemset(o.counters, 0, 2 * sizeof(unsigned));
    }
  }
  if (e == cudaSuccess && o.part_floats < need) {
    if (o.part) cudaFree(o.part);
    o.part = nullptr;
    o.part_floats = 0;
    if ((e = cudaMalloc(&o.part, need * sizeof(float))) == cudaSuccess) o.part_floats = need;
  }
  if (e == cudaSuccess) {
    set_token_kernel<<<1, 1, 0, s>>>(o.tok, seq_len - 1);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) {
    DecodeTokens tok{o.tok, o.tok + 1, 1};
    KvView kv{const_cast<float*>(k_cache), const_cast<float*>(v_cache), nullptr, 0, 0};
    e = launch_decode_attention(q, kv, tok, seq_len, context, o.part, o.counters, s, false);
  }
  if (e != cudaSuccess) {
    set_error("qwen_b200_decode_attention: %s", cudaGetErrorString(e));
    return kStatusCuda;
  }
  return 0;
}

extern "C" int qwen_b200_w8_digit_products(const signed char* codes, int rows, int k, const float* x, int n_tokens,
                                           int* acc, float* step, void* stream) {
  using namespace qb;
  if (!codes || !x || !acc || !step || rows <= 0 || rows % 128 || k <= 0 || k % 128 || n_tokens < 1 ||
      n_tokens > 4 || (reinterpret_cast<uintptr_t>(codes) & 15)) {
    set_error("qwen_b200_w8_digit_products: rows %d / k %d must be positive multiples of 128, n_tokens %d in 1..4, "
              "codes 16-byte aligned",
              rows, k, n_tokens);
    return kStatusInvalid;
  }
  if (!device_accessible(codes) || !device_accessible(x) || !device_accessible(acc) || !device_accessible(step)) {
    set_error("qwen_b200_w8_digit_products: every buffer must be device (or managed) memory");
    return kStatusInvalid;
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    set_error("qwen_b200_w8_digit_products: no current CUDA device");
    return kStatusNoDevice;
  }
  std::lock_guard<std::mutex> lock(g_ops_mu);
  OpScratch& o = g_ops[dev];
  cudaError_t e = cudaSuccess;
  if (o.qsc.acc == nullptr) {
    if ((e = cudaMalloc(&o.qsc.acc, qgemm_acc_ints() * sizeof(int))) == cudaSuccess &&
        (e = cudaMalloc(&o.qsc.cnt, qgemm_counter_count() * sizeof(unsigned))) == cudaSuccess &&
        (e = cudaMemset(o.qsc.acc, 0, qgemm_acc_ints() * sizeof(int))) == cudaSuccess)
      e = cudaMemset(o.qsc.cnt, 0, qgemm_counter_count() * sizeof(unsigned));
    if (e != cudaSuccess) {
      cudaFree(o.qsc.acc);
      cudaFree(o.qsc.cnt);
      o.qsc = QgemmScratch{nullptr, nullptr};
    }
  }
  QgemmMap map;
  if (e == cudaSuccess && !qgemm_make_map(&map, reinterpret_cast<const uint8_t*>(codes), rows, k, 128)) {
    set_error("qwen_b200_w8_digit_products: cuTensorMapEncodeTiled failed");
    return kStatusCuda;
  }
  if (e == cudaSuccess) e = qgemm_raw(map, rows, k, x, n_tokens, acc, step, o.qsc, static_cast<cudaStream_t>(stream));
  if (e == cudaErrorInvalidValue) {
    set_error("qwen_b200_w8_digit_products: k %d needs more shared memory than one CTA has", k);
    return kStatusInvalid;
  }
  if (e != cudaSuccess) {
    set_error("qwen_b200_w8_digit_products: %s", cudaGetErrorString(e));
    return kStatusCuda;
  }
  return 0;
}

extern "C" int qwen_b200_w8_digit_planes(const signed char* codes, int rows, int k, const float* x, int n_tokens,
                                         int* acc, float* step, void* stream) {
  using namespace qb;
  if (!codes || !x || !acc || !step || rows <= 0 || rows % 128 || k <= 0 || k % 128 || n_tokens < 1 ||
      n_tokens > (1 << 16) || (reinterpret_cast<uintptr_t>(codes) & 15) || (reinterpret_cast<uintptr_t>(x) & 15)) {
    set_error("qwen_b200_w8_digit_planes: rows %d / k %d must be positive multiples of 128, n_tokens %d in 1..65536, "
              "codes and x 16-byte aligned",
              rows, k, n_tokens);
    return kStatusInvalid;
  }
  if (!device_accessible(codes) || !device_accessible(x) || !device_accessible(acc) || !device_accessible(step)) {
    set_error("qwen_b200_w8_digit_planes: every buffer must be device (or managed) memory");
    return kStatusInvalid;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int8_t* planes = nullptr;
  float* steps = nullptr;
  const int spad = tgemm_pad(n_tokens);
  cudaError_t e = cudaMallocAsync(&planes, tgemm_plane_bytes(n_tokens, k), s);
  if (e == cudaSuccess) e = cudaMallocAsync(&steps, (size_t)spad * 4, s);
  const DigitPlanes dp{planes, steps, n_tokens, spad, k};
  if (e == cudaSuccess) e = tgemm_digitize(x, dp, s);
  if (e == cudaSuccess) e = tgemm_raw(reinterpret_cast<const uint8_t*>(codes), rows, dp, acc, s);
  if (e == cudaSuccess) e = cudaMemcpyAsync(step, steps, (size_t)n_tokens * 4, cudaMemcpyDeviceToDevice, s);
  if (planes) cudaFreeAsync(planes, s);
  if (steps) cudaFreeAsync(steps, s);
  if (e != cudaSuccess) {
    set_error("qwen_b200_w8_digit_planes: %s", cudaGetErrorString(e));
    return kStatusCuda;
  }
  return 0;
}

extern "C" int qwen_b200_prefill_attention(const float* q, const float* k_cache, const float* v_cache, int seq_len,
                                           float* context, int mode, void* stream) {
  using namespace qb;
  if (!q || !k_cache || !v_cache || !context || seq_len <= 0 || seq_len > kMaxSeq || (mode != 0 && mode != 1) ||
      (reinterpret_cast<uintptr_t>(q) & 15) || (reinterpret_cast<uintptr_t>(k_cache) & 15) ||
      (reinterpret_cast<uintptr_t>(context) & 15)) {
    set_error("qwen_b200_prefill_attention: null buffer, seq_len %d outside 1..%d, mode %d not 0/1, or q / k_cache / "
              "context not 16-byte aligned",
              seq_len, kMaxSeq, mode);
    return kStatusInvalid;
  }
  if (!device_accessible(q) || !device_accessible(k_cache) || !device_accessible(v_cache) ||
      !device_accessible(context)) {
    set_error("qwen_b200_prefill_attention: every buffer must be device (or managed) memory");
    return kStatusInvalid;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaSuccess;
  if (mode == 1) {
    e = launch_prefill_attention(q, k_cache, v_cache, seq_len, context, s);
  } else {
    void* scratch = nullptr;
    const size_t bytes = prefill_attn_tc_scratch_bytes(seq_len);
    e = cudaMallocAsync(&scratch, bytes, s);
    if (e == cudaSuccess) e = launch_prefill_attention_tc(q, k_cache, v_cache, seq_len, context, scratch, bytes, s);
    if (scratch) cudaFreeAsync(scratch, s);
  }
  if (e != cudaSuccess) {
    set_error("qwen_b200_prefill_attention: %s", cudaGetErrorString(e));
    return kStatusCuda;
  }
  return 0;
}

namespace qb {
namespace {
// Pairs of elements through the paired form (the one the attention softmax runs), element 2i in the first
// lane and 2i + 1 in the second, so both lanes are checked.
__global__ void approx_exp_kernel(const float* __restrict__ x, float* __restrict__ y, long long n) {
  const F2 nz = f2_negzero();
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; 2 * i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const bool two = 2 * i + 1 < n;
    float r0, r1;
    approx_exp_fast2(x[2 * i], two ? x[2 * i + 1] : 0.0f, r0, r1, nz);
    y[2 * i] = r0;
    if (two) y[2 * i + 1] = r1;
  }
}
}  // namespace
}  // namespace qb

extern "C" int qwen_b200_prefill_approx_exp(const float* x, float* y, long long n, void* stream) {
  using namespace qb;
  if (!x || !y || n < 0) {
    set_error("qwen_b200_prefill_approx_exp: null buffer or negative n");
    return kStatusInvalid;
  }
  if (!device_accessible(x) || !device_accessible(y)) {
    set_error("qwen_b200_prefill_approx_exp: every buffer must be device (or managed) memory");
    return kStatusInvalid;
  }
  if (n == 0) return 0;
  const long long blocks = std::min<long long>((n / 2 + 256) / 256, 148 * 16);
  approx_exp_kernel<<<(unsigned)blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(x, y, n);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("qwen_b200_prefill_approx_exp: %s", cudaGetErrorString(e));
    return kStatusCuda;
  }
  return 0;
}

extern "C" int qwen_b200_exact_expf(const float* x, float* y, long long n, void* stream) {
  using namespace qb;
  if (!x || !y || n < 0) {
    set_error("qwen_b200_exact_expf: null buffer or negative n");
    return kStatusInvalid;
  }
  if (!device_accessible(x) || !device_accessible(y)) {
    set_error("qwen_b200_exact_expf: every buffer must be device (or managed) memory");
    return kStatusInvalid;
  }
  if (n == 0) return 0;
  const cudaError_t e = exact::launch_expf(x, y, n, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    set_error("qwen_b200_exact_expf: %s", cudaGetErrorString(e));
    return kStatusCuda;
  }
  return 0;
}
