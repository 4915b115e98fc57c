// Persistent batch-1 decode step on the CUDA cores (decode_bs1.cu): every layer of one W8 decode step of a
// single sequence in one launch, with self-validating cross-CTA data words instead of completion counters.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "decode_stack.h"

namespace qb {
namespace bs1 {

// K segments per weight tile of each projection (q|k|v, o, gate|up, down); the tiles and the tiled weight
// image are the persistent tensor-core kernel's (decode_stack.h). o_proj segment s covers query heads
// 3s .. 3s + 2, the heads of one (KV group, half) attention merge group.
__host__ __device__ constexpr int nseg(int s) {
  return s == stack::kQkv ? 6 : s == stack::kO ? 4 : s == stack::kGu ? 1 : 12;
}
__host__ __device__ constexpr int seg_len(int s) { return (stack::nkb(s) + nseg(s) - 1) / nseg(s); }

// Words per layer of the packed split-K block: q|k|v rows at 0, o at 2048, down at 3584.
constexpr int kAccRows = 2048 + 1536 + 1536;
__host__ __device__ constexpr int acc_row(int s) { return s == stack::kQkv ? 0 : s == stack::kO ? 2048 : 3584; }
constexpr int kMergeGroups = kKvHeads * 2;  // attention merge groups: KV group x half of its query heads
constexpr int kGuItems = 140;
// The fewest CTAs a schedule fits on: every CTA holds at most one item of each projection, and down_proj has
// the most items. It is also the default: the step measured 0.6% faster on 144 CTAs than on all 148 SMs.
constexpr int kMinCtas = 12 * 12;
static_assert(stack::tiles(stack::kDown) * nseg(stack::kDown) == kMinCtas, "down_proj items");
static_assert(stack::tiles(stack::kGu) * nseg(stack::kGu) <= kMinCtas, "gate|up items");
static_assert(stack::tiles(stack::kQkv) * nseg(stack::kQkv) <= kMinCtas, "q|k|v items");
constexpr int kPartWords = 4 + kHeadDim;  // one attention chunk partial of one head: m, l, -, -, acc[128]

// Launch-global words (zero before the first launch; the kernel keeps exit_cnt and abort_flag zero between
// launches and advances epoch by one per launch).
struct Sync {
  stack::SyncWord exit_cnt;
  stack::SyncWord abort_flag;
  stack::SyncWord epoch;
};

// Cross-CTA data of one launch. Two kinds of self-validating 64-bit words:
//   packed split-K words (acc): bits 48..63 count the K segments added so far, bits 0..47 hold the sum of
//     (segment total + 2^43); a consumer reads the word until the count is complete. Launch parity
//     (epoch & 1) selects the half; each launch zeroes the other half for the next one.
//   tagged words (part, ctx, cmax, h, hmax, steps): bits 32..63 = ((epoch + 1) << 5 | layer), bits 0..31 =
//     an fp32 value; a consumer reads the word until its tag is the current one. Layer parity selects the
//     half.
struct Buffers {
  unsigned long long* acc;    // [2][kLayers][kAccRows]
  unsigned long long* part;   // [2][kHeads][max_chunks][kPartWords]
  unsigned long long* ctx;    // [2][kHidden] merged attention context
  unsigned long long* cmax;   // [2][kMergeGroups] max |ctx| of each merge group
  unsigned long long* h;      // [2][kInter]
  unsigned long long* hmax;   // [2][kGuItems]
  unsigned long long* steps;  // [kLayers][4] digit step of q|k|v (0), o (1) and down (3)
};
inline size_t acc_words() { return (size_t)2 * kLayers * kAccRows; }
inline size_t part_words(int max_chunks) { return (size_t)2 * kHeads * max_chunks * kPartWords; }
inline size_t ctx_words() { return (size_t)2 * kHidden; }
inline size_t cmax_words() { return (size_t)2 * kMergeGroups; }
inline size_t h_words() { return (size_t)2 * kInter; }
inline size_t hmax_words() { return (size_t)2 * kGuItems; }
inline size_t step_words() { return (size_t)kLayers * 4; }

struct Args {
  const uint8_t* wtiles;     // [28][stack::kLayerTileBytes] pre-swizzled int8 weight units
  const LayerDev* layers;    // [28] device array: scales, biases, norm weights
  const uint16_t* embed;     // fp16 [vocab][1536]
  const int* tokens;         // [1]
  const int* pos;            // [1]
  const int* seq;            // [1]
  const float* rope_cos;     // [positions][64]
  const float* rope_sin;
  float* kv_pool;            // paged KV pool
  const int* page_table;
  int max_pages;
  float* y0;                 // layer outputs, ping-pong [1][1536]; the last layer's is read by the LM head
  float* y1;
  float* dump;               // optional [28][1][1536] copies of the layer outputs
  Buffers buf;
  int max_chunks;            // 64-key chunks the part buffer holds per head
  Sync* sync;
  const uint32_t* item_off;  // [ctas + 1]
  const stack::Item* items;
  // optional [ctas][28][stack::kTraceSlots] stamps: the stage slots of decode_stack.h (global timer, ns), and
  // for the gate|up dot products kTraceUnit + 0/1/2 = global timer at units 0, 8 and the last, + 3/4/5 = SM
  // clock at the same units, + 6 + w = SM clock of worker warp w at the loop's end
  unsigned long long* trace;
  int ring;                  // weight stages in flight per CTA (2..9)
};

// Static per-layer work split over `ctas` CTAs (at most one item per projection and CTA, balanced by 16 KB
// weight units streamed); empty when the items of one projection outnumber the CTAs.
stack::Schedule build_schedule(int ctas);

// Launch over `ctas` CTAs (cooperative: all resident).
cudaError_t launch_decode_bs1(const Args& a, int ctas, cudaStream_t s);
size_t decode_bs1_smem();
unsigned decode_bs1_kernel_error(bool reset);

}  // namespace bs1
}  // namespace qb
