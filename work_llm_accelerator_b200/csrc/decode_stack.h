// Persistent decode kernel (decode_stack.cu): every layer of one W8 decode step in a single launch.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <vector>

#include "qwen_kernels.cuh"

namespace qb {
namespace stack {

// Projection stages of a layer, in execution order (attention runs between kQkv and kO).
enum : int { kQkv = 0, kO = 1, kGu = 2, kDown = 3, kNumProj = 4 };
// Completion counters per layer: one per projection stage plus attention.
enum : int { kDoneQkv = 0, kDoneAttn = 1, kDoneO = 2, kDoneGu = 3, kDoneDown = 4, kDoneSlots = 5 };

// Weight tiles (128 rows), 128-byte K blocks per tile and K segments per tile of each stage.
// q|k|v: one tile per head (12 q, 2 k, 2 v); gate|up: tile j = gate rows 64j.. and up rows 64j..
__host__ __device__ constexpr int tiles(int s) { return s == kQkv ? 16 : s == kO ? 12 : s == kGu ? 140 : 12; }
__host__ __device__ constexpr int nkb(int s) { return s == kDown ? 70 : 12; }
__host__ __device__ constexpr int split(int s) { return s == kQkv ? 6 : s == kO ? 12 : s == kGu ? 1 : 12; }
__host__ __device__ constexpr int seg_blocks(int s) { return (nkb(s) + split(s) - 1) / split(s); }
// first 16 KB unit of each stage in a layer's tiled image (tile-major, K blocks contiguous)
__host__ __device__ constexpr int unit_base(int s) {
  return s == kQkv ? 0 : s == kO ? 16 * 12 : s == kGu ? 16 * 12 + 12 * 12 : 16 * 12 + 12 * 12 + 140 * 12;
}
constexpr int kUnitsPerLayer = 16 * 12 + 12 * 12 + 140 * 12 + 12 * 70;  // 2856
constexpr uint64_t kLayerTileBytes = (uint64_t)kUnitsPerLayer * 16384;   // 46.8 MB
// Work items of a stage (every K segment of every tile): the stage's completion count.
__host__ __device__ constexpr int stage_items(int s) { return tiles(s) * split(s); }
// Split-K integer accumulators of the q|k|v, o and down projections, consumed directly by the next step:
// [parity (layer & 1)][token 4][digit 3][kAccRows]; rows of q|k|v at 0, o at 2048, down at 3584.
constexpr int kAccRows = 2048 + 1536 + 1536;
__host__ __device__ constexpr int acc_row_base(int s) { return s == kQkv ? 0 : s == kO ? 2048 : 3584; }
constexpr size_t kAccInts = (size_t)2 * 4 * 3 * kAccRows;

// One work item: K blocks [kb0, kb1) of one tile; its digit operand starts at block `dslot` of the CTA's
// digit buffer for the stage.
struct Item {
  uint16_t tile;
  uint8_t stage;
  uint8_t kb0, kb1;
  uint8_t dslot;
  uint16_t seg;
};
static_assert(sizeof(Item) == 8, "item packing");

// One synchronisation word per 128-byte line, so that polling one counter does not queue behind atomics
// on its neighbours.
struct alignas(128) SyncWord {
  unsigned v;
  unsigned pad[31];
};

// Device-side synchronisation words (zero between launches; the kernel leaves them zero).
struct SyncWords {
  SyncWord done[kLayers][kDoneSlots];
  SyncWord hmax[kLayers];      // .pad[0..3]: max |h| per token (float bits), for the down projection's step
  SyncWord attn_cnt[4][4];     // per token, KV group x head half
  SyncWord exit_cnt;
  SyncWord abort_flag;
};

// Static per-layer work split over `ctas` CTAs: items of CTA c are items[off[c] .. off[c + 1]), in stage
// order. Balanced by 16 KB units streamed per CTA.
struct Schedule {
  std::vector<uint32_t> off;
  std::vector<Item> items;
  int max_units = 0;
};
Schedule build_schedule(int ctas);

struct Args {
  const uint8_t* wtiles;      // [28][kLayerTileBytes] pre-swizzled int8 weight units
  const LayerDev* layers;     // [28] device array: scales, biases, norm weights (and DDR weights, unused)
  const uint16_t* embed;      // fp16 [vocab][1536]
  const int* tokens;          // [nt]
  const int* pos;             // [nt]
  const int* seq;             // [nt]
  int nt;
  const float* rope_cos;      // [positions][64]
  const float* rope_sin;
  float* kv_pool;             // paged KV pool
  const int* page_table;
  int max_pages;
  float* y0;                  // layer outputs, ping-pong [nt][1536]
  float* y1;
  float* q;                   // [nt][1536]
  float* ctx;                 // [nt][1536]
  float* a;                   // [nt][1536] attention block output
  float* h;                   // [nt][8960]
  float* dump;                // optional [28][nt][1536] copies of the layer outputs
  float* attn_part;           // attention chunk partials
  int attn_max_chunks;
  int* acc;                   // [kAccInts] split-K integer accumulators (zero before their layer's use)
  float* steps;               // [28][4][4] digit step per layer, projection and token
  SyncWords* sync;
  const uint32_t* item_off;   // [ctas + 1]
  const Item* items;
  unsigned long long* trace;  // optional [ctas][28][kTraceSlots] global-timer stamps (ns), see kTrace*
  int ring;                   // weight stages in flight per CTA (2..9)
};

// Timeline slots of the optional trace, per CTA and layer (stage index: 0 q|k|v, 1 attention, 2 o,
// 3 gate|up, 4 down):
//   kTraceWait + i   workers: inputs of stage i available (after the completion-counter wait)
//   kTraceBuilt + i  workers: digits of stage i in shared memory (attention: chunks done)
//   kTraceDone + i   workers: every epilogue of stage i done
//   kTraceIssue + s  producer: first weight unit of projection s issued
//   kTraceMma + s    MMA issuer: last MMA of projection s committed
//   kTraceAcc + j    workers: accumulator of the CTA's last item of split stage j (0 q|k|v, 1 o, 2 down) ready
//   kTraceArrived + j   workers: that item's split-K partial added and signalled
//   kTraceMmaStart + s  MMA issuer: digits of projection s seen, first MMA about to issue
//   kTraceAttnQ      workers: attention inputs (q, new K/V row, history) in shared memory
//   kTraceAttnPart   workers: attention chunk partial written and counted
//   kTraceAttnMerge  workers: attention chunks merged (last chunk only)
//   kTraceUnit + u   MMA issuer: unit u (< 12) of the CTA's gate|up item present in shared memory
//   kTraceUnit + 12 + u   MMA issuer: unit u (< 12) of the CTA's down item present in shared memory
constexpr int kTraceSlots = 64;
constexpr int kTraceUnit = 40;
constexpr int kTraceWait = 0, kTraceBuilt = 5, kTraceDone = 10, kTraceIssue = 16, kTraceMma = 20, kTraceAcc = 24,
              kTraceArrived = 27, kTraceMmaStart = 30, kTraceAttnQ = 34, kTraceAttnPart = 35, kTraceAttnMerge = 36;

// Floats of the attention chunk-partial scratch for `nt` tokens and `max_chunks` 64-key chunks.
inline size_t attn_part_floats(int nt, int max_chunks) { return (size_t)nt * kHeads * max_chunks * (4 + kHeadDim); }

// Launch over `ctas` CTAs (cooperative: all resident). Requires wbits 8 weights in the tiled layout.
cudaError_t launch_decode_stack(const Args& a, int ctas, cudaStream_t s);
// Convert one layer's DDR-image int8 weights into the tiled layout.
cudaError_t launch_tile_layer(const LayerDev& L, uint8_t* dst, cudaStream_t s);
// Dynamic shared memory of one CTA.
size_t decode_stack_smem();
unsigned decode_stack_kernel_error(bool reset);

}  // namespace stack
}  // namespace qb
