// Parameter blocks and kernel declarations shared by the .cu files.
#pragma once

#include <cstdint>
#include <utility>
#include <cuda_runtime.h>

#include "moe_shapes.cuh"

namespace moe {

// Routing methods, in the numbering of flashinfer's RoutingMethodType; this
// operator's own is kRouteDeepSeekV3 (route_token).
enum RouteMethod : int {
  kRouteDefault = 0,            // softmax -> top-k
  kRouteRenormalize = 1,        // top-k -> softmax over the picks
  kRouteDeepSeekV3 = 2,         // sigmoid + bias, group-limited top-8 (this operator)
  kRouteLlama4 = 3,             // top-1 -> sigmoid
  kRouteRenormalizeNaive = 4,   // softmax -> top-k -> renormalise
  kRouteTopK = 5,               // top-k, uniform weights
  // Not a routing rule: the selections come from the caller
  // (moe_b200_run_routed), e.g. the rows an all-to-all dispatch delivered.
  kRouteGiven = 6,
};
// Expert id of the unused selection slots (k >= top_k): never a local expert.
constexpr int kNoExpert = -(1 << 30);

struct RouteParams {
  const float* logits;      // [T, 256] fp32
  const void* bias;         // [256] bf16 or fp32 (may be null for methods other than DeepSeek-V3)
  int bias_is_fp32;
  int num_tokens;           // T
  float routed_scaling_factor;
  int local_expert_offset;
  int32_t* topk_idx;        // [T, 8] global expert ids, best first
  float* topk_w;            // [T, 8]
  uint16_t* out;            // [T, 7168] bf16 output: rows of tokens with no local pick are zeroed (or null)
  int method;               // RouteMethod
  int top_k;                // selections per token, 1..8 (8 for DeepSeek-V3, 1 for Llama4)
  const int32_t* given_idx; // kRouteGiven: [T, top_k] global expert ids (anything else for none)
  const float* given_w;     // kRouteGiven: [T, top_k] final weights
};

struct PermuteParams {
  const int32_t* topk_idx;  // [T, 8]
  const float* topk_w;      // [T, 8]
  int* counts;              // [32] assignments per local expert (written)
  int* chunk_counts;        // [ceil(T/kPermChunk), 33] per-chunk expert counts + touched tokens (multi-CTA path)
  uint32_t* status;         // device status word (cleared)
  int* sched;               // [4] GEMM unit counters (cleared)
  int num_tokens;
  int local_expert_offset;
  int* seg_off;             // [33] segment starts (multiples of kSegAlign)
  int32_t* perm_tok;        // [cap] token of each permuted row, -1 for padding
  float* perm_w;            // [cap] routing weight of each permuted row
  // Combine rows: only tokens with at least one local pick ("touched") get a
  // row of the fp32 combine buffer, numbered in token order.
  int32_t* tok_slot;        // [T] combine row of each token, -1 if untouched
  int32_t* perm_row;        // [cap] combine row of each permuted row, -1 for padding
  int* n_touched;           // [1] number of touched tokens
  int32_t* slot_tok;        // [T] token of each combine row (first n_touched entries)
};

struct GatherParams {
  const int* seg_off;       // [33]
  const int* n_touched;     // [1] rows of y_acc in use
  const int32_t* perm_tok;  // [cap]
  const uint8_t* hidden;    // [T, 7168] e4m3
  const float* hidden_scale;  // [56, T]
  int num_tokens;
  int cap;
  uint8_t* a_perm;          // [cap, 7168] e4m3
  float* sa_perm;           // [56, cap]
  float* y_acc;             // [n_touched, 7168] cleared
  const int* counts;        // [32] (token-major plans, for the GEMM1 K-split rule)
  float* g1_acc;            // token-major GEMM1 K-split sums, cleared when the split is on; or null
};

// Token-major GEMMs of batches with few token tiles: when GEMM1 has fewer
// than kTmSplitUnits (expert, 128-block, 128-token tile) units, it splits K
// into tm_gemm1_splits() parts whose fp32 sums meet in g1_acc, and GEMM2
// applies SwiGLU (grid-wide, before its first C tile) instead of GEMM1's
// epilogue. Fewer than 148 units means at most 9 token tiles (1,152 pairs)
// and at most 1,152 + 9 x 15 padded rows, within kTmSplitRows.
constexpr int kTmSplitUnits = 148;
// Tokens (and threads) per CTA of the multi-CTA permutation (T > 1024).
constexpr int kPermChunk = 256;
constexpr int kTmSplitRows = 1664;

__device__ __forceinline__ int tm_gemm1_splits(int units) {
  if (units <= 0 || units >= kTmSplitUnits) return 1;
  if (4 * units < kTmSplitUnits) return 8;   // 7 of the 56 K blocks per unit
  return 2 * units < kTmSplitUnits ? 4 : 2;
}

// Decode batches (num_tokens <= kDecodeMaxTokens) use a dedicated front end:
// one 8-CTA cluster does routing, permutation, the permuted row copy and the
// clears the K-split GEMM1 needs.
constexpr int kDecodeMaxTokens = 64;
constexpr int kDecodeClusterCtas = 8;

struct DecodeFrontParams {
  int* counts;              // [32] assignments per local expert (written)
  int* seg_off;             // [33] padded segment starts (written)
  int32_t* perm_tok;        // [cap] token of each permuted row, -1 for padding
  float* perm_w;            // [cap] routing weight of each permuted row
  uint32_t* status;         // device status word (cleared)
  int* sched;               // [4] GEMM unit counters (cleared)
  float* g1_acc;            // [cap, 4096] rows of valid (token, expert) pairs cleared
  const uint8_t* hidden;    // [T, 7168] e4m3
  const float* hidden_scale;  // [56, T]
  const uint16_t* hidden_bf16;  // [T, 7168] bf16 when set: rows are quantised while copied (hidden unused)
  uint8_t* a_perm;          // [cap, 7168] valid rows copied from hidden
  float* sa_perm;           // [56, cap] their block scales
  int cap;
  int local_expert_offset;
};

// The three grouped-GEMM flavours built from one kernel template.
enum GemmKind : int {
  kGemm1Fused = 0,  // GEMM1 over the full K, SwiGLU + hi/lo e4m3 split in the epilogue
  kGemm1Split = 1,  // decode GEMM1 over a K slice, fp32 red.add into g1_acc
  kGemm2 = 2,       // GEMM2 (hi + lo operands), weighted fp32 red.add into y_acc
  kGemm2Wide = 3,   // GEMM2 over two 128-row W2 blocks per tile (M = 256)
};

struct GemmParams {
  const int* seg_off;       // [33] padded segment starts
  const int* counts;        // [32] valid rows per segment
  const int32_t* perm_tok;  // [cap]
  const int32_t* perm_row;  // [cap] combine row of each permuted row (GEMM2 epilogues)
  const float* perm_w;      // [cap]
  const float* act_scale;   // GEMM1: sa_perm [56, cap]; GEMM2: c_scale [16, cap]
  const float* w_scale;     // GEMM1: [32, 32, 56]; GEMM2: [32, 56, 16]
  int num_tokens;           // T
  int cap;                  // row capacity of the permuted buffers (8T)
  int splits;               // K slices per output tile
  int tail_splits;          // K slices of the last tail_experts active experts (<= splits: off)
  int tail_experts;
  uint8_t* c_hi;            // [cap, 2048] e4m3
  uint8_t* c_lo;            // [cap, 2048] e4m3
  float* c_scale;           // [16, cap] written by kGemm1Fused / swiglu_quant
  float* g1_acc;            // [cap, 4096] fp32 (kGemm1Split)
  float* y_acc;             // [T, 7168] fp32 (kGemm2; kGemm1Split clears it)
  uint32_t* status;         // device status word
  int* sched;               // this GEMM's unit counter (cleared by the permutation)
  // Decode GEMM2 only: when g1_acc is set, the CTAs first convert the K-split
  // GEMM1 sums into C (SwiGLU, hi/lo e4m3) and count themselves on grid_sync
  // (cleared by the front end); no C tile is loaded before all have.
  int* grid_sync;
};

// Launches `kern` on `stream`; with `dependent` set the launch carries the
// programmatic-stream-serialization attribute, so the kernel may start while
// its predecessor finishes (the kernel itself must griddepcontrol.wait before
// reading the predecessor's results).
template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                          bool dependent, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = dependent ? attr : nullptr;
  cfg.numAttrs = dependent ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

__global__ void route_kernel(RouteParams p);
__global__ void permute_kernel(PermuteParams p);
__global__ void permute_count_kernel(PermuteParams p);
__global__ void permute_place_kernel(PermuteParams p);
__global__ void gather_rows_kernel(GatherParams p);
__global__ void quantize_hidden_kernel(const uint16_t* hidden_bf16, int num_tokens, uint8_t* hidden_fp8,
                                       float* hidden_scale);
__global__ void finalize_kernel(const float* y_acc, const int32_t* slot_tok, const int* n_touched, uint16_t* out,
                                int num_tokens);
// kBf16: dp.hidden_bf16 rows are quantised while copied; otherwise e4m3 rows copied.
template <bool kBf16>
__global__ void route_permute_decode_kernel(RouteParams rp, DecodeFrontParams dp);

}  // namespace moe
