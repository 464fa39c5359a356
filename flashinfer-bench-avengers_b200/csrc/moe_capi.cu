// C ABI of the fused MoE layer (declared in include/moe_b200.h).
//
// Host orchestration replacing solution/cuda/main.cpp:13-142. Differences
// by design:
//   * destination-passing: output and workspace come from the caller, no
//     allocation inside the call;
//   * no host synchronisation: expert segment sizes never leave the device
//     (the reference copies counts to the host, main.cpp:92-103), so a call
//     can be captured in a CUDA graph;
//   * one launch per stage for all 32 experts (the reference loops over
//     experts on the host for GEMM2, main.cpp:112-139).
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <algorithm>
#include <cstring>
#include <mutex>

#include "../../include/moe_b200.h"
#include "gemm_sm100.h"
#include "moe_kernels.cuh"
#include "moe_shapes.cuh"

namespace moe {
namespace {

constexpr size_t kAlign = 256;

size_t align_up(size_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

// Execution plan for one call, a function of T only (so workspace size and
// launch shapes are known without reading device data).
struct Plan {
  bool decode;     // T <= kDecodeMaxTokens: single-CTA front end, stream-K GEMMs
  int g1_bn;
  int g2_bn;
  bool g2_wide;    // two W2 row blocks per GEMM2 tile
  bool token_major;  // prefill: token-major GEMMs (gemm_tm_sm100.cu)
};

// K splits of the decode GEMMs (work units per (expert, row block)). Up to
// MOE_B200_DECODE_SMALL_T tokens a few active experts give GEMM1 fewer
// units than SMs, and it splits MOE_B200_DECODE_G1_SPLITS_SMALL ways
// (measured on one box: 4 tokens 44.7 -> 43.0 us, 1 token 43.6 -> 43.0 us;
// at 16 tokens the two are equal, at 64 tokens 4 splits are 4 us faster).
#ifndef MOE_B200_DECODE_G1_SPLITS
#define MOE_B200_DECODE_G1_SPLITS 4
#endif
#ifndef MOE_B200_DECODE_SMALL_T
#define MOE_B200_DECODE_SMALL_T 8
#endif
#ifndef MOE_B200_DECODE_G1_SPLITS_SMALL
#define MOE_B200_DECODE_G1_SPLITS_SMALL 8
#endif
// The last MOE_B200_DECODE_TAIL_EXPERTS active experts split finer, so the
// final wave of work units is shorter (measured on one box against no tail
// splits: GEMM1 8 ways, T = 16 98.5 -> 95.9 us; GEMM2 4 ways as well, T = 64
// 137.7 -> 134.8 us, but 2 us slower at T <= 4, hence only above
// MOE_B200_DECODE_G2_TAIL_MIN_T tokens).
#ifndef MOE_B200_DECODE_TAIL_EXPERTS
#define MOE_B200_DECODE_TAIL_EXPERTS 2
#endif
#ifndef MOE_B200_DECODE_G1_TAIL_SPLITS
#define MOE_B200_DECODE_G1_TAIL_SPLITS 8
#endif
#ifndef MOE_B200_DECODE_G2_TAIL_SPLITS
#define MOE_B200_DECODE_G2_TAIL_SPLITS 4
#endif
#ifndef MOE_B200_DECODE_G2_TAIL_MIN_T
#define MOE_B200_DECODE_G2_TAIL_MIN_T 16
#endif
#ifndef MOE_B200_DECODE_G2_SPLITS
#define MOE_B200_DECODE_G2_SPLITS 2
#endif

// From this many tokens per call the prefill (token-major) GEMMs are used.
constexpr int64_t kTokenMajorMinTokens = 512;

Plan choose_plan(int64_t T) {
  Plan p{};
  if (T <= kDecodeMaxTokens) {
    // Both GEMMs stream 16-token column groups against 256 weight rows
    // (six 32 KB weight stages in flight per SM); GEMM1 splits K 4 ways.
    p.decode = true;
    p.g1_bn = 16;
    p.g2_bn = 16;
    p.g2_wide = true;
  } else {
    p.decode = false;
    p.g1_bn = 64;
    p.g2_bn = 64;
    p.g2_wide = false;
    p.token_major = T >= kTokenMajorMinTokens;
  }
  return p;
}

struct Layout {
  moe_b200_workspace_layout l;
};

// `picks` is the most local picks a token can have: 8 for the routing rules,
// top_k when the caller gives the routing (moe_b200_run_routed).
moe_b200_workspace_layout make_layout(int64_t T, int picks = kTopK) {
  moe_b200_workspace_layout l;
  std::memset(&l, 0, sizeof(l));
  const Plan plan = choose_plan(T);
  // Permuted-row capacity: every (token, local expert) pair, the padding of
  // 32 segments to kSegAlign rows, and one 128-row tile of slack so tile
  // reads that run past the last segment stay inside the buffers.
  const size_t cap = (static_cast<size_t>(T) * picks + kSegAlign - 1) / kSegAlign * kSegAlign +
                     kExpertsLocal * kSegAlign + 128;
  size_t off = 0;
  l.counts = off;
  l.status = off + kExpertsLocal * sizeof(int);
  l.sched = l.status + 16;
  l.n_touched = l.sched + 4 * sizeof(int);
  off = align_up(l.n_touched + sizeof(int));
  l.seg_off = off;
  off = align_up(off + (kExpertsLocal + 1) * sizeof(int));
  l.chunk_counts = off;
  off = align_up(off + static_cast<size_t>((T + kPermChunk - 1) / kPermChunk) * (kExpertsLocal + 1) * sizeof(int));
  // the routing writes 8 slots per token whatever `picks` is (with 8 picks
  // cap is larger than 8 T, so this is cap)
  const size_t topk_slots = std::max(cap, static_cast<size_t>(T) * kTopK);
  l.topk_idx = off;
  off = align_up(off + topk_slots * sizeof(int32_t));
  l.topk_w = off;
  off = align_up(off + topk_slots * sizeof(float));
  l.perm_tok = off;
  off = align_up(off + cap * sizeof(int32_t));
  l.perm_w = off;
  off = align_up(off + cap * sizeof(float));
  l.perm_row = off;
  off = align_up(off + cap * sizeof(int32_t));
  l.tok_slot = off;
  off = align_up(off + static_cast<size_t>(T) * sizeof(int32_t));
  l.a_perm = off;
  off = align_up(off + cap * kHidden);
  l.sa_perm = off;
  off = align_up(off + cap * kHiddenBlocks * sizeof(float));
  l.c_hi = off;
  off = align_up(off + cap * kInter);
  l.c_lo = off;
  off = align_up(off + cap * kInter);
  l.c_scale = off;
  off = align_up(off + cap * kInterBlocks * sizeof(float));
  l.y_acc = off;
  off = align_up(off + static_cast<size_t>(T) * kHidden * sizeof(float));
  if (plan.decode) {
    l.g1_acc = off;
    off = align_up(off + cap * kGemm1Out * sizeof(float));
  } else if (plan.token_major) {
    // K-split GEMM1 sums of batches with few token tiles (kTmSplitRows rows)
    l.g1_acc = off;
    off = align_up(off + static_cast<size_t>(kTmSplitRows) * kGemm1Out * sizeof(float));
  }
  l.slot_tok = off;
  off = align_up(off + static_cast<size_t>(T) * sizeof(int32_t));
  if (!plan.decode) {
    // e4m3 copy of bf16 hidden states (moe_b200_run_bf16_hidden), one row per token
    l.hidden_q = off;
    off = align_up(off + static_cast<size_t>(T) * kHidden);
    l.hidden_qs = off;
    off = align_up(off + static_cast<size_t>(T) * kHiddenBlocks * sizeof(float));
  }
  l.total_bytes = off;
  l.cap_rows = static_cast<int64_t>(cap);
  return l;
}

// ---------------------------------------------------------------- driver
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
    }
  });
  return fn;
}

// 2-D byte matrix [rows, inner] with row pitch `inner`, 128-byte swizzle.
bool encode_u8_2d(CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows,
                  uint32_t box_inner, uint32_t box_rows) {
  EncodeTiledFn fn = get_encode_fn();
  if (fn == nullptr) return false;
  const cuuint64_t dims[2] = {inner, rows};
  const cuuint64_t strides[1] = {inner};
  const cuuint32_t box[2] = {box_inner, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// ---------------------------------------------------------------- device
struct DeviceInfo {
  int checked = 0;
  int ok = 0;
  int sm_count = 0;
};

constexpr int kMaxDevices = 64;
DeviceInfo g_dev[kMaxDevices];
std::mutex g_dev_mu;

int current_device_info(DeviceInfo* out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return MOE_B200_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return MOE_B200_ERR_UNSUPPORTED_DEVICE;
  std::lock_guard<std::mutex> lock(g_dev_mu);
  DeviceInfo& d = g_dev[dev];
  if (!d.checked) {
    int major = 0, minor = 0, sms = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
      return MOE_B200_ERR_CUDA;
    }
    d.ok = (major == 10 && minor == 0) ? 1 : 0;
    d.sm_count = sms;
    d.checked = 1;
  }
  *out = d;
  return d.ok ? MOE_B200_OK : MOE_B200_ERR_UNSUPPORTED_DEVICE;
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

int64_t div_up(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Upper bound on the number of work units of a grouped GEMM, from T only.
int grid_for(int64_t T, int bn, int row_blocks, int splits, int sm_count) {
  const int64_t tiles_a = div_up(T * kTopK, bn) + kExpertsLocal;
  const int64_t tiles_b = static_cast<int64_t>(kExpertsLocal) * div_up(T, bn);
  const int64_t units = (tiles_a < tiles_b ? tiles_a : tiles_b) * row_blocks * splits;
  return static_cast<int>(units < sm_count ? units : sm_count);
}

// Selections supplied by the caller (moe_b200_run_routed): [T, top_k]
// global expert ids and final weights; null for the routing rules.
struct GivenPicks {
  const int32_t* idx = nullptr;
  const float* w = nullptr;
};

int launch_route(const float* logits, const void* bias, int bias_dtype, int T, float rsf,
                 int local_off, int32_t* topk_idx, float* topk_w, uint16_t* out, int method, int top_k,
                 cudaStream_t s, const GivenPicks& given = GivenPicks{}) {
  RouteParams rp;
  rp.given_idx = given.idx;
  rp.given_w = given.w;
  rp.logits = logits;
  rp.bias = bias;
  rp.bias_is_fp32 = bias_dtype == MOE_B200_BIAS_FP32 ? 1 : 0;
  rp.num_tokens = T;
  rp.routed_scaling_factor = rsf;
  rp.local_expert_offset = local_off;
  rp.topk_idx = topk_idx;
  rp.topk_w = topk_w;
  rp.out = out;
  rp.method = method;
  rp.top_k = top_k;
  // The first kernel of a call is launched without the dependent-launch
  // attribute, so it starts only after all earlier work on the stream.
  route_kernel<<<static_cast<unsigned>(div_up(T, 8)), 256, 0, s>>>(rp);
  return cudaGetLastError() == cudaSuccess ? MOE_B200_OK : MOE_B200_ERR_CUDA;
}

thread_local cudaEvent_t t_stage_events[MOE_B200_NUM_STAGE_EVENTS];
thread_local bool t_stage_events_on = false;

// While the stream is being captured the marks are external event records,
// so they also fire when the captured CUDA graph is replayed.
void mark_stage(int i, cudaStream_t s) {
  if (!t_stage_events_on) return;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(s, &cs) != cudaSuccess) return;
  if (cs == cudaStreamCaptureStatusActive)
    cudaEventRecordWithFlags(t_stage_events[i], s, cudaEventRecordExternal);
  else
    cudaEventRecord(t_stage_events[i], s);
}

// Decode plan (T <= kDecodeMaxTokens): four launches,
//   route_permute_decode (one 8-CTA cluster: routing, permutation, permuted
//     row copy, clears of the unit counters and of the g1_acc rows)
//   -> K-split GEMM1 (red.add into g1_acc; also clears y_acc)
//   -> GEMM2: first C = silu(gate) * up as the hi/lo e4m3 pair from the
//      GEMM1 sums (all CTAs, then a grid-wide count before any C tile is
//      loaded; W2 tiles stream meanwhile), then two W2 blocks per tile, K
//      split 2 ways, red.add into y_acc
//   -> finalize (bf16).
int run_decode(const float* routing_logits, const void* routing_bias, int routing_bias_dtype, int method,
               int top_k, const void* hidden_states, const float* hidden_states_scale, bool hidden_bf16,
               const void* gemm1_weights,
               const float* gemm1_weights_scale, const void* gemm2_weights,
               const float* gemm2_weights_scale, int local_off, float rsf, int T, void* output,
               uint8_t* ws, const moe_b200_workspace_layout& l, const DeviceInfo& di, cudaStream_t s,
               const GivenPicks& given = GivenPicks{}) {
  // Four K slices (units of 0.46 MB) keep the SMs evenly loaded; more slices
  // add red.add and unit-switch overhead unless few experts are active.
  const int g1_splits = T <= MOE_B200_DECODE_SMALL_T ? MOE_B200_DECODE_G1_SPLITS_SMALL : MOE_B200_DECODE_G1_SPLITS;
  constexpr int kG2Splits = MOE_B200_DECODE_G2_SPLITS;
  constexpr int kBN = 16;
  const int cap = static_cast<int>(l.cap_rows);
  int* counts = reinterpret_cast<int*>(ws + l.counts);
  uint32_t* status = reinterpret_cast<uint32_t*>(ws + l.status);
  int* sched = reinterpret_cast<int*>(ws + l.sched);
  int* seg_off = reinterpret_cast<int*>(ws + l.seg_off);
  int32_t* perm_tok = reinterpret_cast<int32_t*>(ws + l.perm_tok);
  float* perm_w = reinterpret_cast<float*>(ws + l.perm_w);
  uint8_t* c_hi = ws + l.c_hi;
  uint8_t* c_lo = ws + l.c_lo;
  float* c_scale = reinterpret_cast<float*>(ws + l.c_scale);
  float* y_acc = reinterpret_cast<float*>(ws + l.y_acc);
  float* g1_acc = reinterpret_cast<float*>(ws + l.g1_acc);

  uint8_t* a_perm = ws + l.a_perm;
  float* sa_perm = reinterpret_cast<float*>(ws + l.sa_perm);
  CUtensorMap tm_aperm, tm_w13, tm_w2, tm_chi, tm_clo;
  if (!encode_u8_2d(&tm_aperm, a_perm, kHidden, cap, 128, kBN) ||
      !encode_u8_2d(&tm_w13, gemm1_weights, kHidden, static_cast<uint64_t>(kExpertsLocal) * kGemm1Out,
                    128, 128) ||
      !encode_u8_2d(&tm_w2, gemm2_weights, kInter, static_cast<uint64_t>(kExpertsLocal) * kHidden, 128,
                    128) ||
      !encode_u8_2d(&tm_chi, c_hi, kInter, cap, 128, kBN) ||
      !encode_u8_2d(&tm_clo, c_lo, kInter, cap, 128, kBN))
    return MOE_B200_ERR_DRIVER;

  mark_stage(0, s);
  mark_stage(1, s);
  RouteParams rp;
  rp.logits = routing_logits;
  rp.bias = routing_bias;
  rp.bias_is_fp32 = routing_bias_dtype == MOE_B200_BIAS_FP32 ? 1 : 0;
  rp.num_tokens = T;
  rp.routed_scaling_factor = rsf;
  rp.local_expert_offset = local_off;
  rp.topk_idx = reinterpret_cast<int32_t*>(ws + l.topk_idx);
  rp.topk_w = reinterpret_cast<float*>(ws + l.topk_w);
  rp.out = nullptr;
  rp.method = method;
  rp.top_k = top_k;
  rp.given_idx = given.idx;
  rp.given_w = given.w;
  DecodeFrontParams dp;
  dp.counts = counts;
  dp.seg_off = seg_off;
  dp.perm_tok = perm_tok;
  dp.perm_w = perm_w;
  dp.status = status;
  dp.sched = sched;
  dp.g1_acc = g1_acc;
  dp.hidden = hidden_bf16 ? nullptr : static_cast<const uint8_t*>(hidden_states);
  dp.hidden_scale = hidden_bf16 ? nullptr : hidden_states_scale;
  dp.hidden_bf16 = hidden_bf16 ? static_cast<const uint16_t*>(hidden_states) : nullptr;
  dp.a_perm = a_perm;
  dp.sa_perm = sa_perm;
  dp.cap = cap;
  dp.local_expert_offset = local_off;
  // First kernel of the call: no dependent-launch attribute. The cluster
  // shape is compiled into the kernel.
  if (hidden_bf16)
    route_permute_decode_kernel<true><<<kDecodeClusterCtas, 256, 0, s>>>(rp, dp);
  else
    route_permute_decode_kernel<false><<<kDecodeClusterCtas, 256, 0, s>>>(rp, dp);
  if (cudaGetLastError() != cudaSuccess) return MOE_B200_ERR_CUDA;
  mark_stage(2, s);
  mark_stage(3, s);

  GemmParams g1;
  std::memset(&g1, 0, sizeof(g1));
  g1.seg_off = seg_off;
  g1.counts = counts;
  g1.perm_tok = perm_tok;
  g1.perm_row = perm_tok;   // decode: y_acc has one row per token
  g1.perm_w = perm_w;
  g1.act_scale = sa_perm;
  g1.w_scale = gemm1_weights_scale;
  g1.num_tokens = T;
  g1.cap = cap;
  g1.splits = g1_splits;
  g1.tail_splits = MOE_B200_DECODE_G1_TAIL_SPLITS;
  g1.tail_experts = MOE_B200_DECODE_TAIL_EXPERTS;
  g1.c_hi = c_hi;
  g1.c_lo = c_lo;
  g1.c_scale = c_scale;
  g1.g1_acc = g1_acc;
  g1.y_acc = y_acc;
  g1.status = status;
  g1.sched = sched;
  // The front end releases GEMM1 right after writing and fencing the segment
  // table, so GEMM1 reads it and starts streaming weight tiles while the
  // front end still copies the permuted rows (early tables).
  const int grid1 = grid_for(T, kBN, kInterBlocks, g1_splits, di.sm_count);
  if (launch_moe_gemm(kGemm1Split, kBN, tm_w13, tm_aperm, tm_aperm, g1, grid1, true, s) != cudaSuccess)
    return MOE_B200_ERR_CUDA;
  mark_stage(4, s);

  GemmParams g2 = g1;
  g2.act_scale = c_scale;
  g2.w_scale = gemm2_weights_scale;
  g2.splits = kG2Splits;
  g2.tail_splits = T > MOE_B200_DECODE_G2_TAIL_MIN_T ? MOE_B200_DECODE_G2_TAIL_SPLITS : 0;
  g2.tail_experts = MOE_B200_DECODE_TAIL_EXPERTS;
  g2.sched = sched + 1;
  g2.grid_sync = sched + 2;
  const int grid2 = grid_for(T, kBN, kHiddenBlocks / 2, kG2Splits, di.sm_count);
  if (launch_moe_gemm(kGemm2Wide, kBN, tm_w2, tm_chi, tm_clo, g2, grid2, true, s) != cudaSuccess)
    return MOE_B200_ERR_CUDA;
  mark_stage(5, s);

  const int fgrid = 4 * T < di.sm_count * 8 ? 4 * T : di.sm_count * 8;   // 4 row segments
  if (output != nullptr &&
      launch_kernel(finalize_kernel, fgrid, 256, 0, s, true, static_cast<const float*>(y_acc),
                    static_cast<const int32_t*>(nullptr), static_cast<const int*>(nullptr),
                    static_cast<uint16_t*>(output), T) != cudaSuccess)
    return MOE_B200_ERR_CUDA;
  mark_stage(6, s);
  return MOE_B200_OK;
}

}  // namespace
}  // namespace moe

using namespace moe;

// A routing method and top_k the routing kernels support: DeepSeek-V3 with
// its 8 picks, Llama4 with 1, the others with 1 to 8.
static bool valid_routing(int method, int top_k, bool given_allowed = false) {
  if (method == kRouteGiven && !given_allowed) return false;   // only through moe_b200_run_routed
  switch (method) {
    case MOE_B200_ROUTING_DEEPSEEK_V3: return top_k == kTopK;
    case MOE_B200_ROUTING_LLAMA4: return top_k == 1;
    case MOE_B200_ROUTING_DEFAULT:
    case MOE_B200_ROUTING_RENORMALIZE:
    case MOE_B200_ROUTING_RENORMALIZE_NAIVE:
    case MOE_B200_ROUTING_TOPK:
    case kRouteGiven: return top_k >= 1 && top_k <= kTopK;
    default: return false;
  }
}

extern "C" {

int moe_b200_abi_version(void) { return 9; }

int moe_b200_set_stage_events(void* const* events, int num_events) {
  if (events == nullptr) {
    t_stage_events_on = false;
    return MOE_B200_OK;
  }
  if (num_events != MOE_B200_NUM_STAGE_EVENTS) return MOE_B200_ERR_INVALID_ARGUMENT;
  for (int i = 0; i < MOE_B200_NUM_STAGE_EVENTS; ++i) {
    if (events[i] == nullptr) return MOE_B200_ERR_INVALID_ARGUMENT;
    t_stage_events[i] = static_cast<cudaEvent_t>(events[i]);
  }
  t_stage_events_on = true;
  return MOE_B200_OK;
}

size_t moe_b200_workspace_bytes(int64_t num_tokens) {
  if (num_tokens < 0 || num_tokens > MOE_B200_MAX_TOKENS) return 0;
  return make_layout(num_tokens).total_bytes;
}

int moe_b200_get_workspace_layout(int64_t num_tokens, moe_b200_workspace_layout* out) {
  if (out == nullptr || num_tokens < 0 || num_tokens > MOE_B200_MAX_TOKENS)
    return MOE_B200_ERR_INVALID_ARGUMENT;
  *out = make_layout(num_tokens);
  return MOE_B200_OK;
}

size_t moe_b200_routed_workspace_bytes(int64_t num_tokens, int top_k) {
  if (num_tokens < 0 || num_tokens > MOE_B200_MAX_TOKENS || top_k < 1 || top_k > kTopK) return 0;
  return make_layout(num_tokens, top_k).total_bytes;
}

int moe_b200_get_routed_workspace_layout(int64_t num_tokens, int top_k, moe_b200_workspace_layout* out) {
  if (out == nullptr || num_tokens < 0 || num_tokens > MOE_B200_MAX_TOKENS || top_k < 1 || top_k > kTopK)
    return MOE_B200_ERR_INVALID_ARGUMENT;
  *out = make_layout(num_tokens, top_k);
  return MOE_B200_OK;
}

const char* moe_b200_status_string(int status) {
  switch (status) {
    case MOE_B200_OK: return "ok";
    case MOE_B200_ERR_INVALID_ARGUMENT: return "invalid argument";
    case MOE_B200_ERR_MISALIGNED: return "misaligned pointer";
    case MOE_B200_ERR_WORKSPACE_TOO_SMALL: return "workspace too small";
    case MOE_B200_ERR_UNSUPPORTED_DEVICE: return "current device is not an sm_100 (B200) GPU";
    case MOE_B200_ERR_DRIVER: return "cuTensorMapEncodeTiled unavailable or rejected a tensor map";
    case MOE_B200_ERR_CUDA: return "CUDA runtime error";
    case MOE_B200_ERR_DEVICE_TIMEOUT: return "a kernel gave up a bounded wait (device timeout)";
    default: return "unknown status";
  }
}

int moe_b200_route(const float* routing_logits, const void* routing_bias, int routing_bias_dtype,
                   int64_t num_tokens, double routed_scaling_factor, int32_t* topk_idx,
                   float* topk_w, void* stream) {
  return moe_b200_route_method(MOE_B200_ROUTING_DEEPSEEK_V3, kTopK, routing_logits, routing_bias,
                               routing_bias_dtype, num_tokens, routed_scaling_factor, topk_idx, topk_w, stream);
}

int moe_b200_route_method(int routing_method, int top_k, const float* routing_logits, const void* routing_bias,
                          int routing_bias_dtype, int64_t num_tokens, double routed_scaling_factor,
                          int32_t* topk_idx, float* topk_w, void* stream) {
  if (num_tokens < 0 || num_tokens > MOE_B200_MAX_TOKENS) return MOE_B200_ERR_INVALID_ARGUMENT;
  if (routing_bias_dtype != MOE_B200_BIAS_BF16 && routing_bias_dtype != MOE_B200_BIAS_FP32)
    return MOE_B200_ERR_INVALID_ARGUMENT;
  if (!valid_routing(routing_method, top_k)) return MOE_B200_ERR_INVALID_ARGUMENT;
  if (num_tokens == 0) return MOE_B200_OK;
  if (!routing_logits || (!routing_bias && routing_method == MOE_B200_ROUTING_DEEPSEEK_V3) || !topk_idx ||
      !topk_w)
    return MOE_B200_ERR_INVALID_ARGUMENT;
  if (!aligned(routing_logits, 16) || !aligned(routing_bias, 16) || !aligned(topk_idx, 16) ||
      !aligned(topk_w, 16))
    return MOE_B200_ERR_MISALIGNED;
  DeviceInfo di;
  int st = current_device_info(&di);
  if (st != MOE_B200_OK) return st;
  return launch_route(routing_logits, routing_bias, routing_bias_dtype, static_cast<int>(num_tokens),
                      static_cast<float>(routed_scaling_factor), 0, topk_idx, topk_w, nullptr, routing_method,
                      top_k, static_cast<cudaStream_t>(stream));
}

int moe_b200_read_status(const void* workspace, uint32_t* status, void* stream) {
  if (workspace == nullptr || status == nullptr) return MOE_B200_ERR_INVALID_ARGUMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const moe_b200_workspace_layout l = make_layout(0);
  uint32_t v = 0;
  if (cudaMemcpyAsync(&v, static_cast<const uint8_t*>(workspace) + l.status, sizeof(v),
                      cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return MOE_B200_ERR_CUDA;
  *status = v;
  return v == 0 ? MOE_B200_OK : MOE_B200_ERR_DEVICE_TIMEOUT;
}

// The layer on e4m3 hidden states with their block scales, or (hidden_bf16)
// on bf16 hidden states that the row copy into the permuted buffers
// quantises (hidden_states_scale unused).
static int run_layer(const float* routing_logits, const void* routing_bias, int routing_bias_dtype,
                     int routing_method, int top_k,
                     const void* hidden_states, const float* hidden_states_scale, bool hidden_bf16,
                     const void* gemm1_weights, const float* gemm1_weights_scale,
                     const void* gemm2_weights, const float* gemm2_weights_scale,
                     int64_t local_expert_offset, double routed_scaling_factor, int64_t num_tokens,
                     void* output, void* workspace, size_t workspace_bytes, void* stream,
                     const GivenPicks& given = GivenPicks{}) {
  // ---- argument checks (no device work before they pass) -----------------
  if (num_tokens < 0 || num_tokens > MOE_B200_MAX_TOKENS) return MOE_B200_ERR_INVALID_ARGUMENT;
  if (routing_bias_dtype != MOE_B200_BIAS_BF16 && routing_bias_dtype != MOE_B200_BIAS_FP32)
    return MOE_B200_ERR_INVALID_ARGUMENT;
  if (!valid_routing(routing_method, top_k, given.idx != nullptr || given.w != nullptr))
    return MOE_B200_ERR_INVALID_ARGUMENT;
  if (num_tokens == 0) return MOE_B200_OK;
  const bool given_picks = routing_method == kRouteGiven;
  if (given_picks ? (!given.idx || !given.w || !aligned(given.idx, 4) || !aligned(given.w, 4))
                  : !routing_logits)
    return given_picks && given.idx && given.w ? MOE_B200_ERR_MISALIGNED : MOE_B200_ERR_INVALID_ARGUMENT;
  if ((!routing_bias && routing_method == MOE_B200_ROUTING_DEEPSEEK_V3) || !hidden_states ||
      (!hidden_bf16 && !hidden_states_scale) ||
      !gemm1_weights || !gemm1_weights_scale || !gemm2_weights || !gemm2_weights_scale || !workspace)
    return MOE_B200_ERR_INVALID_ARGUMENT;
  if (!aligned(routing_logits, 16) || !aligned(routing_bias, 16) || !aligned(hidden_states, 16) ||
      !aligned(gemm1_weights, 16) || !aligned(gemm2_weights, 16) || !aligned(output, 16) ||
      !aligned(hidden_states_scale, 4) || !aligned(gemm1_weights_scale, 4) ||
      !aligned(gemm2_weights_scale, 4) || !aligned(workspace, kAlign))
    return MOE_B200_ERR_MISALIGNED;
  const moe_b200_workspace_layout l = make_layout(num_tokens, given_picks ? top_k : kTopK);
  if (workspace_bytes < l.total_bytes) return MOE_B200_ERR_WORKSPACE_TOO_SMALL;
  DeviceInfo di;
  int st = current_device_info(&di);
  if (st != MOE_B200_OK) return st;

  const int T = static_cast<int>(num_tokens);
  const int cap = static_cast<int>(l.cap_rows);
  // Offsets outside [-2^20, 2^20] select no local expert either way.
  int local_off = 1 << 21;
  if (local_expert_offset > -(1 << 20) && local_expert_offset < (1 << 20))
    local_off = static_cast<int>(local_expert_offset);
  const Plan plan = choose_plan(num_tokens);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int* counts = reinterpret_cast<int*>(ws + l.counts);
  uint32_t* status = reinterpret_cast<uint32_t*>(ws + l.status);
  int* sched = reinterpret_cast<int*>(ws + l.sched);
  int* seg_off = reinterpret_cast<int*>(ws + l.seg_off);
  int32_t* topk_idx = reinterpret_cast<int32_t*>(ws + l.topk_idx);
  float* topk_w = reinterpret_cast<float*>(ws + l.topk_w);
  int32_t* perm_tok = reinterpret_cast<int32_t*>(ws + l.perm_tok);
  float* perm_w = reinterpret_cast<float*>(ws + l.perm_w);
  uint8_t* a_perm = ws + l.a_perm;
  float* sa_perm = reinterpret_cast<float*>(ws + l.sa_perm);
  uint8_t* c_hi = ws + l.c_hi;
  uint8_t* c_lo = ws + l.c_lo;
  float* c_scale = reinterpret_cast<float*>(ws + l.c_scale);
  float* y_acc = reinterpret_cast<float*>(ws + l.y_acc);
  int32_t* perm_row = reinterpret_cast<int32_t*>(ws + l.perm_row);
  int32_t* tok_slot = reinterpret_cast<int32_t*>(ws + l.tok_slot);
  int* n_touched = reinterpret_cast<int*>(ws + l.n_touched);
  int32_t* slot_tok = reinterpret_cast<int32_t*>(ws + l.slot_tok);

  if (plan.decode)
    return run_decode(routing_logits, routing_bias, routing_bias_dtype, routing_method, top_k, hidden_states,
                      hidden_states_scale, hidden_bf16, gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, local_off,
                      static_cast<float>(routed_scaling_factor), T, output, ws, l, di, s, given);

  // ---- tensor maps ---------------------------------------------------------
  CUtensorMap tm_aperm, tm_w13, tm_w2, tm_chi, tm_clo;
  const uint32_t a_box = plan.token_major ? 128 : plan.g1_bn;
  const uint32_t c_box = plan.token_major ? 128 : plan.g2_bn;
  if (!encode_u8_2d(&tm_aperm, a_perm, kHidden, cap, 128, a_box) ||
      !encode_u8_2d(&tm_w13, gemm1_weights, kHidden, static_cast<uint64_t>(kExpertsLocal) * kGemm1Out,
                    128, 128) ||
      !encode_u8_2d(&tm_w2, gemm2_weights, kInter, static_cast<uint64_t>(kExpertsLocal) * kHidden, 128,
                    128) ||
      !encode_u8_2d(&tm_chi, c_hi, kInter, cap, 128, c_box) ||
      !encode_u8_2d(&tm_clo, c_lo, kInter, cap, 128, c_box))
    return MOE_B200_ERR_DRIVER;

  // ---- launches ------------------------------------------------------------
  // Nothing is cleared here: the permutation counts without atomics and
  // clears the status word, the gather kernel clears the accumulation
  // buffers, so the workspace may hold anything when the call starts.
  mark_stage(0, s);
  if (hidden_bf16) {
    // bf16 hidden states: each token row is quantised once into the
    // workspace, and the rest of the call reads that e4m3 copy (a row is
    // copied once per local pick, 4.4 times per token in the prefill
    // workload, so quantising inside the row copy repeats the work)
    uint8_t* hq = ws + l.hidden_q;
    float* hqs = reinterpret_cast<float*>(ws + l.hidden_qs);
    quantize_hidden_kernel<<<static_cast<unsigned>(div_up(T, 8)), 256, 0, s>>>(
        static_cast<const uint16_t*>(hidden_states), T, hq, hqs);
    if (cudaGetLastError() != cudaSuccess) return MOE_B200_ERR_CUDA;
    hidden_states = hq;
    hidden_states_scale = hqs;
  }
  mark_stage(1, s);
  st = launch_route(routing_logits, routing_bias, routing_bias_dtype, T,
                    static_cast<float>(routed_scaling_factor), local_off, topk_idx, topk_w,
                    static_cast<uint16_t*>(output), routing_method, top_k, s, given);
  if (st != MOE_B200_OK) return st;
  mark_stage(2, s);

  PermuteParams pp;
  pp.topk_idx = topk_idx;
  pp.topk_w = topk_w;
  pp.counts = counts;
  pp.chunk_counts = reinterpret_cast<int*>(ws + l.chunk_counts);
  pp.status = status;
  pp.sched = sched;
  pp.num_tokens = T;
  pp.local_expert_offset = local_off;
  pp.seg_off = seg_off;
  pp.perm_tok = perm_tok;
  pp.perm_w = perm_w;
  pp.perm_row = perm_row;
  pp.tok_slot = tok_slot;
  pp.n_touched = n_touched;
  pp.slot_tok = slot_tok;
  if (T <= 1024) {
    if (launch_kernel(permute_kernel, 1, 1024, 0, s, true, pp) != cudaSuccess) return MOE_B200_ERR_CUDA;
  } else {
    const int chunks = static_cast<int>(div_up(T, kPermChunk));
    if (launch_kernel(permute_count_kernel, chunks, kPermChunk, 0, s, true, pp) != cudaSuccess ||
        launch_kernel(permute_place_kernel, chunks, kPermChunk, 0, s, true, pp) != cudaSuccess)
      return MOE_B200_ERR_CUDA;
  }
  GatherParams gp;
  gp.seg_off = seg_off;
  gp.n_touched = n_touched;
  gp.perm_tok = perm_tok;
  gp.hidden = static_cast<const uint8_t*>(hidden_states);
  gp.hidden_scale = hidden_states_scale;
  gp.num_tokens = T;
  gp.cap = cap;
  gp.a_perm = a_perm;
  gp.sa_perm = sa_perm;
  gp.y_acc = y_acc;
  gp.counts = counts;
  gp.g1_acc = plan.token_major ? reinterpret_cast<float*>(ws + l.g1_acc) : nullptr;
  int ggrid = static_cast<int>(div_up(cap, 8));
  if (ggrid < di.sm_count) ggrid = di.sm_count;
  if (ggrid > di.sm_count * 4) ggrid = di.sm_count * 4;
  if (launch_kernel(gather_rows_kernel, ggrid, 256, 0, s, true, gp) != cudaSuccess) return MOE_B200_ERR_CUDA;
  mark_stage(3, s);

  GemmParams g1;
  std::memset(&g1, 0, sizeof(g1));
  g1.seg_off = seg_off;
  g1.counts = counts;
  g1.perm_tok = perm_tok;
  g1.perm_row = perm_row;
  g1.perm_w = perm_w;
  g1.act_scale = sa_perm;
  g1.w_scale = gemm1_weights_scale;
  g1.num_tokens = T;
  g1.cap = cap;
  g1.splits = 1;
  g1.c_hi = c_hi;
  g1.c_lo = c_lo;
  g1.c_scale = c_scale;
  g1.g1_acc = plan.token_major ? reinterpret_cast<float*>(ws + l.g1_acc) : nullptr;
  g1.status = status;
  g1.sched = sched;
  const int grid1 = grid_for(num_tokens, plan.g1_bn, kInterBlocks, 1, di.sm_count);
  if (plan.token_major) {
    const int grid_tm = grid_for(num_tokens, 128, kInterBlocks, 1, di.sm_count);
    if (launch_moe_gemm_tm(true, tm_w13, tm_aperm, tm_aperm, g1, grid_tm, s) != cudaSuccess)
      return MOE_B200_ERR_CUDA;
  } else {
    if (launch_moe_gemm(kGemm1Fused, plan.g1_bn, tm_w13, tm_aperm, tm_aperm, g1, grid1, true, s) != cudaSuccess)
      return MOE_B200_ERR_CUDA;
  }

  mark_stage(4, s);
  GemmParams g2 = g1;
  g2.act_scale = c_scale;
  g2.sched = sched + 1;
  g2.w_scale = gemm2_weights_scale;
  g2.splits = 1;
  g2.y_acc = y_acc;
  // token-major GEMM2 counts its CTAs here after the SwiGLU phase of a
  // K-split GEMM1 (cleared by the permutation)
  g2.grid_sync = plan.token_major ? sched + 2 : nullptr;
  const int g2_kind = plan.g2_wide ? kGemm2Wide : kGemm2;
  const int grid2 = grid_for(num_tokens, plan.g2_bn, plan.g2_wide ? kHiddenBlocks / 2 : kHiddenBlocks,
                             1, di.sm_count);
  if (plan.token_major) {
    const int grid_tm = grid_for(num_tokens, 128, kHiddenBlocks / 2, 1, di.sm_count);
    if (launch_moe_gemm_tm(false, tm_w2, tm_chi, tm_clo, g2, grid_tm, s) != cudaSuccess)
      return MOE_B200_ERR_CUDA;
  } else if (launch_moe_gemm(g2_kind, plan.g2_bn, tm_w2, tm_chi, tm_clo, g2, grid2, true, s) != cudaSuccess) {
    return MOE_B200_ERR_CUDA;
  }
  mark_stage(5, s);

  const int fgrid = 4 * T < di.sm_count * 8 ? 4 * T : di.sm_count * 8;   // 4 row segments
  if (output != nullptr &&
      launch_kernel(finalize_kernel, fgrid, 256, 0, s, true, static_cast<const float*>(y_acc),
                    static_cast<const int32_t*>(slot_tok), static_cast<const int*>(n_touched),
                    static_cast<uint16_t*>(output), T) != cudaSuccess)
    return MOE_B200_ERR_CUDA;
  mark_stage(6, s);
  return MOE_B200_OK;
}

int moe_b200_run(const float* routing_logits, const void* routing_bias, int routing_bias_dtype,
                 const void* hidden_states, const float* hidden_states_scale,
                 const void* gemm1_weights, const float* gemm1_weights_scale,
                 const void* gemm2_weights, const float* gemm2_weights_scale,
                 int64_t local_expert_offset, double routed_scaling_factor, int64_t num_tokens,
                 void* output, void* workspace, size_t workspace_bytes, void* stream) {
  return run_layer(routing_logits, routing_bias, routing_bias_dtype, MOE_B200_ROUTING_DEEPSEEK_V3, kTopK,
                   hidden_states, hidden_states_scale, false, gemm1_weights, gemm1_weights_scale, gemm2_weights,
                   gemm2_weights_scale, local_expert_offset, routed_scaling_factor, num_tokens, output, workspace,
                   workspace_bytes, stream);
}

int moe_b200_run_routing(int routing_method, int top_k, const float* routing_logits, const void* routing_bias,
                         int routing_bias_dtype, const void* hidden_states, const float* hidden_states_scale,
                         const void* gemm1_weights, const float* gemm1_weights_scale, const void* gemm2_weights,
                         const float* gemm2_weights_scale, int64_t local_expert_offset,
                         double routed_scaling_factor, int64_t num_tokens, void* output, void* workspace,
                         size_t workspace_bytes, void* stream) {
  return run_layer(routing_logits, routing_bias, routing_bias_dtype, routing_method, top_k, hidden_states,
                   hidden_states_scale, false, gemm1_weights, gemm1_weights_scale, gemm2_weights,
                   gemm2_weights_scale, local_expert_offset, routed_scaling_factor, num_tokens, output, workspace,
                   workspace_bytes, stream);
}

int moe_b200_run_routed(const int32_t* topk_idx, const float* topk_w, int top_k, const void* hidden_states,
                        const float* hidden_states_scale, const void* gemm1_weights,
                        const float* gemm1_weights_scale, const void* gemm2_weights,
                        const float* gemm2_weights_scale, int64_t local_expert_offset, int64_t num_tokens,
                        void* output, void* workspace, size_t workspace_bytes, void* stream) {
  GivenPicks given;
  given.idx = topk_idx;
  given.w = topk_w;
  return run_layer(nullptr, nullptr, MOE_B200_BIAS_BF16, kRouteGiven, top_k, hidden_states, hidden_states_scale,
                   false, gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale,
                   local_expert_offset, 1.0, num_tokens, output, workspace, workspace_bytes, stream, given);
}

int moe_b200_run_bf16_hidden(const float* routing_logits, const void* routing_bias, int routing_bias_dtype,
                             const void* hidden_states, const void* gemm1_weights,
                             const float* gemm1_weights_scale, const void* gemm2_weights,
                             const float* gemm2_weights_scale, int64_t local_expert_offset,
                             double routed_scaling_factor, int64_t num_tokens, void* output, void* workspace,
                             size_t workspace_bytes, void* stream) {
  return run_layer(routing_logits, routing_bias, routing_bias_dtype, MOE_B200_ROUTING_DEEPSEEK_V3, kTopK,
                   hidden_states, nullptr, true, gemm1_weights,
                   gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, local_expert_offset,
                   routed_scaling_factor, num_tokens, output, workspace, workspace_bytes, stream);
}

int moe_b200_quantize_hidden(const void* hidden_states, int64_t num_tokens, void* hidden_fp8, float* hidden_scale,
                             void* stream) {
  if (num_tokens < 0 || num_tokens > MOE_B200_MAX_TOKENS) return MOE_B200_ERR_INVALID_ARGUMENT;
  if (num_tokens == 0) return MOE_B200_OK;
  if (!hidden_states || !hidden_fp8 || !hidden_scale) return MOE_B200_ERR_INVALID_ARGUMENT;
  if (!aligned(hidden_states, 16) || !aligned(hidden_fp8, 16) || !aligned(hidden_scale, 4))
    return MOE_B200_ERR_MISALIGNED;
  DeviceInfo di;
  const int st = current_device_info(&di);
  if (st != MOE_B200_OK) return st;
  quantize_hidden_kernel<<<static_cast<unsigned>(div_up(num_tokens, 8)), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(hidden_states), static_cast<int>(num_tokens), static_cast<uint8_t*>(hidden_fp8),
      hidden_scale);
  return cudaGetLastError() == cudaSuccess ? MOE_B200_OK : MOE_B200_ERR_CUDA;
}

}  // extern "C"
