// Token-parallel expert parallelism: all-to-all dispatch and combine over
// NVLink peer memory.
//
// Here every rank holds its own tokens (different on every rank) and owns
// S 32-expert shards: rank q owns global experts [32 S q, 32 S (q + 1)).
// Each rank routes its own tokens (DeepSeek-V3, all 256 experts), then
//   plan      (one CTA) numbers, for every destination rank, its tokens with
//             at least one pick there, in token order; writes its row of the
//             send-count matrix into every rank's area and announces the call
//             (release store, system scope);
//   dispatch  waits for every rank's row, places token t's row for
//             destination q at row off(q, r) + slot of q's receive slab, where
//             off is the exclusive sum over lower source ranks, and writes
//             there by peer stores the wire format of one (token, destination)
//             row: the token's e4m3 row (7,168 B), its 56 block scales (into
//             the slab's [56, R] scale matrix) and its eight picks with only
//             those on q kept (others: no expert, weight 0); a token travels
//             once to each rank it has picks on (DeepSeek-V3 keeps 4 groups of
//             32 experts, so at most 4 ranks), not once per pick; then it
//             counts its CTAs on every rank and waits for all of them;
//   layer     moe_b200_run_routed on the slab, once per owned shard (each row
//             is a token with its picks on this rank; a shard takes those in
//             its 32 experts, and its layer already sums them into one combine
//             row; rows past the received count hold no pick), combine rows
//             left in each shard's workspace;
//   combine   announces, waits for every rank, and forms each own token's
//             output as the fp32 sum of its combine rows on the destination
//             ranks' shards (peer loads): each rank's shards in shard order,
//             then the ranks in rank order (the order of the expert-parallel
//             combine), rounded once to bf16.
// The order of rows inside a slab depends only on the routing, so results do
// not depend on timing. Counters only grow (signed-difference compares, so
// they may wrap); every wait gives up after one second with a status bit and
// poisons every rank's area, after which every call returns at once until the
// counter blocks are zeroed. No multicast; no library kernel reads peer memory.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

#include "../../include/moe_b200.h"
#include "moe_kernels.cuh"
#include "moe_ptx.cuh"
#include "moe_shapes.cuh"

namespace moe {

namespace {

constexpr uint32_t kStatusTimeoutPeer = 1u << 7;
constexpr uint32_t kStatusPoisoned = 1u << 8;
constexpr uint32_t kStatusRecvOverflow = 1u << 9;   // a destination's slab was too small
constexpr int kA2aMaxRanks = 8;
constexpr int kA2aThreads = 256;
constexpr int kA2aCtasPerSm = 2;                     // all CTAs resident: they wait for each other
constexpr int kPlanThreads = 1024;

// Counter block of a rank's area: counters in bytes [0, 256), the count
// matrix in [256, 512).
struct A2aCounters {
  static constexpr size_t kFlagsDispatch = 0;   // int32[8]: call announced by each source rank (plan)
  static constexpr size_t kDoneDispatch = 32;   // int32: CTAs (all ranks) that finished writing into this slab
  static constexpr size_t kFlagsCombine = 64;   // int32[8]: call announced by each rank (combine)
  static constexpr size_t kCalls = 96;          // int32: completed calls of this rank
  static constexpr size_t kFinished = 100;      // int32: combine CTAs of this rank that finished a call
  static constexpr size_t kPoison = 104;        // int32: nonzero once a wait gave up
  static constexpr size_t kStatus = 108;        // uint32: status bits of this rank's current call
  static constexpr size_t kRecvRows = 112;      // int32: rows received by the last dispatch
  static constexpr size_t kCounts = 256;        // int32[8][8]: picks sent from rank [src] to rank [dst]
  static constexpr size_t kEnd = 512;
};
static_assert(A2aCounters::kEnd == MOE_B200_A2A_COUNTER_BYTES, "counter block size in the header");

size_t align256(size_t x) { return (x + 255) / 256 * 256; }

// Offsets inside a rank's area for max_tokens own tokens and a receive slab
// of `cap` rows; identical on every rank (all ranks pass the same sizes).
moe_b200_a2a_layout a2a_layout(int64_t max_tokens, int64_t cap) {
  moe_b200_a2a_layout l;
  std::memset(&l, 0, sizeof(l));
  size_t off = A2aCounters::kEnd;
  l.send_slot = off;
  off = align256(off + static_cast<size_t>(max_tokens) * kA2aMaxRanks * sizeof(int32_t));
  l.dest_row = off;
  off = align256(off + static_cast<size_t>(max_tokens) * kA2aMaxRanks * sizeof(int32_t));
  l.slab_idx = off;
  off = align256(off + static_cast<size_t>(cap) * kTopK * sizeof(int32_t));
  l.slab_w = off;
  off = align256(off + static_cast<size_t>(cap) * kTopK * sizeof(float));
  l.slab_scale = off;
  off = align256(off + static_cast<size_t>(cap) * kHiddenBlocks * sizeof(float));
  l.slab_rows = off;
  off = align256(off + static_cast<size_t>(cap) * kHidden);
  l.total_bytes = off;
  return l;
}

struct A2aParams {
  uint8_t* area[kA2aMaxRanks];          // every rank's area (this process's mapping)
  const int32_t* topk_idx;              // [T, 8] this rank's picks, global expert ids
  const float* topk_w;                  // [T, 8]
  const uint8_t* hidden;                // [T, 7168] e4m3 (dispatch)
  const float* hidden_scale;            // [56, T] (dispatch)
  const float* y[kA2aMaxRanks];         // combine: every shard's fp32 combine rows, rank-major
  const int32_t* slot[kA2aMaxRanks];    // combine: each shard's row -> combine row map (null: row = row)
  uint16_t* out;                        // combine: this rank's output, bf16 [T, 7168]
  size_t send_slot, dest_row, slab_idx, slab_w, slab_scale, slab_rows;   // area offsets
  int rank, world, shards, num_tokens, cap;
};

__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void red_release_sys_add(int* p, int v) {
  asm volatile("red.release.sys.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ bool wait_at_least(const int* p, uint32_t target) {
  const uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (static_cast<int32_t>(static_cast<uint32_t>(ld_acquire_sys(p)) - target) < 0) {
    if ((++spins & 63u) == 0u && globaltimer_ns() - t0 > kWaitBudgetNs) return false;
  }
  return true;
}

__device__ __forceinline__ int* ctr(uint8_t* area, size_t off) { return reinterpret_cast<int*>(area + off); }

__device__ __forceinline__ void set_status(const A2aParams& p, uint32_t bits) {
  atomicOr(reinterpret_cast<unsigned int*>(p.area[p.rank] + A2aCounters::kStatus), bits);
}

__device__ __forceinline__ void give_up(const A2aParams& p) {
  set_status(p, kStatusTimeoutPeer);
  for (int q = 0; q < p.world; ++q) st_release_sys(ctr(p.area[q], A2aCounters::kPoison), 1);
}

__device__ __forceinline__ bool poisoned(const A2aParams& p) {
  return *reinterpret_cast<volatile int*>(p.area[p.rank] + A2aCounters::kPoison) != 0;
}

// Destination rank of a global expert id, or -1 (no pick / out of range).
__device__ __forceinline__ int dest_rank(int e, int shards) {
  return (e >= 0 && e < kExpertsGlobal) ? e / (kExpertsLocal * shards) : -1;
}

__device__ __forceinline__ uint2 pack_bf16x4(float x, float y, float z, float w) {
  const __nv_bfloat162 lo = __floats2bfloat162_rn(x, y);
  const __nv_bfloat162 hi = __floats2bfloat162_rn(z, w);
  return make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
}

}  // namespace

// ---------------------------------------------------------------- plan
// One CTA: numbers, for every destination, this rank's tokens with a pick
// there, in token order (ballot ranks inside a warp, a per-destination scan
// over the warps), then publishes the counts and the call.
__global__ void __launch_bounds__(kPlanThreads) a2a_plan_kernel(A2aParams p) {
  __shared__ int s_warp_cnt[kPlanThreads / 32][kA2aMaxRanks];
  __shared__ int s_running[kA2aMaxRanks];
  __shared__ int s_poisoned;
  pdl_wait();
  const int W = p.world;
  uint8_t* mine = p.area[p.rank];
  if (threadIdx.x == 0) {
    *reinterpret_cast<volatile uint32_t*>(mine + A2aCounters::kStatus) = 0u;
    s_poisoned = poisoned(p) ? 1 : 0;
    if (s_poisoned) set_status(p, kStatusPoisoned);
  }
  if (threadIdx.x < kA2aMaxRanks) s_running[threadIdx.x] = 0;
  __syncthreads();
  if (s_poisoned) return;
  const uint32_t call = *reinterpret_cast<volatile uint32_t*>(mine + A2aCounters::kCalls) + 1u;
  int32_t* send_slot = reinterpret_cast<int32_t*>(mine + p.send_slot);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t lt = (1u << lane) - 1u;
  const int T = p.num_tokens;
  for (int base = 0; base < T; base += kPlanThreads) {
    const int t = base + static_cast<int>(threadIdx.x);
    uint32_t mask = 0;   // destinations this token has a pick on
    if (t < T) {
#pragma unroll
      for (int k = 0; k < kTopK; ++k) {
        const int q = dest_rank(__ldg(p.topk_idx + t * kTopK + k), p.shards);
        if (q >= 0) mask |= 1u << q;
      }
    }
    int in_warp[kA2aMaxRanks];
#pragma unroll
    for (int d = 0; d < kA2aMaxRanks; ++d) {
      in_warp[d] = 0;
      if (d < W) {
        const uint32_t m = __ballot_sync(0xffffffffu, (mask >> d) & 1u);
        in_warp[d] = __popc(m & lt);
        if (lane == 0) s_warp_cnt[warp][d] = __popc(m);
      }
    }
    __syncthreads();
    if (threadIdx.x < W) {   // exclusive scan over the warps, one destination per thread
      int run = s_running[threadIdx.x];
      for (int w = 0; w < kPlanThreads / 32; ++w) {
        const int c = s_warp_cnt[w][threadIdx.x];
        s_warp_cnt[w][threadIdx.x] = run;
        run += c;
      }
      s_running[threadIdx.x] = run;
    }
    __syncthreads();
    if (t < T) {
#pragma unroll
      for (int d = 0; d < kA2aMaxRanks; ++d)
        send_slot[t * kA2aMaxRanks + d] = (d < W && ((mask >> d) & 1u)) ? s_warp_cnt[warp][d] + in_warp[d] : -1;
    }
    __syncthreads();
  }
  // this rank's row of the count matrix into every rank's area, then the call
  if (threadIdx.x < W * W) {
    const int dst_area = threadIdx.x / W, q = threadIdx.x % W;
    reinterpret_cast<int*>(p.area[dst_area] + A2aCounters::kCounts)[p.rank * kA2aMaxRanks + q] = s_running[q];
  }
  __syncthreads();
  if (threadIdx.x < W) {
    __threadfence_system();
    st_release_sys(ctr(p.area[threadIdx.x], A2aCounters::kFlagsDispatch) + p.rank, static_cast<int>(call));
  }
}

// ---------------------------------------------------------------- dispatch
__global__ void __launch_bounds__(kA2aThreads, kA2aCtasPerSm) a2a_dispatch_kernel(A2aParams p) {
  __shared__ int s_ok;
  __shared__ int s_live;
  __shared__ int s_off[kA2aMaxRanks];
  __shared__ int s_recv;
  pdl_wait();   // the plan kernel has published this rank's counts
  const int W = p.world;
  uint8_t* mine = p.area[p.rank];
  // the poison word is read once for the CTA (a peer may set it meanwhile),
  // so every thread takes the same path through the barriers below
  if (threadIdx.x == 0) {
    s_live = poisoned(p) ? 0 : 1;
    s_ok = 1;
  }
  __syncthreads();
  if (!s_live) return;   // the plan kernel has set the status bit
  const uint32_t call = *reinterpret_cast<volatile uint32_t*>(mine + A2aCounters::kCalls) + 1u;
  if (threadIdx.x < W &&
      !wait_at_least(ctr(mine, A2aCounters::kFlagsDispatch) + threadIdx.x, call)) {
    give_up(p);
    s_ok = 0;
  }
  __syncthreads();
  if (!s_ok) return;
  const volatile int* counts = reinterpret_cast<const volatile int*>(mine + A2aCounters::kCounts);
  if (threadIdx.x < W) {   // where this rank's picks start in destination q's slab
    int off = 0;
    for (int src = 0; src < p.rank; ++src) off += counts[src * kA2aMaxRanks + threadIdx.x];
    s_off[threadIdx.x] = off;
  }
  if (threadIdx.x == 0) {
    int r = 0;
    for (int src = 0; src < W; ++src) r += counts[src * kA2aMaxRanks + p.rank];
    s_recv = r;
  }
  __syncthreads();

  // one warp per (token, destination): row (448 x 16 B), 56 scales and the
  // token's picks on that destination (the other picks: no expert)
  const int32_t* send_slot = reinterpret_cast<const int32_t*>(mine + p.send_slot);
  int32_t* dest_row = reinterpret_cast<int32_t*>(mine + p.dest_row);
  const int lane = threadIdx.x & 31;
  const int warps = static_cast<int>(gridDim.x) * (kA2aThreads / 32);
  const int n = p.num_tokens * kA2aMaxRanks;
  for (int i = static_cast<int>(blockIdx.x) * (kA2aThreads / 32) + (threadIdx.x >> 5); i < n; i += warps) {
    const int t = i / kA2aMaxRanks;
    const int q = i - t * kA2aMaxRanks;
    const int slot = send_slot[i];
    int j = -1;
    if (q < W && slot >= 0) {
      j = s_off[q] + slot;
      if (j >= p.cap) {
        if (lane == 0) set_status(p, kStatusRecvOverflow);
        j = -1;
      }
    }
    if (lane == 0) dest_row[i] = j;
    if (j < 0) continue;
    uint8_t* dst = p.area[q];
    const uint4* src_row = reinterpret_cast<const uint4*>(p.hidden + static_cast<int64_t>(t) * kHidden);
    uint4* dst_row = reinterpret_cast<uint4*>(dst + p.slab_rows + static_cast<int64_t>(j) * kHidden);
    uint4 v[kHidden / 16 / 32];
#pragma unroll
    for (int c = 0; c < kHidden / 16 / 32; ++c) v[c] = __ldg(src_row + lane + 32 * c);
#pragma unroll
    for (int c = 0; c < kHidden / 16 / 32; ++c) dst_row[lane + 32 * c] = v[c];
    float* dst_scale = reinterpret_cast<float*>(dst + p.slab_scale);
    for (int b = lane; b < kHiddenBlocks; b += 32)
      dst_scale[static_cast<int64_t>(b) * p.cap + j] = __ldg(p.hidden_scale + static_cast<int64_t>(b) * p.num_tokens + t);
    if (lane < kTopK) {
      const int e = __ldg(p.topk_idx + t * kTopK + lane);
      const bool here = dest_rank(e, p.shards) == q;
      reinterpret_cast<int32_t*>(dst + p.slab_idx)[static_cast<int64_t>(j) * kTopK + lane] = here ? e : kNoExpert;
      reinterpret_cast<float*>(dst + p.slab_w)[static_cast<int64_t>(j) * kTopK + lane] =
          here ? __ldg(p.topk_w + t * kTopK + lane) : 0.f;
    }
  }
  // rows past the received count carry no pick (the layer skips them)
  const int recv = min(s_recv, p.cap);
  if (s_recv > p.cap && blockIdx.x == 0 && threadIdx.x == 0) set_status(p, kStatusRecvOverflow);
  int32_t* my_idx = reinterpret_cast<int32_t*>(mine + p.slab_idx);
  float* my_w = reinterpret_cast<float*>(mine + p.slab_w);
  const int64_t pad = static_cast<int64_t>(p.cap - recv) * kTopK;
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * kA2aThreads + threadIdx.x; r < pad;
       r += static_cast<int64_t>(gridDim.x) * kA2aThreads) {
    my_idx[static_cast<int64_t>(recv) * kTopK + r] = kNoExpert;
    my_w[static_cast<int64_t>(recv) * kTopK + r] = 0.f;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) *ctr(mine, A2aCounters::kRecvRows) = recv;

  // count this CTA on every rank, wait until every CTA wrote into this slab
  __syncthreads();
  if (threadIdx.x < W) {
    __threadfence_system();
    red_release_sys_add(ctr(p.area[threadIdx.x], A2aCounters::kDoneDispatch), 1);
  }
  if (threadIdx.x == 0 &&
      !wait_at_least(ctr(mine, A2aCounters::kDoneDispatch), call * static_cast<uint32_t>(W) * gridDim.x))
    give_up(p);
}

// ---------------------------------------------------------------- combine
__global__ void __launch_bounds__(kA2aThreads, kA2aCtasPerSm) a2a_combine_kernel(A2aParams p) {
  __shared__ int s_ok;
  __shared__ int s_live;
  pdl_wait();   // this rank's layer calls on its slab have completed
  const int W = p.world;
  uint8_t* mine = p.area[p.rank];
  // one read of the poison word for the CTA, as in the dispatch
  if (threadIdx.x == 0) {
    s_live = poisoned(p) ? 0 : 1;
    s_ok = 1;
  }
  __syncthreads();
  if (!s_live) {
    if (threadIdx.x == 0) set_status(p, kStatusPoisoned);
    return;
  }
  const uint32_t call = *reinterpret_cast<volatile uint32_t*>(mine + A2aCounters::kCalls) + 1u;
  if (blockIdx.x == 0 && threadIdx.x < W)
    st_release_sys(ctr(p.area[threadIdx.x], A2aCounters::kFlagsCombine) + p.rank, static_cast<int>(call));
  if (threadIdx.x < W && !wait_at_least(ctr(mine, A2aCounters::kFlagsCombine) + threadIdx.x, call)) {
    give_up(p);
    s_ok = 0;
  }
  __syncthreads();
  if (s_ok) {
    // token t, column quads j and 896 + j: its combine rows on every shard of
    // every destination rank (sources rank-major: shard sh = q * S + s),
    // each rank's shards summed in shard order, then the ranks in rank order
    constexpr int kHalfQuads = kHidden / 8;
    const int32_t* dest_row = reinterpret_cast<const int32_t*>(mine + p.dest_row);
    const int S = p.shards;
    const int items = p.num_tokens * kHalfQuads;
    for (int it = static_cast<int>(blockIdx.x) * kA2aThreads + static_cast<int>(threadIdx.x); it < items;
         it += static_cast<int>(gridDim.x) * kA2aThreads) {
      const int t = it / kHalfQuads;
      const int j = it - t * kHalfQuads;
      const float* src[kTopK];
#pragma unroll
      for (int sh = 0; sh < kTopK; ++sh) {   // W * S = 8 shards
        src[sh] = nullptr;
        const int r = dest_row[t * kA2aMaxRanks + sh / S];
        if (r >= 0) {
          const int row = p.slot[sh] != nullptr ? p.slot[sh][r] : r;
          if (row >= 0) src[sh] = p.y[sh] + static_cast<int64_t>(row) * kHidden;
        }
      }
      float4 u[kTopK], v[kTopK];
#pragma unroll
      for (int sh = 0; sh < kTopK; ++sh) {
        u[sh] = make_float4(0.f, 0.f, 0.f, 0.f);
        v[sh] = u[sh];
        if (src[sh] != nullptr) {
          u[sh] = reinterpret_cast<const float4*>(src[sh])[j];
          v[sh] = reinterpret_cast<const float4*>(src[sh])[kHalfQuads + j];
        }
      }
      float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      float b[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int sh = 0; sh < kTopK; ++sh) {
        b[0] += u[sh].x; b[1] += u[sh].y; b[2] += u[sh].z; b[3] += u[sh].w;
        b[4] += v[sh].x; b[5] += v[sh].y; b[6] += v[sh].z; b[7] += v[sh].w;
        if ((sh + 1) % S == 0) {
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            a[c] += b[c];
            b[c] = 0.f;
          }
        }
      }
      uint2* orow = reinterpret_cast<uint2*>(p.out + static_cast<int64_t>(t) * kHidden);
      orow[j] = pack_bf16x4(a[0], a[1], a[2], a[3]);
      orow[kHalfQuads + j] = pack_bf16x4(a[4], a[5], a[6], a[7]);
    }
  }
  // the last CTA of this rank advances the call number
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t f = atomicAdd(reinterpret_cast<unsigned int*>(mine + A2aCounters::kFinished), 1u) + 1u;
    if (f == call * gridDim.x) *reinterpret_cast<volatile uint32_t*>(mine + A2aCounters::kCalls) = call;
  }
}

}  // namespace moe

using namespace moe;

namespace {

int a2a_grid(int* grid) {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
    return MOE_B200_ERR_CUDA;
  *grid = kA2aCtasPerSm * sms;
  return MOE_B200_OK;
}

bool a2a_sizes_ok(int64_t num_tokens, int64_t max_tokens, int64_t cap) {
  return num_tokens >= 0 && max_tokens >= 0 && num_tokens <= max_tokens && max_tokens <= MOE_B200_MAX_TOKENS &&
         cap >= 1 && cap <= MOE_B200_MAX_TOKENS;
}

// Common argument checks; fills the area pointers and layout offsets.
int a2a_params(void* const* rank_areas, int rank, int world, int shards_per_rank, int64_t num_tokens,
               int64_t max_tokens, int64_t cap, A2aParams* p) {
  if (rank_areas == nullptr || world < 1 || world > kA2aMaxRanks || rank < 0 || rank >= world ||
      shards_per_rank < 1 || world * shards_per_rank != kExpertsGlobal / kExpertsLocal ||
      !a2a_sizes_ok(num_tokens, max_tokens, cap))
    return MOE_B200_ERR_INVALID_ARGUMENT;
  std::memset(p, 0, sizeof(*p));
  for (int q = 0; q < world; ++q) {
    if (rank_areas[q] == nullptr) return MOE_B200_ERR_INVALID_ARGUMENT;
    if (reinterpret_cast<uintptr_t>(rank_areas[q]) % 256 != 0) return MOE_B200_ERR_MISALIGNED;
    p->area[q] = static_cast<uint8_t*>(rank_areas[q]);
  }
  const moe_b200_a2a_layout l = a2a_layout(max_tokens, cap);
  p->send_slot = l.send_slot;
  p->dest_row = l.dest_row;
  p->slab_idx = l.slab_idx;
  p->slab_w = l.slab_w;
  p->slab_scale = l.slab_scale;
  p->slab_rows = l.slab_rows;
  p->rank = rank;
  p->world = world;
  p->shards = shards_per_rank;
  p->num_tokens = static_cast<int>(num_tokens);
  p->cap = static_cast<int>(cap);
  return MOE_B200_OK;
}

}  // namespace

extern "C" {

size_t moe_b200_a2a_area_bytes(int64_t max_tokens, int64_t recv_capacity) {
  if (!a2a_sizes_ok(0, max_tokens, recv_capacity)) return 0;
  return a2a_layout(max_tokens, recv_capacity).total_bytes;
}

int moe_b200_a2a_get_layout(int64_t max_tokens, int64_t recv_capacity, moe_b200_a2a_layout* out) {
  if (out == nullptr || !a2a_sizes_ok(0, max_tokens, recv_capacity)) return MOE_B200_ERR_INVALID_ARGUMENT;
  *out = a2a_layout(max_tokens, recv_capacity);
  return MOE_B200_OK;
}

int moe_b200_a2a_dispatch(const int32_t* topk_idx, const float* topk_w, const void* hidden_states,
                          const float* hidden_states_scale, int64_t num_tokens, int64_t max_tokens,
                          int64_t recv_capacity, void* const* rank_areas, int rank, int world,
                          int shards_per_rank, void* stream) {
  A2aParams p;
  int st = a2a_params(rank_areas, rank, world, shards_per_rank, num_tokens, max_tokens, recv_capacity, &p);
  if (st != MOE_B200_OK) return st;
  if (num_tokens > 0 && (!topk_idx || !topk_w || !hidden_states || !hidden_states_scale))
    return MOE_B200_ERR_INVALID_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(hidden_states) % 16 != 0) return MOE_B200_ERR_MISALIGNED;
  p.topk_idx = topk_idx;
  p.topk_w = topk_w;
  p.hidden = static_cast<const uint8_t*>(hidden_states);
  p.hidden_scale = hidden_states_scale;
  int grid = 0;
  if ((st = a2a_grid(&grid)) != MOE_B200_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // every rank runs plan and dispatch every call, also with no tokens: the
  // ranks meet in them
  if (launch_kernel(a2a_plan_kernel, 1, kPlanThreads, 0, s, true, p) != cudaSuccess ||
      launch_kernel(a2a_dispatch_kernel, grid, kA2aThreads, 0, s, true, p) != cudaSuccess)
    return MOE_B200_ERR_CUDA;
  return MOE_B200_OK;
}

int moe_b200_a2a_combine(const int32_t* topk_idx, void* const* shard_workspaces, void* const* rank_areas, int rank,
                         int world, int shards_per_rank, int64_t num_tokens, int64_t max_tokens,
                         int64_t recv_capacity, void* output, void* stream) {
  A2aParams p;
  int st = a2a_params(rank_areas, rank, world, shards_per_rank, num_tokens, max_tokens, recv_capacity, &p);
  if (st != MOE_B200_OK) return st;
  if (shard_workspaces == nullptr || (num_tokens > 0 && (!topk_idx || !output))) return MOE_B200_ERR_INVALID_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(output) % 16 != 0) return MOE_B200_ERR_MISALIGNED;
  // every shard's layer ran on recv_capacity rows of up to 8 given picks
  moe_b200_workspace_layout l;
  if (moe_b200_get_routed_workspace_layout(recv_capacity, kTopK, &l) != MOE_B200_OK)
    return MOE_B200_ERR_INVALID_ARGUMENT;
  for (int q = 0; q < world * shards_per_rank; ++q) {
    uint8_t* ws = static_cast<uint8_t*>(shard_workspaces[q]);
    if (ws == nullptr) return MOE_B200_ERR_INVALID_ARGUMENT;
    if (reinterpret_cast<uintptr_t>(ws) % 256 != 0) return MOE_B200_ERR_MISALIGNED;
    p.y[q] = reinterpret_cast<const float*>(ws + l.y_acc);
    p.slot[q] = recv_capacity <= kDecodeMaxTokens ? nullptr : reinterpret_cast<const int32_t*>(ws + l.tok_slot);
  }
  p.topk_idx = topk_idx;
  p.out = static_cast<uint16_t*>(output);
  int grid = 0;
  if ((st = a2a_grid(&grid)) != MOE_B200_OK) return st;
  if (launch_kernel(a2a_combine_kernel, grid, kA2aThreads, 0, static_cast<cudaStream_t>(stream), true, p) !=
      cudaSuccess)
    return MOE_B200_ERR_CUDA;
  return MOE_B200_OK;
}

int moe_b200_a2a_read_status(const void* area, uint32_t* status, int32_t* recv_rows, void* stream) {
  if (area == nullptr || status == nullptr) return MOE_B200_ERR_INVALID_ARGUMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint32_t v[2] = {0u, 0u};
  static_assert(A2aCounters::kRecvRows == A2aCounters::kStatus + 4, "status and row count are adjacent");
  if (cudaMemcpyAsync(v, static_cast<const uint8_t*>(area) + A2aCounters::kStatus, sizeof(v),
                      cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return MOE_B200_ERR_CUDA;
  *status = v[0];
  if (recv_rows != nullptr) *recv_rows = static_cast<int32_t>(v[1]);
  return v[0] == 0 ? MOE_B200_OK : MOE_B200_ERR_DEVICE_TIMEOUT;
}

}  // extern "C"
