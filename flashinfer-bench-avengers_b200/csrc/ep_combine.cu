// Expert-parallel combine over NVLink peer memory.
//
// With expert parallelism every rank runs the layer on the same tokens for
// its own expert shards (one moe_b200_run per 32-expert shard, each with its
// own workspace) and leaves the fp32 combine rows in those workspaces
// (output = NULL). This kernel then forms the bf16 output of the whole layer
// on every rank in one launch:
//   0. with several shards per rank, sum this rank's shards' rows in shard
//      order into one fp32 row per token (its partial sum; local work, so
//      that step 2 reads one partial per rank over NVLink instead of every
//      shard's rows), and count the CTA when done;
//   1. announce "my combine rows are final" to every peer (a release store at
//      system scope of a call counter into the peer's flag array, once every
//      CTA of this rank has counted itself in step 0) and wait (bounded)
//      until every peer has announced;
//   2. reduce this rank's 1/W slice of the token rows: for each row, the fp32
//      rows of every shard of every rank (or every rank's partial sum) are
//      read (plain loads of peer memory over NVLink for the other ranks'),
//      summed in fp32 (each rank's shards in shard order, then the ranks in
//      rank order) and rounded once to bf16; the result is stored into this
//      rank's output and into the output staging area of every other rank
//      (plain stores to peer memory) -- reduce-scatter and all-gather in one
//      pass, with the sum formed before the single bf16 rounding;
//   3. count this CTA locally (after a system-scope fence over its peer
//      stores); the last CTA of the rank to finish tells every rank with one
//      release reduction at system scope; wait (bounded) until every rank
//      has told this rank, and copy the other ranks' rows from the staging
//      area to the caller's output.
// With one rank (all shards on one GPU) only the reduction runs, straight
// into the output, and the counters are not touched.
// Decode-size calls (at most kEpLLMaxTokens tokens) on two or more ranks use
// flagged lines instead of steps 1-3, so that no fence or counter sits on the
// critical path (the fences and the two all-rank counts cost about 20 us at
// 64 tokens, against a few microseconds of data): every 16-byte line carries
// two 4-byte values, each followed by the call number, stored with one
// 16-byte store and polled with one 16-byte load until both flags read the
// call number (the scheme of NCCL's LL protocol).
//   A. each rank sums its own shards' rows that another rank owns and stores
//      them, as flagged fp32 lines, into the owner's receive slot for it;
//   B. each rank forms its own rows: the ranks' partial sums in rank order
//      (its own from its shards, the others' polled from its receive slots),
//      one bf16 rounding, into its output and, as flagged bf16 lines, into
//      every other rank's receive rows;
//   C. each rank polls its receive rows for the other ranks' rows and copies
//      them into its output.
// A rank overwrites a peer's receive area for call c + 1 only after its own
// call c has completed, which needed every line the peer had to read for
// call c, so one receive area per rank suffices.
// The call number grows (it is kept in the EP area); the per-call counters
// are cleared by the last CTA of each call, once no CTA of the call still
// waits and before this rank can announce the next call, so nothing has to
// be cleared between calls, the grid may follow the token count, and the
// sequence can be captured in a CUDA graph. No multicast and no library
// kernel touches peer memory; every wait
// gives up after one second with a status bit instead of hanging. A wait that
// gives up leaves the ranks' counters out of step, so it also marks every
// rank's area as poisoned: every later combine on those areas returns at once
// with a status bit, until every rank has zeroed its whole area (the
// counter block and the flagged lines, whose call numbers restart).
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

constexpr uint32_t kStatusTimeoutPeer = 1u << 7;   // a peer never announced / wrote its slice
constexpr uint32_t kStatusPoisoned = 1u << 8;      // an earlier combine on these areas gave up a wait
constexpr int kEpMaxRanks = 8;
constexpr int kEpMaxSources = 8;                   // shards summed by one combine, over all ranks
constexpr int kEpThreads = 256;
// CTAs of the combine per SM. All of them must be resident at once (they
// wait for each other), which __launch_bounds__ guarantees for two 256-thread
// CTAs per SM when nothing else runs on the device.
constexpr int kEpCtasPerSm = 2;
// Calls with at most this many tokens use the flagged-line protocol.
constexpr int kEpLLMaxTokens = kDecodeMaxTokens;
constexpr int kLLPartLines = kHidden / 2;                 // flagged fp32 lines per row (2 values each)
constexpr int kLLOutLines = kHidden / 4;                  // flagged bf16 lines per row (4 values each)
constexpr int kLLPartRows = kEpLLMaxTokens + kEpMaxRanks;  // W slots of ceil(T / W) rows
constexpr int kLLPollGroup = 4;                            // peers whose lines are loaded together

// Layout of a rank's expert-parallel area (moe_b200_ep_area_bytes): the
// counters and the flagged-line buffers sit at fixed offsets, so calls with
// different token counts find them in the same place. Bytes [0, kCounters)
// are the counter block.
struct EpArea {
  static constexpr size_t kFlags = 0;       // int32[kEpMaxRanks]: call number announced by each rank
  static constexpr size_t kDone = 64;       // int32: ranks that finished writing into this staging (this call)
  static constexpr size_t kFinished = 68;   // int32: CTAs of this rank that finished this call
  static constexpr size_t kCalls = 72;      // int32: completed calls of this rank
  static constexpr size_t kPoison = 76;     // int32: nonzero once a combine on these areas gave up a wait
  static constexpr size_t kWritten = 80;    // int32: CTAs of this rank that finished writing (this call)
  static constexpr size_t kSummed = 84;     // int32: CTAs of this rank that finished its shard sums (this call)
  static constexpr size_t kCounters = 256;  // end of the counter block
  // flagged-line protocol: fp32 partial rows received from each rank (slot
  // r at row r * ceil(T / W)), then the bf16 rows received from their owners
  static constexpr size_t kLLPart = kCounters;
  static constexpr size_t kLLOut = kLLPart + static_cast<size_t>(kLLPartRows) * kLLPartLines * 16;
  static constexpr size_t kStage = kLLOut + static_cast<size_t>(kEpLLMaxTokens) * kLLOutLines * 16;   // bf16[T, 7168] output staging
};
static_assert(EpArea::kCounters == MOE_B200_EP_COUNTER_BYTES, "counter block size in the header");
static_assert(EpArea::kStage % 256 == 0, "staging alignment");

struct EpParams {
  uint8_t* area[kEpMaxRanks];          // each rank's EP area (this process's mapping)
  const float* y[kEpMaxSources];       // each shard's fp32 combine rows, rank-major
  const int32_t* slot[kEpMaxSources];  // each shard's token -> combine row map, null: row = token
  // Staged protocol with several shards per rank: each rank's fp32 sum of
  // its own shards' rows, one row per token, in a region of its first shard
  // workspace that the layer no longer needs (the permuted activation copy)
  float* partial[kEpMaxRanks];
  uint16_t* out;                       // this rank's output, bf16 [T, 7168]
  uint32_t* status;                    // this rank's status word
  int rank, world, sources, num_tokens;
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

// Spins (bounded) until *p has reached target. The counters only grow and
// wrap around after 2^32 increments, so "reached" is a signed difference,
// valid while the two are less than 2^31 apart. Returns false on timeout.
__device__ __forceinline__ bool wait_at_least(const int* p, uint32_t target) {
  const uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (static_cast<int32_t>(static_cast<uint32_t>(ld_acquire_sys(p)) - target) < 0) {
    if ((++spins & 63u) == 0u && globaltimer_ns() - t0 > kWaitBudgetNs) return false;
  }
  return true;
}

// Column quads of a row: item (t, j) covers columns 4j .. 4j+3 and
// 3584+4j .. +3 of token t; consecutive threads take consecutive j, so every
// load instruction of a warp reads 512 contiguous bytes.
struct Bf16Quads {
  uint2 a, b;
};

__device__ __forceinline__ uint2 pack_bf16x4(float x, float y, float z, float w) {
  const __nv_bfloat162 lo = __floats2bfloat162_rn(x, y);
  const __nv_bfloat162 hi = __floats2bfloat162_rn(z, w);
  return make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
}

constexpr int kHalfQuads = kHidden / 8;   // 896: quads per half row

struct F32Quads {
  float4 a, b;
};

// The fp32 sums (before rounding) of columns 4j .. 4j+3 and 3584+4j .. +3
// of token t's rows over `n` sources: the shards q0 .. q0 + n - 1 (row map
// p.slot), or with kPartials the ranks' partial sums (row = token). Every
// source's row index and data are loaded before the sum (up to 16 loads in
// flight per thread); absent rows add +0.0, which leaves the sum's bits as
// they are (the sum starts at +0.0). Sources are summed in groups of
// `group` (one rank's shards, in shard order), then the groups in order;
// with one group, or groups of one, this is the plain sum in source order.
template <bool kPartials>
__device__ __forceinline__ F32Quads sum_quads(const EpParams& p, int t, int j, int q0, int n, int group) {
  int row[kEpMaxSources];
#pragma unroll
  for (int q = 0; q < kEpMaxSources; ++q) {
    if constexpr (kPartials) {
      row[q] = q < n ? t : -1;
    } else {
      row[q] = q < n ? (p.slot[q0 + q] != nullptr ? __ldg(p.slot[q0 + q] + t) : t) : -1;
    }
  }
  float4 u[kEpMaxSources], v[kEpMaxSources];
#pragma unroll
  for (int q = 0; q < kEpMaxSources; ++q) {
    u[q] = make_float4(0.f, 0.f, 0.f, 0.f);
    v[q] = u[q];
    if (row[q] >= 0) {
      const float* base = kPartials ? p.partial[q] : p.y[q0 + q];
      const float4* src = reinterpret_cast<const float4*>(base + static_cast<int64_t>(row[q]) * kHidden);
      u[q] = src[j];
      v[q] = src[kHalfQuads + j];
    }
  }
  float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  float b[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  int in_group = 0;
#pragma unroll
  for (int q = 0; q < kEpMaxSources; ++q) {
    b[0] += u[q].x; b[1] += u[q].y; b[2] += u[q].z; b[3] += u[q].w;
    b[4] += v[q].x; b[5] += v[q].y; b[6] += v[q].z; b[7] += v[q].w;
    if (q < n && ++in_group == group) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        a[i] += b[i];
        b[i] = 0.f;
      }
      in_group = 0;
    }
  }
  return {make_float4(a[0], a[1], a[2], a[3]), make_float4(a[4], a[5], a[6], a[7])};
}

__device__ __forceinline__ Bf16Quads round_quads(const F32Quads& f) {
  return {pack_bf16x4(f.a.x, f.a.y, f.a.z, f.a.w), pack_bf16x4(f.b.x, f.b.y, f.b.z, f.b.w)};
}

// The bf16 rounding of the sum over every shard of every rank: each rank's
// shards in shard order, then the ranks in rank order.
__device__ __forceinline__ Bf16Quads reduce_quads(const EpParams& p, int t, int j) {
  return round_quads(sum_quads<false>(p, t, j, 0, p.sources, p.sources / p.world));
}

// Stores the two results into a bf16 [T, 7168] row-major destination.
__device__ __forceinline__ void store_quads(uint8_t* dst, int t, int j, const Bf16Quads& o) {
  uint2* row = reinterpret_cast<uint2*>(dst + static_cast<int64_t>(t) * kHidden * 2);
  row[j] = o.a;
  row[kHalfQuads + j] = o.b;
}

// A wait gave up: record it and poison every rank's area, so that no later
// combine runs on counters (or flagged lines) that are out of step.
__device__ __forceinline__ void give_up(const EpParams& p) {
  atomicOr(p.status, kStatusTimeoutPeer);
  for (int q = 0; q < p.world; ++q) st_release_sys(reinterpret_cast<int*>(p.area[q] + EpArea::kPoison), 1);
}

// One flagged line: values a and b, each followed by the call number.
__device__ __forceinline__ void st_line(uint8_t* dst, uint32_t a, uint32_t b, uint32_t flag) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(dst), "r"(a), "r"(flag), "r"(b), "r"(flag)
               : "memory");
}

// One load of a flagged line (values in x and z, flags in y and w).
__device__ __forceinline__ uint4 ld_line_once(const uint8_t* src) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(src)
               : "memory");
  return v;
}

// Polls a flagged line until both of its flags read `flag`; false once the
// deadline (globaltimer) has passed.
__device__ __forceinline__ bool ld_line(const uint8_t* src, uint32_t flag, uint64_t deadline, uint32_t& a,
                                        uint32_t& b) {
  for (uint32_t spins = 1;; ++spins) {
    uint32_t x, f0, y, f1;
    asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(x), "=r"(f0), "=r"(y), "=r"(f1)
                 : "l"(src)
                 : "memory");
    if (f0 == flag && f1 == flag) {
      a = x;
      b = y;
      return true;
    }
    if ((spins & 63u) == 0u && globaltimer_ns() > deadline) return false;
  }
}

// Rows [row_lo(q), row_lo(q + 1)) of the T tokens belong to rank q.
__device__ __forceinline__ int row_lo(int q, int T, int W) {
  return static_cast<int>(static_cast<int64_t>(T) * q / W);
}

__device__ __forceinline__ int row_owner(int t, int T, int W) {
  int q = static_cast<int>(static_cast<int64_t>(t) * W / T);
  while (row_lo(q + 1, T, W) <= t) ++q;
  while (row_lo(q, T, W) > t) --q;
  return q;
}

// Flagged-line protocol (see the top of this file) for W >= 2 ranks and
// T <= kEpLLMaxTokens; decode-size combine rows are indexed by token.
// Returns false after giving up a wait (status set, areas poisoned).
__device__ bool combine_lines(const EpParams& p, uint32_t call, int first, int stride) {
  const int W = p.world, T = p.num_tokens, me = p.rank;
  const int S = p.sources / W;   // shards per rank
  const int mlo = row_lo(me, T, W), mhi = row_lo(me + 1, T, W);
  const int nmine = mhi - mlo;
  const int slot_rows = (T + W - 1) / W;
  const uint64_t deadline = globaltimer_ns() + kWaitBudgetNs;
  uint8_t* out = reinterpret_cast<uint8_t*>(p.out);
  uint8_t* mine = p.area[me];

  // ---- A. my partial sums of the other ranks' rows -> their receive slots
  const int items_a = (T - nmine) * kLLPartLines;
  for (int it = first; it < items_a; it += stride) {
    const int r = it / kLLPartLines;
    const int line = it - r * kLLPartLines;
    const int t = r < mlo ? r : r + nmine;
    const int q = row_owner(t, T, W);
    float2 v = make_float2(0.f, 0.f);
    for (int s = 0; s < S; ++s) {
      const float2 y = reinterpret_cast<const float2*>(p.y[me * S + s] + static_cast<int64_t>(t) * kHidden)[line];
      v.x += y.x;
      v.y += y.y;
    }
    uint8_t* dst = p.area[q] + EpArea::kLLPart +
                   (static_cast<size_t>(me * slot_rows + (t - row_lo(q, T, W))) * kLLPartLines + line) * 16;
    st_line(dst, __float_as_uint(v.x), __float_as_uint(v.y), call);
  }

  // ---- B. my rows: sum of the ranks' partials in rank order, one rounding
  const int items_b = nmine * kLLOutLines;
  for (int it = first; it < items_b; it += stride) {
    const int rr = it / kLLOutLines;
    const int line = it - rr * kLLOutLines;   // columns 4 line .. 4 line + 3
    const int t = mlo + rr;
    float a[4] = {0.f, 0.f, 0.f, 0.f};
    // Ranks in groups of four: the lines of a group's peers are all loaded
    // before any flag is checked (one round trip per group instead of one
    // per line); only lines not yet written are polled again.
    for (int r0 = 0; r0 < W; r0 += kLLPollGroup) {
      uint4 l0[kLLPollGroup], l1[kLLPollGroup];
#pragma unroll
      for (int i = 0; i < kLLPollGroup; ++i) {
        const int r = r0 + i;
        if (r < W && r != me) {
          const uint8_t* src =
              mine + EpArea::kLLPart + (static_cast<size_t>(r * slot_rows + rr) * kLLPartLines + 2 * line) * 16;
          l0[i] = ld_line_once(src);
          l1[i] = ld_line_once(src + 16);
        }
      }
#pragma unroll
      for (int i = 0; i < kLLPollGroup; ++i) {
        const int r = r0 + i;
        if (r >= W) continue;
        float v[4];
        if (r == me) {
          v[0] = v[1] = v[2] = v[3] = 0.f;
          for (int s = 0; s < S; ++s) {
            const float4 y =
                reinterpret_cast<const float4*>(p.y[me * S + s] + static_cast<int64_t>(t) * kHidden)[line];
            v[0] += y.x;
            v[1] += y.y;
            v[2] += y.z;
            v[3] += y.w;
          }
        } else {
          const uint8_t* src =
              mine + EpArea::kLLPart + (static_cast<size_t>(r * slot_rows + rr) * kLLPartLines + 2 * line) * 16;
          uint32_t x0 = l0[i].x, x1 = l0[i].z, x2 = l1[i].x, x3 = l1[i].z;
          if (!(l0[i].y == call && l0[i].w == call) && !ld_line(src, call, deadline, x0, x1)) return false;
          if (!(l1[i].y == call && l1[i].w == call) && !ld_line(src + 16, call, deadline, x2, x3)) return false;
          v[0] = __uint_as_float(x0);
          v[1] = __uint_as_float(x1);
          v[2] = __uint_as_float(x2);
          v[3] = __uint_as_float(x3);
        }
        a[0] += v[0];
        a[1] += v[1];
        a[2] += v[2];
        a[3] += v[3];
      }
    }
    const uint2 o = pack_bf16x4(a[0], a[1], a[2], a[3]);
    reinterpret_cast<uint2*>(out + static_cast<int64_t>(t) * kHidden * 2)[line] = o;
    for (int q = 0; q < W; ++q)
      if (q != me)
        st_line(p.area[q] + EpArea::kLLOut + (static_cast<size_t>(t) * kLLOutLines + line) * 16, o.x, o.y, call);
  }

  // ---- C. the other ranks' rows from my receive rows
  const int items_c = (T - nmine) * kLLOutLines;
  for (int it = first; it < items_c; it += stride) {
    const int r = it / kLLOutLines;
    const int line = it - r * kLLOutLines;
    const int t = r < mlo ? r : r + nmine;
    uint2 o;
    if (!ld_line(mine + EpArea::kLLOut + (static_cast<size_t>(t) * kLLOutLines + line) * 16, call, deadline, o.x, o.y))
      return false;
    reinterpret_cast<uint2*>(out + static_cast<int64_t>(t) * kHidden * 2)[line] = o;
  }
  return true;
}

// Steps 1-3 (see the top of this file) for W >= 2 ranks. Returns the same
// value in every thread of the CTA: false after giving up a wait (status set,
// areas poisoned).
__device__ bool combine_staged(const EpParams& p, uint32_t call, int first, int stride, int& s_ok) {
  const int W = p.world;
  const int T = p.num_tokens;
  uint8_t* out = reinterpret_cast<uint8_t*>(p.out);
  uint8_t* mine = p.area[p.rank];
  const int S = p.sources / W;
  if (threadIdx.x == 0) s_ok = 1;
  // ---- 0. this rank's shard sums, one fp32 row per token ------------------
  if (S > 1) {
    float* dst = p.partial[p.rank];
    const int n = T * kHalfQuads;
    for (int it = first; it < n; it += stride) {
      const int t = it / kHalfQuads;
      const int j = it - t * kHalfQuads;
      const F32Quads v = sum_quads<false>(p, t, j, p.rank * S, S, S);
      float4* row = reinterpret_cast<float4*>(dst + static_cast<int64_t>(t) * kHidden);
      row[j] = v.a;
      row[kHalfQuads + j] = v.b;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence_system();   // peers read the partial sums after the announcement
      red_release_gpu_add(reinterpret_cast<int*>(mine + EpArea::kSummed), 1);
    }
  }
  // ---- 1. announce and wait for every rank -------------------------------
  __syncthreads();
  if (blockIdx.x == 0 && threadIdx.x < W) {
    if (S > 1 && !wait_at_least(reinterpret_cast<const int*>(mine + EpArea::kSummed), gridDim.x)) {
      give_up(p);
      s_ok = 0;
    } else {
      st_release_sys(reinterpret_cast<int*>(p.area[threadIdx.x] + EpArea::kFlags) + p.rank, static_cast<int>(call));
    }
  }
  if (threadIdx.x < W &&
      !wait_at_least(reinterpret_cast<const int*>(mine + EpArea::kFlags) + threadIdx.x, call)) {
    give_up(p);
    s_ok = 0;
  }
  __syncthreads();
  if (!s_ok) return false;

  // ---- 2. reduce this rank's rows: into its own output, and into every
  //         peer's staging area ---------------------------------------------
  const int r0 = static_cast<int>(static_cast<int64_t>(T) * p.rank / W);
  const int r1 = static_cast<int>(static_cast<int64_t>(T) * (p.rank + 1) / W);
  const int items = (r1 - r0) * kHalfQuads;
  for (int it = first; it < items; it += stride) {
    const int rel = it / kHalfQuads;
    const int t = r0 + rel;
    const int j = it - rel * kHalfQuads;
    // one partial sum per rank (step 0), or every shard's rows
    const Bf16Quads o = S > 1 ? round_quads(sum_quads<true>(p, t, j, 0, W, 1)) : reduce_quads(p, t, j);
    store_quads(out, t, j, o);
    for (int q = 0; q < W; ++q)
      if (q != p.rank) store_quads(p.area[q] + EpArea::kStage, t, j, o);
  }

  // ---- 3. count this CTA locally; the last CTA of this rank to finish
  //         writing tells every rank (one release per peer); wait until every
  //         rank has written this rank's staging, copy the other ranks' rows
  //         out of it -------------------------------------------------------
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();   // this CTA's peer stores are visible system-wide
    const int before = atom_add_acq_rel_gpu(reinterpret_cast<int*>(mine + EpArea::kWritten), 1);
    if (before == static_cast<int>(gridDim.x) - 1) {
      __threadfence_system();
      for (int q = 0; q < W; ++q) red_release_sys_add(reinterpret_cast<int*>(p.area[q] + EpArea::kDone), 1);
    }
    if (!wait_at_least(reinterpret_cast<const int*>(mine + EpArea::kDone), static_cast<uint32_t>(W))) {
      give_up(p);
      s_ok = 0;
    }
  }
  __syncthreads();
  if (s_ok) {
    // 16-byte units, 896 per row: everything but this rank's rows
    const uint4* stage = reinterpret_cast<const uint4*>(mine + EpArea::kStage);
    uint4* out16 = reinterpret_cast<uint4*>(out);
    const int lo = r0 * kHalfQuads, hi = r1 * kHalfQuads;
    const int n16 = T * kHalfQuads - (hi - lo);
    for (int i = first; i < n16; i += stride) {
      const int k = i < lo ? i : i + (hi - lo);
      out16[k] = stage[k];
    }
  }
  return s_ok != 0;
}

}  // namespace

__global__ void __launch_bounds__(kEpThreads, kEpCtasPerSm) ep_combine_kernel(EpParams p) {
  __shared__ int s_ok;
  __shared__ int s_poisoned;
  pdl_wait();   // this rank's layer calls (their GEMM2 reductions) have completed
  const int W = p.world;
  const int T = p.num_tokens;
  // items (a token row and a quad index j < 896) fit in int32: T <= 2^18
  const int stride = static_cast<int>(gridDim.x) * kEpThreads;
  const int first = static_cast<int>(blockIdx.x) * kEpThreads + static_cast<int>(threadIdx.x);
  uint8_t* out = reinterpret_cast<uint8_t*>(p.out);

  if (W == 1) {   // one rank: a plain reduction of its shards into the output
    const int items = T * kHalfQuads;
    for (int it = first; it < items; it += stride) {
      const int t = it / kHalfQuads;
      const int j = it - t * kHalfQuads;
      store_quads(out, t, j, reduce_quads(p, t, j));
    }
    return;
  }

  uint8_t* mine = p.area[p.rank];
  // one read for the whole CTA: a peer may poison the area meanwhile, and
  // every thread must take the same path (barriers below)
  if (threadIdx.x == 0) s_poisoned = *reinterpret_cast<volatile int*>(mine + EpArea::kPoison) != 0;
  __syncthreads();
  if (s_poisoned) {
    if (threadIdx.x == 0) atomicOr(p.status, kStatusPoisoned);
    return;
  }
  const uint32_t call = *reinterpret_cast<volatile uint32_t*>(mine + EpArea::kCalls) + 1u;

  bool ok;
  if (T <= kEpLLMaxTokens) {
    ok = combine_lines(p, call, first, stride);
    if (!ok) give_up(p);
    ok = __syncthreads_or(ok ? 0 : 1) == 0;
  } else {
    ok = combine_staged(p, call, first, stride, s_ok);
  }
  if (!ok) return;
  // The last CTA of this rank to finish clears the per-call counters and
  // advances the call number: every CTA has passed its waits by then, and no
  // peer writes this area for the next call before this rank announces it.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const int f = atom_add_acq_rel_gpu(reinterpret_cast<int*>(mine + EpArea::kFinished), 1) + 1;
    if (f == static_cast<int>(gridDim.x)) {
      *reinterpret_cast<volatile int*>(mine + EpArea::kWritten) = 0;
      *reinterpret_cast<volatile int*>(mine + EpArea::kDone) = 0;
      *reinterpret_cast<volatile int*>(mine + EpArea::kFinished) = 0;
      *reinterpret_cast<volatile int*>(mine + EpArea::kSummed) = 0;
      __threadfence();
      *reinterpret_cast<volatile uint32_t*>(mine + EpArea::kCalls) = call;
    }
  }
}

}  // namespace moe

using namespace moe;

extern "C" {

size_t moe_b200_ep_area_bytes(int64_t num_tokens) {
  if (num_tokens < 0 || num_tokens > MOE_B200_MAX_TOKENS) return 0;
  return EpArea::kStage + (static_cast<size_t>(num_tokens) * kHidden * 2 + 255) / 256 * 256;
}

int moe_b200_ep_combine_shards(void* const* shard_workspaces, int shards_per_rank, void* const* rank_areas,
                               int rank, int world, int64_t num_tokens, void* output, void* stream) {
  if (shard_workspaces == nullptr || rank_areas == nullptr || output == nullptr || world < 1 ||
      world > kEpMaxRanks || shards_per_rank < 1 || world * shards_per_rank > kEpMaxSources || rank < 0 ||
      rank >= world || num_tokens < 0 || num_tokens > MOE_B200_MAX_TOKENS)
    return MOE_B200_ERR_INVALID_ARGUMENT;
  if (num_tokens == 0) return MOE_B200_OK;
  moe_b200_workspace_layout l;
  if (moe_b200_get_workspace_layout(num_tokens, &l) != MOE_B200_OK) return MOE_B200_ERR_INVALID_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(output) % 16 != 0) return MOE_B200_ERR_MISALIGNED;
  const int sources = world * shards_per_rank;
  EpParams p;
  for (int q = 0; q < kEpMaxRanks; ++q) p.area[q] = nullptr;
  for (int q = 0; q < kEpMaxSources; ++q) {
    p.y[q] = nullptr;
    p.slot[q] = nullptr;
  }
  for (int q = 0; q < world; ++q) {
    uint8_t* area = static_cast<uint8_t*>(rank_areas[q]);
    if (area == nullptr) return MOE_B200_ERR_INVALID_ARGUMENT;
    if (reinterpret_cast<uintptr_t>(area) % 256 != 0) return MOE_B200_ERR_MISALIGNED;
    p.area[q] = area;
  }
  for (int q = 0; q < sources; ++q) {
    uint8_t* ws = static_cast<uint8_t*>(shard_workspaces[q]);
    if (ws == nullptr) return MOE_B200_ERR_INVALID_ARGUMENT;
    if (reinterpret_cast<uintptr_t>(ws) % 256 != 0) return MOE_B200_ERR_MISALIGNED;
    p.y[q] = reinterpret_cast<const float*>(ws + l.y_acc);
    // decode-size calls keep one combine row per token
    p.slot[q] = num_tokens <= kDecodeMaxTokens ? nullptr : reinterpret_cast<const int32_t*>(ws + l.tok_slot);
  }
  for (int q = 0; q < kEpMaxRanks; ++q)
    p.partial[q] = q < world ? reinterpret_cast<float*>(static_cast<uint8_t*>(shard_workspaces[q * shards_per_rank]) +
                                                        l.a_perm)
                             : nullptr;
  static_assert(sizeof(float) * kHidden <= 8 * kHidden, "a_perm holds one fp32 row per token");
  p.out = static_cast<uint16_t*>(output);
  // this rank's first shard workspace holds the status word the caller reads
  p.status = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(shard_workspaces[rank * shards_per_rank]) +
                                         l.status);
  p.rank = rank;
  p.world = world;
  p.sources = sources;
  p.num_tokens = static_cast<int>(num_tokens);
  // One thread per reduced item (a row's column quads j and 896 + j), at most
  // two CTAs per SM (all resident at once: they wait on the peers). The
  // per-call counters are cleared at the end of every call, so the grid may
  // differ between calls.
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
    return MOE_B200_ERR_CUDA;
  // (flagged lines: one thread per line of the rows this rank sends, about
  // T * 3584 lines, as the largest of the three phases)
  const int64_t rows_per_rank = (num_tokens + world - 1) / world;
  const int64_t items = (world > 1 && num_tokens <= kEpLLMaxTokens) ? num_tokens * kLLPartLines
                                                                     : rows_per_rank * (kHidden / 8);
  const int64_t want = (items + kEpThreads - 1) / kEpThreads;
  const int grid = static_cast<int>(want < kEpCtasPerSm * sms ? (want > 0 ? want : 1) : kEpCtasPerSm * sms);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (launch_kernel(ep_combine_kernel, grid, kEpThreads, 0, s, true, p) != cudaSuccess)
    return MOE_B200_ERR_CUDA;
  return MOE_B200_OK;
}

int moe_b200_ep_combine(void* const* rank_workspaces, void* const* rank_areas, int rank, int world,
                        int64_t num_tokens, void* output, void* stream) {
  return moe_b200_ep_combine_shards(rank_workspaces, 1, rank_areas, rank, world, num_tokens, output, stream);
}

// ---- device buffers shared between processes (CUDA IPC) -------------------

int moe_b200_ep_buffer_alloc(size_t bytes, void** ptr) {
  if (ptr == nullptr || bytes == 0) return MOE_B200_ERR_INVALID_ARGUMENT;
  *ptr = nullptr;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) {
    cudaGetLastError();
    return MOE_B200_ERR_CUDA;
  }
  if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
    cudaFree(p);
    return MOE_B200_ERR_CUDA;
  }
  *ptr = p;
  return MOE_B200_OK;
}

int moe_b200_ep_buffer_free(void* ptr) {
  if (ptr == nullptr) return MOE_B200_OK;
  return cudaFree(ptr) == cudaSuccess ? MOE_B200_OK : MOE_B200_ERR_CUDA;
}

int moe_b200_ipc_get_handle(const void* buffer, void* handle) {
  if (buffer == nullptr || handle == nullptr) return MOE_B200_ERR_INVALID_ARGUMENT;
  static_assert(sizeof(cudaIpcMemHandle_t) == MOE_B200_IPC_HANDLE_BYTES, "IPC handle size in the header");
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, const_cast<void*>(buffer)) != cudaSuccess) {
    cudaGetLastError();
    return MOE_B200_ERR_CUDA;
  }
  memcpy(handle, &h, sizeof(h));
  return MOE_B200_OK;
}

int moe_b200_ipc_open_handle(const void* handle, void** buffer) {
  if (handle == nullptr || buffer == nullptr) return MOE_B200_ERR_INVALID_ARGUMENT;
  *buffer = nullptr;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
    cudaGetLastError();
    return MOE_B200_ERR_CUDA;
  }
  *buffer = p;
  return MOE_B200_OK;
}

int moe_b200_ipc_close_handle(void* buffer) {
  if (buffer == nullptr) return MOE_B200_OK;
  return cudaIpcCloseMemHandle(buffer) == cudaSuccess ? MOE_B200_OK : MOE_B200_ERR_CUDA;
}

}  // extern "C"
