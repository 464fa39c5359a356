// Grouped FP8 block-scale GEMMs of the MoE layer on sm_100a tensor cores.
//
// Orientation ("swap-AB"): the MMA's M side is 128 weight rows of one
// expert, its N side is a tile of BN permuted token rows, both operands are
// e4m3 and K-major in shared memory with the 128-byte swizzle. One 128-wide
// K block is four tcgen05.mma (K = 32 each) into a fresh TMEM accumulator;
// the epilogue warps then fold it into fp32 registers with the block scale of
// that K block (weight scale, a scalar for the whole tile, times the
// activation scale, one per token column). That promotion is what the
// reference does for GEMM1 (solution/cuda/kernel.cu:784-832); here it runs
// out of a double-buffered TMEM accumulator, so the MMA of block k+1 overlaps
// the promotion of block k.
//
// Roles (one CTA per SM, persistent over a static tile list):
//   warp 0        TMA producer: weight tiles and permuted token rows (2-D
//                 TMA), block scales (one bulk copy + cp.async per K block)
//   warp 1        TMEM owner and single-thread MMA issuer
//   warp 2        scale combiner: weight scale x activation scale per column
//   warp 3        spare (keeps the epilogue warpgroup-aligned)
//   warps 4..     epilogue: TMEM -> registers, promotion, final epilogue;
//                 4 or 8 warps, each owning one TMEM lane quarter and a
//                 group of token columns
//
// GEMM1 computes, for 128 intermediate rows i of block `blk`, both
//   up[i]   = W13[e, blk*128 + i, :]        . A[tok, :]
//   gate[i] = W13[e, 2048 + blk*128 + i, :] . A[tok, :]
// and its fused epilogue writes C = silu(gate) * up (reference semantics,
// solution/cuda/kernel.h:207) as two e4m3 operands C = s * (hi + lo) with
// s = amax/448 per (row, 128-block) -- the residual lo keeps ~8 significant
// bits, so GEMM2 sees C at close to bf16 precision while staying on the
// e4m3 tensor-core path.
// GEMM2 computes O[h] = W2[e, h, :] . C[row, :] (hi and lo accumulate into
// one TMEM accumulator) and red.adds w * O into the fp32 output rows; its
// wide form covers two 128-row W2 blocks per tile (M = 256), which cuts the
// token-tile traffic per FLOP by a third.
#include <cuda.h>
#include <cuda_fp8.h>
#include <cstdint>

#include "gemm_sm100.h"
#include "moe_kernels.cuh"
#include "moe_ptx.cuh"
#include "moe_shapes.cuh"
#include "swiglu.cuh"

namespace moe {

template <int kKind, int BN, int kStages, int kEpiWarps_>
struct GemmTraits {
  static constexpr bool kIsG1 = kKind == kGemm1Fused || kKind == kGemm1Split;
  // weight tiles per stage: GEMM1 up + gate, GEMM2 one or two W2 row blocks
  static constexpr int kNumA = (kKind == kGemm2) ? 1 : 2;
  // token tiles per stage: GEMM1 activation rows, GEMM2 the hi and lo parts of C
  static constexpr int kNumB = kIsG1 ? 1 : 2;
  static constexpr int kATileBytes = 128 * 128;
  static constexpr int kBTileBytes = BN * 128;
  static constexpr int kStageBytes = kNumA * kATileBytes + kNumB * kBTileBytes;
  static constexpr int kKBlocks = kIsG1 ? kHiddenBlocks : kInterBlocks;
  static constexpr int kRowBlocks = kIsG1 ? kInterBlocks : kHiddenBlocks / kNumA;
  // GEMM2's hi and lo token tiles sit back to back in shared memory with the
  // same swizzled layout, so one MMA with N = 2 * BN covers both: half the
  // MMA instructions (the decode GEMM2 is issue-bound at N = 16), and the
  // epilogue adds the two column halves.
  static constexpr bool kMergeB = kNumB == 2;
  static constexpr int kMmaN = kMergeB ? 2 * BN : BN;
  static constexpr int kAccCols = kNumA * kMmaN;  // fp32 TMEM columns per accumulator buffer
  static constexpr int kTmemCols = (2 * kAccCols <= 32) ? 32
                                   : (2 * kAccCols <= 64) ? 64
                                   : (2 * kAccCols <= 128) ? 128
                                   : (2 * kAccCols <= 256) ? 256 : 512;
  // The scale ring must not be shallower than the stage ring, or it caps the
  // bytes in flight (the decode kernels are latency x bytes-in-flight bound).
  static constexpr int kScaleSlots = kStages + 4 > 8 ? kStages + 4 : 8;
  // scale slot: raw[BN] | wscale[4] | combined[kNumA][BN]
  static constexpr int kSlotFloats = BN + 4 + kNumA * BN;
  // Warps 0..3 are the role warpgroup (producer, MMA, scale combiner, one
  // spare); warps 4.. are the epilogue. Epilogue warp w reads TMEM lane
  // quarter w % 4 and the column group (w - 4) / 4.
  static constexpr int kRoleWarps = 4;
  static constexpr int kEpiWarps = kEpiWarps_;
  static constexpr int kWarpsPerQuarter = kEpiWarps / 4;
  static constexpr int kCPT = BN / kWarpsPerQuarter;   // token columns per epilogue thread
  static constexpr int kThreads = (kRoleWarps + kEpiWarps) * 32;
  static constexpr int kColsPerLane = BN >= 32 ? BN / 32 : 1;
  static constexpr uint32_t kIdesc = idesc_e4m3_f32<128, kMmaN>();
  // shared memory layout (offsets from the 1024-aligned base)
  static constexpr int kOffStages = 0;
  static constexpr int kOffRing = kStages * kStageBytes;
  static constexpr int kOffBars = kOffRing + kScaleSlots * kSlotFloats * 4;
  // Work units are handed out dynamically: the producer takes the next unit
  // from a per-call counter and passes it to the other roles through a small
  // ring (s_units + full/empty barriers).
  static constexpr int kUnitSlots = 4;
  static constexpr int kUnitConsumers = 2 + kEpiWarps;  // MMA, scale combiner, epilogue warps
  static constexpr int kNumBars = 2 * kStages + 4 + 3 * kScaleSlots + 2 * kUnitSlots;
  static constexpr int kOffMisc = kOffBars + kNumBars * 8;
  // misc: tmem base (4) | abort (4) | unit_pre[33] | seg[33] | cnt[32] | epilogue scratch
  static constexpr int kOffUnitPre = kOffMisc + 16;
  static constexpr int kOffSeg = kOffUnitPre + 34 * 4;
  static constexpr int kOffCnt = kOffSeg + 34 * 4;
  static constexpr int kOffSplits = kOffCnt + 32 * 4;
  static constexpr int kOffUnits = kOffSplits + 32 * 4;
  static constexpr int kOffEpi = kOffUnits + kUnitSlots * 4;
  // epilogue scratch (GEMM1 fused epilogue): red[4][BN] | inv[BN]
  static constexpr int kEpiBytes = (4 * BN + BN) * 4;
  static constexpr int kSmemBytes = kOffEpi + kEpiBytes + 1024;  // + alignment slack

  static_assert(BN % 16 == 0 && BN >= 16 && kMmaN <= 256 && kColsPerLane <= 2, "BN");
  static_assert(2 * kAccCols <= 512, "two accumulator buffers must fit in TMEM");
  static_assert(kEpiWarps % 4 == 0 && kCPT >= 16 && kCPT % 16 == 0, "epilogue column split");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory");
};

struct Tile {
  int e, blk, ks, tt, row0, nvalid, kb0, kb1;
};

// Unit u -> tile. Units run expert by expert; within an expert token tile
// fastest, then K slice, then row block. s_splits[e] is expert e's K slices.
template <int BN, int kKBlocks>
__device__ __forceinline__ void decode_tile(int u, const int* s_unit_pre, const int* s_seg,
                                            const int* s_cnt, const int* s_splits, Tile& t) {
  int e = 0;
#pragma unroll 1
  while (s_unit_pre[e + 1] <= u) ++e;
  const int splits = s_splits[e];
  const int cnt = s_cnt[e];
  const int nt = (cnt + BN - 1) / BN;
  int local = u - s_unit_pre[e];
  t.e = e;
  t.tt = local % nt;
  local /= nt;
  t.ks = local % splits;
  t.blk = local / splits;
  t.row0 = s_seg[e] + t.tt * BN;
  t.nvalid = min(BN, cnt - t.tt * BN);
  t.kb0 = t.ks * kKBlocks / splits;
  t.kb1 = (t.ks + 1) * kKBlocks / splits;
}

// Column-wise max over the 32 lanes of a warp for 32 columns: after the
// butterfly lane l holds the max of column l (31 shuffles instead of 160).
__device__ __forceinline__ float warp_colmax32(const float (&v)[32], int lane) {
  float a[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const bool hi = lane & 16;
    const float keep = hi ? v[16 + j] : v[j];
    const float send = hi ? v[j] : v[16 + j];
    a[j] = fmaxf(keep, __shfl_xor_sync(0xffffffffu, send, 16));
  }
  float b[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const bool hi = lane & 8;
    const float keep = hi ? a[8 + j] : a[j];
    const float send = hi ? a[j] : a[8 + j];
    b[j] = fmaxf(keep, __shfl_xor_sync(0xffffffffu, send, 8));
  }
  float c[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const bool hi = lane & 4;
    const float keep = hi ? b[4 + j] : b[j];
    const float send = hi ? b[j] : b[4 + j];
    c[j] = fmaxf(keep, __shfl_xor_sync(0xffffffffu, send, 4));
  }
  float d[2];
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const bool hi = lane & 2;
    const float keep = hi ? c[2 + j] : c[j];
    const float send = hi ? c[j] : c[2 + j];
    d[j] = fmaxf(keep, __shfl_xor_sync(0xffffffffu, send, 2));
  }
  const bool hi = lane & 1;
  const float keep = hi ? d[1] : d[0];
  const float send = hi ? d[0] : d[1];
  return fmaxf(keep, __shfl_xor_sync(0xffffffffu, send, 1));
}


// GEMM1 final epilogue: h = silu(gate) * up for the 128 intermediate columns
// of block t.blk (one per epilogue thread row) and the token columns
// col0 .. col0+CPT of this thread, written as the e4m3 pair C = s * (hi + lo)
// with s = amax / 448 per (token row, 128-block). acc0 = up, acc1 = gate;
// acc0 is overwritten. Every epilogue thread must call it (named barrier 1).
template <int BN, int CPT>
__device__ __forceinline__ void swiglu_quant_store(float (&acc0)[CPT], const float (&acc1)[CPT],
                                                   const Tile& t, int q, int col0, int lane, int et,
                                                   int row_in_tile, float* s_red, float* s_inv,
                                                   const GemmParams& p, uint32_t epi_threads) {
#pragma unroll
  for (int c = 0; c < CPT; ++c) acc0[c] = silu_mul(acc1[c], acc0[c]);
  named_bar_sync(1, epi_threads);   // the previous tile's readers of s_red / s_inv are done
#pragma unroll
  for (int g = 0; g < (CPT + 31) / 32; ++g) {
    float v[32];
#pragma unroll
    for (int c = 0; c < 32; ++c) v[c] = (g * 32 + c < CPT) ? fabsf(acc0[min(g * 32 + c, CPT - 1)]) : 0.f;
    const float m = warp_colmax32(v, lane);
    if (g * 32 + lane < CPT) s_red[q * BN + col0 + g * 32 + lane] = m;
  }
  named_bar_sync(1, epi_threads);
  if (et < BN) {
    const float amax = fmaxf(fmaxf(s_red[et], s_red[BN + et]), fmaxf(s_red[2 * BN + et], s_red[3 * BN + et]));
    s_inv[et] = amax > 0.f ? 448.0f / amax : 0.f;
    if (et < t.nvalid) p.c_scale[static_cast<int64_t>(t.blk) * p.cap + t.row0 + et] = amax * (1.0f / 448.0f);
  }
  named_bar_sync(1, epi_threads);
  const int col = t.blk * kBlk + row_in_tile;
#pragma unroll
  for (int c = 0; c < CPT; ++c) {
    if (col0 + c < t.nvalid) {
      const float x = acc0[c] * s_inv[col0 + c];
      const __nv_fp8_e4m3 qh(x);
      const float r = x - static_cast<float>(qh);
      const __nv_fp8_e4m3 ql(r);
      const int64_t off = static_cast<int64_t>(t.row0 + col0 + c) * kInter + col;
      p.c_hi[off] = qh.__x;
      p.c_lo[off] = ql.__x;
    }
  }
}

template <int kKind, int BN, int kStages, int kEpiWarps>
__global__ void __launch_bounds__(GemmTraits<kKind, BN, kStages, kEpiWarps>::kThreads, 1)
    moe_gemm_kernel(const __grid_constant__ CUtensorMap tm_w,
                    const __grid_constant__ CUtensorMap tm_b0,
                    const __grid_constant__ CUtensorMap tm_b1, const GemmParams p,
                    const int early_tables) {
  using Tr = GemmTraits<kKind, BN, kStages, kEpiWarps>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  float* ring = reinterpret_cast<float*>(smem + Tr::kOffRing);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Tr::kOffBars);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + kStages;
  uint64_t* accf_bar = bars + 2 * kStages;
  uint64_t* acce_bar = accf_bar + 2;
  uint64_t* sraw_bar = acce_bar + 2;
  uint64_t* sfull_bar = sraw_bar + Tr::kScaleSlots;
  uint64_t* sempty_bar = sfull_bar + Tr::kScaleSlots;
  uint64_t* ufull_bar = sempty_bar + Tr::kScaleSlots;
  uint64_t* uempty_bar = ufull_bar + Tr::kUnitSlots;
  volatile int* s_units = reinterpret_cast<volatile int*>(smem + Tr::kOffUnits);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + Tr::kOffMisc);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + Tr::kOffMisc + 4);
  int* s_unit_pre = reinterpret_cast<int*>(smem + Tr::kOffUnitPre);
  int* s_seg = reinterpret_cast<int*>(smem + Tr::kOffSeg);
  int* s_cnt = reinterpret_cast<int*>(smem + Tr::kOffCnt);
  int* s_splits = reinterpret_cast<int*>(smem + Tr::kOffSplits);
  float* s_red = reinterpret_cast<float*>(smem + Tr::kOffEpi);   // [4][BN]
  float* s_inv = s_red + 4 * BN;                                 // [BN]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int splits = p.splits;

  // ---------------------------------------------------------------- setup
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_w);
    prefetch_tmap(&tm_b0);
    if (!Tr::kIsG1) prefetch_tmap(&tm_b1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&full_bar[s]), 1);
      mbar_init(smem_u32(&empty_bar[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&accf_bar[b]), 1);
      mbar_init(smem_u32(&acce_bar[b]), Tr::kEpiWarps);
    }
    for (int s = 0; s < Tr::kScaleSlots; ++s) {
      mbar_init(smem_u32(&sraw_bar[s]), 2);   // bulk copy's expect_tx + one cp.async arrival
      mbar_init(smem_u32(&sfull_bar[s]), 1);
      mbar_init(smem_u32(&sempty_bar[s]), Tr::kEpiWarps);
    }
    for (int s = 0; s < Tr::kUnitSlots; ++s) {
      mbar_init(smem_u32(&ufull_bar[s]), 1);
      mbar_init(smem_u32(&uempty_bar[s]), Tr::kUnitConsumers);
    }
    *s_abort = 0;
    fence_mbar_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(s_tmem), Tr::kTmemCols);
    tmem_relinquish();
  }
  // Everything up to pdl_wait() overlaps the previous kernel's tail
  // (programmatic dependent launch). With early_tables the segment table is
  // final before this grid is launched -- the non-decode permutation has
  // completed (the kernels in between release their dependents only after
  // their own wait), and the decode front end releases its dependents only
  // after writing and fencing the table -- so it can be read here and the
  // producer issues the first stages' weight tiles, which no earlier kernel
  // writes, before waiting. Without it everything waits first.
  if (!early_tables) pdl_wait();
  if (warp == 2) {
    // per-expert tile counts -> prefix over experts of the work units
    // L2 reads: with early_tables the table may have been written by a grid
    // that is still running
    const int lo = __ldcg(p.seg_off + lane);
    const int cnt = __ldcg(p.counts + lane);
    // The last tail_experts active experts run tail_splits K slices: the
    // final wave of units is then shorter, so fewer SMs idle at the end.
    int my_splits = splits;
    if (p.tail_splits > splits) {
      const uint32_t active = __ballot_sync(0xffffffffu, cnt > 0);
      const int later = __popc(active & ~((2u << lane) - 1u));   // active experts after this one
      if (cnt > 0 && later < p.tail_experts) my_splits = p.tail_splits;
    }
    const int units = ((cnt + BN - 1) / BN) * Tr::kRowBlocks * my_splits;
    int incl = units;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += o;
    }
    s_unit_pre[lane + 1] = incl;
    s_seg[lane] = lo;
    s_cnt[lane] = cnt;
    s_splits[lane] = my_splits;
    if (lane == 0) s_unit_pre[0] = 0;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *s_tmem;
  const int total_units = s_unit_pre[kExpertsLocal];

  if (warp == 0) {
    // ======================================================== TMA producer
    // The first unit and the weight tiles of its first stages are taken
    // before waiting for the previous kernel (the stages are fresh, so no
    // empty-slot wait; the unit counter was cleared by the permutation).
    int u = -1;
    if (lane == 0) u = atomicAdd(p.sched, 1);
    u = __shfl_sync(0xffffffffu, u, 0);
    if (u >= total_units) u = -1;
    int pre_issued = 0;
    if (u >= 0 && early_tables) {
      Tile t;
      decode_tile<BN, Tr::kKBlocks>(u, s_unit_pre, s_seg, s_cnt, s_splits, t);
      const int nkb = t.kb1 - t.kb0;
      const int rot = (t.blk * 5 + t.e * 3) % nkb;
      pre_issued = nkb < kStages ? nkb : kStages;
      if (lane == 0) {
        int arow0, arow1;
        if constexpr (Tr::kIsG1) {
          arow0 = t.e * kGemm1Out + t.blk * kBlk;
          arow1 = arow0 + kInter;
        } else {
          arow0 = t.e * kHidden + t.blk * Tr::kNumA * kBlk;
          arow1 = arow0 + kBlk;
        }
        for (int i = 0; i < pre_issued; ++i) {
          const int kb = t.kb0 + (i + rot) % nkb;
          uint8_t* st = smem + Tr::kOffStages + i * Tr::kStageBytes;
          const uint32_t fb = smem_u32(&full_bar[i]);
          mbar_arrive_expect_tx(fb, Tr::kStageBytes);
          tma_load_2d(smem_u32(st), &tm_w, fb, kb * kBlk, arow0);
          if constexpr (Tr::kNumA == 2) tma_load_2d(smem_u32(st + Tr::kATileBytes), &tm_w, fb, kb * kBlk, arow1);
        }
      }
    }
    pdl_wait();
    pdl_launch_next();
    int stage = 0;
    uint32_t ph = 0;
    int slot = 0;
    uint32_t sph = 0;
    int uslot = 0;
    uint32_t uph = 0;
    int iter = 0;
    bool ok = true;
    bool c_ready = p.grid_sync == nullptr;   // decode GEMM2: C is produced in this kernel
    while (ok) {
      // publish the unit (or the end marker -1) to the other roles
      if (!mbar_wait(smem_u32(&uempty_bar[uslot]), uph ^ 1, s_abort, p.status, kStatusTimeoutProducer)) break;
      if (lane == 0) {
        s_units[uslot] = u;
        mbar_arrive(smem_u32(&ufull_bar[uslot]));
      }
      __syncwarp();
      if (++uslot == Tr::kUnitSlots) { uslot = 0; uph ^= 1; }
      if (u < 0) break;
      Tile t;
      decode_tile<BN, Tr::kKBlocks>(u, s_unit_pre, s_seg, s_cnt, s_splits, t);
      int arow0, arow1 = 0, wrow0, wrow1 = 0;
      if constexpr (Tr::kIsG1) {
        arow0 = t.e * kGemm1Out + t.blk * kBlk;
        arow1 = arow0 + kInter;
        wrow0 = (t.e * kGemm1OutBlocks + t.blk) * kHiddenBlocks;
        wrow1 = (t.e * kGemm1OutBlocks + kInterBlocks + t.blk) * kHiddenBlocks;
      } else {
        arow0 = t.e * kHidden + t.blk * Tr::kNumA * kBlk;
        arow1 = arow0 + kBlk;
        wrow0 = (t.e * kHiddenBlocks + t.blk * Tr::kNumA) * kInterBlocks;
        wrow1 = wrow0 + kInterBlocks;
      }
      // K blocks are visited in a tile-dependent rotation: weight rows are
      // 2 KB (W2) or 7 KB (W13) apart, and CTAs that all start at K block 0
      // would aim their 128-byte row slices at the same address residues.
      // Each weight tile here belongs to one CTA, so no L2 sharing is lost.
      const int nkb = t.kb1 - t.kb0;
      const int rot = (t.blk * 5 + t.e * 3) % nkb;
      for (int i = 0; i < nkb; ++i) {
        const int kb = t.kb0 + (i + rot) % nkb;
        const bool weights_issued = iter < pre_issued;
        ++iter;
        if ((!weights_issued &&
             !mbar_wait(smem_u32(&empty_bar[stage]), ph ^ 1, s_abort, p.status, kStatusTimeoutProducer)) ||
            !mbar_wait(smem_u32(&sempty_bar[slot]), sph ^ 1, s_abort, p.status, kStatusTimeoutProducer)) {
          ok = false;
          break;
        }
        if (!c_ready) {
          // The token tiles (C) and their scales are written by every CTA of
          // this grid: wait until all have counted themselves on grid_sync.
          if (lane == 0) {
            const uint64_t t0 = globaltimer_ns();
            uint32_t spins = 0;
            while (ld_acquire_gpu(p.grid_sync) < static_cast<int>(gridDim.x)) {
              if ((++spins & 63u) == 0u) {
                if (*s_abort) break;
                if (globaltimer_ns() - t0 > kWaitBudgetNs) {
                  atomicOr(p.status, kStatusTimeoutGridSync);
                  *s_abort = 1;
                  break;
                }
              }
            }
            fence_proxy_async_global();
          }
          __syncwarp();
          if (*s_abort) {
            ok = false;
            break;
          }
          c_ready = true;
        }
        if (lane == 0) {
          uint8_t* st = smem + Tr::kOffStages + stage * Tr::kStageBytes;
          const uint32_t fb = smem_u32(&full_bar[stage]);
          const int kx = kb * kBlk;
          if (!weights_issued) {
            mbar_arrive_expect_tx(fb, Tr::kStageBytes);
            tma_load_2d(smem_u32(st), &tm_w, fb, kx, arow0);
            if constexpr (Tr::kNumA == 2) tma_load_2d(smem_u32(st + Tr::kATileBytes), &tm_w, fb, kx, arow1);
          }
          uint8_t* bt = st + Tr::kNumA * Tr::kATileBytes;
          tma_load_2d(smem_u32(bt), &tm_b0, fb, kx, t.row0);
          if constexpr (Tr::kNumB == 2) tma_load_2d(smem_u32(bt + Tr::kBTileBytes), &tm_b1, fb, kx, t.row0);
          // Scales of this K block: the BN activation scales are contiguous in
          // the permuted row order (segment starts are 16-row aligned), the
          // weight scale(s) are single floats.
          float* sp = ring + slot * Tr::kSlotFloats;
          const uint32_t sb = smem_u32(&sraw_bar[slot]);
          mbar_arrive_expect_tx(sb, BN * 4);
          bulk_load(smem_u32(sp), p.act_scale + static_cast<int64_t>(kb) * p.cap + t.row0, BN * 4, sb);
          cp_async_4(smem_u32(sp + BN), p.w_scale + wrow0 + kb);
          if constexpr (Tr::kNumA == 2) cp_async_4(smem_u32(sp + BN + 1), p.w_scale + wrow1 + kb);
          cp_async_arrive_noinc(sb);
        }
        __syncwarp();
        if (++stage == kStages) { stage = 0; ph ^= 1; }
        if (++slot == Tr::kScaleSlots) { slot = 0; sph ^= 1; }
      }
      if (lane == 0) u = atomicAdd(p.sched, 1);
      u = __shfl_sync(0xffffffffu, u, 0);
      if (u >= total_units) u = -1;
    }
  } else if (warp == 1) {
    // ========================================================== MMA issuer
    pdl_wait();
    pdl_launch_next();
    int stage = 0;
    uint32_t ph = 0;
    int abuf = 0;
    uint32_t aph = 0;
    bool ok = true;
    int uslot = 0;
    uint32_t uph = 0;
    while (ok) {
      if (!mbar_wait(smem_u32(&ufull_bar[uslot]), uph, s_abort, p.status, kStatusTimeoutUnit)) break;
      const int u = s_units[uslot];
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&uempty_bar[uslot]));
      if (++uslot == Tr::kUnitSlots) { uslot = 0; uph ^= 1; }
      if (u < 0) break;
      Tile t;
      decode_tile<BN, Tr::kKBlocks>(u, s_unit_pre, s_seg, s_cnt, s_splits, t);
      for (int kb = t.kb0; kb < t.kb1; ++kb) {
        if (!mbar_wait(smem_u32(&full_bar[stage]), ph, s_abort, p.status, kStatusTimeoutMma) ||
            !mbar_wait(smem_u32(&acce_bar[abuf]), aph ^ 1, s_abort, p.status, kStatusTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t st = smem_u32(smem + Tr::kOffStages + stage * Tr::kStageBytes);
          const uint32_t d = tmem_base + abuf * Tr::kAccCols;
          // accumulator a (columns a*kMmaN..) = A_a . [token tiles], fresh at
          // k = 0 of every K block (GEMM2: columns BN.. hold the lo part)
#pragma unroll
          for (int k = 0; k < 4; ++k) {
#pragma unroll
            for (int a = 0; a < Tr::kNumA; ++a) {
              const uint64_t adesc = sw128_kmajor_desc(st + a * Tr::kATileBytes + 32 * k);
              const uint64_t bdesc = sw128_kmajor_desc(st + Tr::kNumA * Tr::kATileBytes + 32 * k);
              umma_f8(d + a * Tr::kMmaN, adesc, bdesc, Tr::kIdesc, k > 0 ? 1u : 0u);
            }
          }
          umma_commit(smem_u32(&empty_bar[stage]));
          umma_commit(smem_u32(&accf_bar[abuf]));
        }
        __syncwarp();
        if (++stage == kStages) { stage = 0; ph ^= 1; }
        if (++abuf == 2) { abuf = 0; aph ^= 1; }
      }
    }
  } else if (warp == 2) {
    // ======================================================= scale combiner
    pdl_wait();
    pdl_launch_next();
    int slot = 0;
    uint32_t sph = 0;
    bool ok = true;
    int uslot = 0;
    uint32_t uph = 0;
    while (ok) {
      if (!mbar_wait(smem_u32(&ufull_bar[uslot]), uph, s_abort, p.status, kStatusTimeoutUnit)) break;
      const int u = s_units[uslot];
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&uempty_bar[uslot]));
      if (++uslot == Tr::kUnitSlots) { uslot = 0; uph ^= 1; }
      if (u < 0) break;
      Tile t;
      decode_tile<BN, Tr::kKBlocks>(u, s_unit_pre, s_seg, s_cnt, s_splits, t);
      for (int kb = t.kb0; kb < t.kb1; ++kb) {
        if (!mbar_wait(smem_u32(&sraw_bar[slot]), sph, s_abort, p.status, kStatusTimeoutScale)) {
          ok = false;
          break;
        }
        float* sp = ring + slot * Tr::kSlotFloats;
        const float w0 = sp[BN];
        const float w1 = Tr::kNumA == 2 ? sp[BN + 1] : 0.f;
#pragma unroll
        for (int i = 0; i < Tr::kColsPerLane; ++i) {
          const int c = lane + 32 * i;
          if (c < BN) {
            const float a = sp[c];
            sp[BN + 4 + c] = a * w0;
            if constexpr (Tr::kNumA == 2) sp[BN + 4 + BN + c] = a * w1;
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&sfull_bar[slot]));
        if (++slot == Tr::kScaleSlots) { slot = 0; sph ^= 1; }
      }
    }
  } else if (warp < Tr::kRoleWarps) {
    // spare warp of the role warpgroup
    pdl_wait();
    pdl_launch_next();
  } else {
    // ============================================================ epilogue
    pdl_wait();
    pdl_launch_next();
    constexpr int CPT = Tr::kCPT;
    const int ew = warp - Tr::kRoleWarps;
    const int q = warp & 3;                   // TMEM lane quarter of this warp
    const int col0 = (ew >> 2) * CPT;         // first token column of this warp
    const int row_in_tile = q * 32 + lane;    // weight row inside the 128-row block
    const int et = ew * 32 + lane;            // 0.. inside the epilogue group
    const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
    constexpr uint32_t kEpiThreads = 32 * Tr::kEpiWarps;
    if constexpr (kKind == kGemm2Wide) {
      if (p.grid_sync != nullptr) {
        // Decode plan: convert the K-split GEMM1 sums of every valid
        // (token, expert) row into C, one (row, 128-block) per warp task over
        // the whole grid, then count this CTA on grid_sync. The producer
        // streams its first weight tiles meanwhile. Valid pair v is row
        // seg[e] + v - cpre[e] of expert e (cpre = exclusive prefix of counts).
        const int cnt = s_cnt[lane];
        int incl = cnt;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
          const int o = __shfl_up_sync(0xffffffffu, incl, off);
          if (lane >= off) incl += o;
        }
        const int pairs = __shfl_sync(0xffffffffu, incl, 31);
        const int nwarps = static_cast<int>(gridDim.x) * Tr::kEpiWarps;
        for (int task = static_cast<int>(blockIdx.x) * Tr::kEpiWarps + ew; task < pairs * kInterBlocks;
             task += nwarps) {
          const int v = task / kInterBlocks;
          const int e = __popc(__ballot_sync(0xffffffffu, incl <= v));
          const int row = s_seg[e] + v - (__shfl_sync(0xffffffffu, incl, e) - __shfl_sync(0xffffffffu, cnt, e));
          swiglu_quant_row_block(p, row, task % kInterBlocks, lane);
        }
        fence_proxy_async_global();   // C is read back through TMA
        __threadfence();
        named_bar_sync(1, kEpiThreads);
        if (et == 0) red_release_gpu_add(p.grid_sync, 1);
      }
    }
    if constexpr (kKind == kGemm1Split) {
      // The decode plan clears GEMM2's combine buffer here, spread over all
      // CTAs while they wait for their first accumulator.
      const int64_t n4 = static_cast<int64_t>(p.num_tokens) * (kHidden / 4);
      float4* y4 = reinterpret_cast<float4*>(p.y_acc);
      for (int64_t i = static_cast<int64_t>(blockIdx.x) * kEpiThreads + et; i < n4;
           i += static_cast<int64_t>(gridDim.x) * kEpiThreads)
        y4[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    int slot = 0;
    uint32_t sph = 0;
    int abuf = 0;
    uint32_t aph = 0;
    bool ok = true;
    float acc0[CPT];
    float acc1[CPT];  // second accumulator (gate / second W2 block); unused when kNumA == 1
    int uslot = 0;
    uint32_t uph = 0;
    while (ok) {
      if (!mbar_wait(smem_u32(&ufull_bar[uslot]), uph, s_abort, p.status, kStatusTimeoutUnit)) break;
      const int u = s_units[uslot];
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&uempty_bar[uslot]));
      if (++uslot == Tr::kUnitSlots) { uslot = 0; uph ^= 1; }
      if (u < 0) break;
      Tile t;
      decode_tile<BN, Tr::kKBlocks>(u, s_unit_pre, s_seg, s_cnt, s_splits, t);
      // per-column data for the final epilogue, loaded early by every
      // epilogue warp itself (lane l: columns l and l + 32), so the warps
      // share nothing through shared memory and need no barrier
      int my_tok[Tr::kColsPerLane];
      float my_w[Tr::kColsPerLane];
#pragma unroll
      for (int i = 0; i < Tr::kColsPerLane; ++i) {
        my_tok[i] = 0;
        my_w[i] = 0.f;
        if constexpr (!Tr::kIsG1) {
          const int c = lane + 32 * i;
          if (c < BN && c < t.nvalid) {
            my_tok[i] = p.perm_row[t.row0 + c];
            my_w[i] = p.perm_w[t.row0 + c];
          }
        }
      }
#pragma unroll
      for (int c = 0; c < CPT; ++c) acc0[c] = 0.f;
      if constexpr (Tr::kNumA == 2) {
#pragma unroll
        for (int c = 0; c < CPT; ++c) acc1[c] = 0.f;
      }
      for (int kb = t.kb0; kb < t.kb1; ++kb) {
        if (!mbar_wait(smem_u32(&sfull_bar[slot]), sph, s_abort, p.status, kStatusTimeoutEpilogue) ||
            !mbar_wait(smem_u32(&accf_bar[abuf]), aph, s_abort, p.status, kStatusTimeoutEpilogue)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float* comb0 = ring + slot * Tr::kSlotFloats + BN + 4 + col0;
        const uint32_t taddr = lane_base + abuf * Tr::kAccCols + col0;
        // One phase per accumulator (up, gate / the two W2 blocks): every TMEM
        // load of the phase is issued before a single wait, then the
        // promotion FMAs run (GEMM2: of hi + lo, in chunks of 32 columns).
        constexpr int kChunk = Tr::kMergeB ? (CPT < 32 ? CPT : 32) : CPT;
#pragma unroll
        for (int ph_i = 0; ph_i < Tr::kNumA; ++ph_i) {
          float* acc = (ph_i == 0) ? acc0 : acc1;
          const float4* sc4 = reinterpret_cast<const float4*>(comb0 + ph_i * BN);
#pragma unroll
          for (int c0 = 0; c0 < CPT; c0 += kChunk) {
            uint32_t v[kChunk];
            uint32_t vlo[Tr::kMergeB ? kChunk : 1];
            const uint32_t ta = taddr + ph_i * Tr::kMmaN + c0;
            if constexpr (kChunk % 32 == 0) {
#pragma unroll
              for (int ch = 0; ch < kChunk / 32; ++ch) {
                tmem_ld32(ta + ch * 32, *reinterpret_cast<uint32_t(*)[32]>(&v[ch * 32]));
                if constexpr (Tr::kMergeB)
                  tmem_ld32(ta + BN + ch * 32, *reinterpret_cast<uint32_t(*)[32]>(&vlo[ch * 32]));
              }
            } else {
#pragma unroll
              for (int ch = 0; ch < kChunk / 16; ++ch) {
                tmem_ld16(ta + ch * 16, *reinterpret_cast<uint32_t(*)[16]>(&v[ch * 16]));
                if constexpr (Tr::kMergeB)
                  tmem_ld16(ta + BN + ch * 16, *reinterpret_cast<uint32_t(*)[16]>(&vlo[ch * 16]));
              }
            }
            tmem_wait_ld();
#pragma unroll
            for (int c4 = 0; c4 < kChunk / 4; ++c4) {
              const float4 sc = sc4[c0 / 4 + c4];
              const float scv[4] = {sc.x, sc.y, sc.z, sc.w};
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const int c = 4 * c4 + j;
                float x = __uint_as_float(v[c]);
                if constexpr (Tr::kMergeB) x += __uint_as_float(vlo[c]);
                acc[c0 + c] = fmaf(x, scv[j], acc[c0 + c]);
              }
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(smem_u32(&acce_bar[abuf]));
          mbar_arrive(smem_u32(&sempty_bar[slot]));
        }
        if (++slot == Tr::kScaleSlots) { slot = 0; sph ^= 1; }
        if (++abuf == 2) { abuf = 0; aph ^= 1; }
      }
      if (!ok) break;

      // ------------------------------------------------- final epilogue
      if constexpr (kKind == kGemm1Fused) {
        swiglu_quant_store<BN, CPT>(acc0, acc1, t, q, col0, lane, et, row_in_tile, s_red, s_inv, p, kEpiThreads);
      } else if constexpr (kKind == kGemm1Split) {
        // Add this K slice into g1_acc (rows cleared by the decode front end);
        // swiglu_quant_kernel converts the sums once every slice is in.
        const int col = t.blk * kBlk + row_in_tile;
#pragma unroll
        for (int c = 0; c < CPT; ++c) {
          if (col0 + c < t.nvalid) {
            float* dst = p.g1_acc + static_cast<int64_t>(t.row0 + col0 + c) * kGemm1Out + col;
            red_add_f32(dst, acc0[c]);
            red_add_f32(dst + kInter, acc1[c]);
          }
        }
      } else {
        const int col = t.blk * Tr::kNumA * kBlk + row_in_tile;
#pragma unroll
        for (int c = 0; c < CPT; ++c) {
          // column col0 + c's token row and weight, from the lane that loaded them
          const int cc = col0 + c;
          const int reg = Tr::kColsPerLane > 1 ? cc / 32 : 0;
          const int tok = __shfl_sync(0xffffffffu, reg == 0 ? my_tok[0] : my_tok[Tr::kColsPerLane - 1], cc & 31);
          const float w = __shfl_sync(0xffffffffu, reg == 0 ? my_w[0] : my_w[Tr::kColsPerLane - 1], cc & 31);
          if (cc < t.nvalid) {
            float* dst = p.y_acc + static_cast<int64_t>(tok) * kHidden + col;
            red_add_f32(dst, acc0[c] * w);
            if constexpr (Tr::kNumA == 2) red_add_f32(dst + kBlk, acc1[c] * w);
          }
        }
      }
    }
  }

  // --------------------------------------------------------------- teardown
  if (*s_abort) {
    // Let copies that may still be in flight land before the CTA retires.
    const uint64_t t0 = globaltimer_ns();
    while (globaltimer_ns() - t0 < 2000000ull) {
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Tr::kTmemCols);
  }
}

// ---------------------------------------------------------------- launchers
template <int kKind, int BN, int kStages, int kEpiWarps>
static cudaError_t launch_one(const CUtensorMap& w, const CUtensorMap& b0, const CUtensorMap& b1,
                              const GemmParams& p, int grid, bool early_tables, cudaStream_t stream) {
  using Tr = GemmTraits<kKind, BN, kStages, kEpiWarps>;
  auto kern = moe_gemm_kernel<kKind, BN, kStages, kEpiWarps>;
  static int checked_device = -1;
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (checked_device != dev) {
    err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Tr::kSmemBytes);
    if (err != cudaSuccess) return err;
    checked_device = dev;
  }
  return launch_kernel(kern, grid, Tr::kThreads, Tr::kSmemBytes, stream, true, w, b0, b1, p,
                       early_tables ? 1 : 0);
}

// Decode (T <= 64): kGemm1Split / kGemm2Wide with 16-token tiles; mid-size
// batches (64 < T < 512): kGemm1Fused / kGemm2 with 64-token tiles; larger
// batches use the token-major kernels (gemm_tm_sm100.cu).
#define MOE_GEMM_CONFIGS(X)            \
  X(kGemm1Fused, 64, 5, 4)             \
  X(kGemm1Split, 16, 6, 4)             \
  X(kGemm2Wide, 16, 6, 4)              \
  X(kGemm2, 64, 6, 4)

cudaError_t launch_moe_gemm(int kind, int bn, const CUtensorMap& w, const CUtensorMap& b0,
                            const CUtensorMap& b1, const GemmParams& p, int grid,
                            bool early_tables, cudaStream_t stream) {
#define MOE_GEMM_DISPATCH(K, BN_, S, E) \
  if (kind == K && bn == BN_) return launch_one<K, BN_, S, E>(w, b0, b1, p, grid, early_tables, stream);
  MOE_GEMM_CONFIGS(MOE_GEMM_DISPATCH)
#undef MOE_GEMM_DISPATCH
  return cudaErrorInvalidValue;
}

bool gemm_config_supported(int kind, int bn) {
#define MOE_GEMM_SUPPORTED(K, BN_, S, E) \
  if (kind == K && bn == BN_) return true;
  MOE_GEMM_CONFIGS(MOE_GEMM_SUPPORTED)
#undef MOE_GEMM_SUPPORTED
  return false;
}

}  // namespace moe
