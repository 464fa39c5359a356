// Token-major grouped FP8 GEMMs for prefill-size batches (sm_100a).
//
// The MMA's M side is 128 permuted token rows (one TMEM lane each) and its N
// side is 256 weight rows of one expert, K-major e4m3 operands with the
// 128-byte swizzle, one tcgen05.mma M=128 N=256 K=32 per 32 K-elements.
// After each 128-wide K block the epilogue folds the fresh accumulator into
// fp32 registers with that block's scale. In this orientation the scale of a
// TMEM lane's whole 128-column weight block is a single number, token scale
// times weight scale, so the promotion is one FFMA per element with a
// register operand -- no per-column scale loads. (The swap-AB kernels in
// gemm_sm100.cu keep weights on M; they serve decode-size batches, where a
// token tile of 16 keeps the MMA small.)
//
// GEMM1 tile: 128 tokens x (128 up rows + 128 gate rows of intermediate
// block `blk`); epilogue C = silu(gate) * up (solution/cuda/kernel.h:207),
// written as the hi/lo e4m3 pair with one scale per (row, 128-block).
// GEMM2 tile: 128 tokens x 256 W2 rows (two 128-row blocks); the hi and lo
// parts of C accumulate into one accumulator; epilogue red.adds w * O into
// the fp32 combine rows with 16-byte vector reductions.
//
// Roles: warp 0 TMA producer, warp 1 TMEM owner + MMA issuer, warp 2 scale
// combiner, warp 3 spare, warps 4-11 epilogue (TMEM lane quarter w % 4,
// column half (w - 4) / 4). The scale combiner multiplies each K block's
// token scales by its weight-block scales into a per-accumulator-buffer
// array and arrives on the same barrier as the MMA's commit, so an epilogue
// warp waits once per K block and reads its two scales with plain loads.
// The role warpgroup drops to 56 registers and the epilogue warpgroups rise
// to 224.
#include <cuda.h>
#include <cuda_fp8.h>
#include <cstdint>

#include "gemm_sm100.h"
#include "moe_kernels.cuh"
#include "moe_ptx.cuh"
#include "moe_shapes.cuh"
#include "swiglu.cuh"

namespace moe {

template <bool kG1, int kStages>
struct TmTraits {
  static constexpr int BM = 128;                   // token rows per tile
  static constexpr int BW = 256;                   // weight rows per tile
  static constexpr int kATileBytes = BM * 128;     // one token operand per K block
  static constexpr int kNumA = kG1 ? 1 : 2;        // activations / C hi + lo
  static constexpr int kBTileBytes = BW * 128;
  static constexpr int kStageBytes = kNumA * kATileBytes + kBTileBytes;
  static constexpr int kKBlocks = kG1 ? kHiddenBlocks : kInterBlocks;
  static constexpr int kRowBlocks = kG1 ? kInterBlocks : kHiddenBlocks / 2;
  static constexpr int kAccCols = 256;
  static constexpr int kTmemCols = 512;            // two accumulator buffers
  static constexpr int kScaleSlots = 8;
  static constexpr int kSlotFloats = BM + 4;       // token scales | weight scales x2 | pad
  static constexpr int kEpiWarps = 8;
  static constexpr int kThreads = (4 + kEpiWarps) * 32;
  static constexpr uint32_t kIdesc = idesc_e4m3_f32<128, 256>();
  static constexpr int kLaunchRegs = 168;
  static constexpr int kRoleRegs = 56;
  static constexpr int kEpiRegs = 224;
  static_assert(kRoleRegs * 128 + kEpiRegs * 32 * kEpiWarps <= kLaunchRegs * kThreads,
                "register split exceeds the block's launch registers");

  static constexpr int kOffRing = kStages * kStageBytes;
  static constexpr int kOffBars = kOffRing + kScaleSlots * kSlotFloats * 4;
  // Work units are handed out dynamically through a small ring (s_units +
  // full/empty barriers), like the swap-AB kernels.
  static constexpr int kUnitSlots = 4;
  static constexpr int kUnitConsumers = 2 + kEpiWarps;   // MMA warp + scale warp + epilogue warps
  static constexpr int kNumBars = 2 * kStages + 4 + 2 * kScaleSlots + 2 * kUnitSlots;
  static constexpr int kOffMisc = kOffBars + kNumBars * 8;
  static constexpr int kOffUnitPre = kOffMisc + 16;
  static constexpr int kOffSeg = kOffUnitPre + 34 * 4;
  static constexpr int kOffCnt = kOffSeg + 34 * 4;
  static constexpr int kOffUnits = kOffCnt + 32 * 4;
  static constexpr int kOffRed = kOffUnits + kUnitSlots * 4;   // [2][BM] row maxima (GEMM1)
  // GEMM2 combine staging: per epilogue warp 32 rows x 16 floats, rows
  // kStagePitch bytes apart (64 B of data + 16 B pad: conflict-free float4
  // stores from lanes that each own a row).
  static constexpr int kStagePitch = 80;
  static constexpr int kOffStage = kOffRed + 2 * BM * 4;
  static constexpr int kStageWarpBytes = 32 * kStagePitch;
  // Combined scales of the two accumulator buffers: [buffer][column half][row].
  static constexpr int kOffComb = kOffStage + (kG1 ? 0 : kEpiWarps * kStageWarpBytes);
  static constexpr int kSmemBytes = kOffComb + 2 * 2 * BM * 4 + 1024;
  static_assert(kOffComb % 16 == 0 && (kSlotFloats * 4) % 16 == 0, "float4 scale access");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory");
};

namespace {

__device__ __forceinline__ void red_add_v4(float* addr, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b), "f"(c),
               "f"(d)
               : "memory");
}

// Two fp32 lanes in one 64-bit register pair, for the packed FMA below.
__device__ __forceinline__ uint64_t pack_f32x2(uint32_t lo_bits, uint32_t hi_bits) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo_bits), "r"(hi_bits));
  return r;
}

__device__ __forceinline__ void unpack_f32x2(uint64_t p, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(p));
}

// d = a * b + c on two fp32 lanes at once (two IEEE round-to-nearest FMAs in
// one instruction): halves the promotion's FMA issue slots.
__device__ __forceinline__ uint64_t ffma_f32x2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

// silu(g) * u with the fast exponential and division (relative error ~1e-7,
// far below the 8-bit precision C keeps as the hi/lo e4m3 pair).
__device__ __forceinline__ float silu_mul_fast(float g, float u) {
  return __fdividef(g, 1.0f + __expf(-g)) * u;
}

__device__ __forceinline__ uint32_t pack_e4m3x4(float a, float b, float c, float d) {
  const uint32_t lo = __nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
  const uint32_t hi = __nv_cvt_float2_to_fp8x2(make_float2(c, d), __NV_SATFINITE, __NV_E4M3);
  return lo | (hi << 16);
}

__device__ __forceinline__ float e4m3_round(float x) {
  const __nv_fp8_e4m3 q(x);
  return static_cast<float>(q);
}

// Units of work: per expert ceil(count / 128) token tiles x kRowBlocks weight
// blocks, token tiles fastest so CTAs running at the same time share the
// weight block through L2. Units are handed out in increasing order by an
// atomic counter, so faster CTAs take more of them.
struct TmTile {
  int e, blk, row0, nvalid, kb0, kb1;
};

// With `splits` > 1 (GEMM2 of batches with fewer units than CTAs) each
// (expert, block, token tile) is split into K ranges of kblocks / splits
// blocks, adjacent in the unit order; their partial sums meet in the
// combine rows' fp32 reductions.
__device__ __forceinline__ void tm_decode(int u, const int* s_unit_pre, const int* s_seg, const int* s_cnt,
                                          int splits, int kblocks, TmTile& t) {
  int e = 0;
#pragma unroll 1
  while (s_unit_pre[e + 1] <= u) ++e;
  const int cnt = s_cnt[e];
  const int nt = (cnt + 127) / 128;
  const int local = u - s_unit_pre[e];
  const int ks = local % splits;
  const int rest = local / splits;
  const int tt = rest % nt;
  t.e = e;
  t.blk = rest / nt;
  t.row0 = s_seg[e] + tt * 128;
  t.nvalid = min(128, cnt - tt * 128);
  const int per = kblocks / splits;
  t.kb0 = ks * per;
  t.kb1 = t.kb0 + per;
}

// GEMM2 units in groups of kG2BlockGroup W2 column blocks: (block group,
// expert, block in group, token tile), token tiles fastest (K splits
// fastest of all). Each unit red.adds into a 256-column block of its
// tokens' combine rows; ordering by column block keeps that block of every
// token's row in L2 while all experts add into it, where the expert-major
// order re-fetched the combine rows from DRAM for every expert (78% of the
// reduction sectors missed L2 in a T=4096 capture). The token tiles of one
// (expert, block) still run side by side and share the W2 tile through L2.
#ifndef MOE_B200_G2_BLOCK_GROUP
#define MOE_B200_G2_BLOCK_GROUP 4
#endif
constexpr int kG2BlockGroup = MOE_B200_G2_BLOCK_GROUP;
static_assert((kHiddenBlocks / 2) % kG2BlockGroup == 0, "block groups tile the 28 W2 column blocks");

__device__ __forceinline__ void tm_decode_g2(int u, const int* s_unit_pre, const int* s_seg, const int* s_cnt,
                                             int splits, int kblocks, TmTile& t) {
  constexpr int kRowBlocks = kHiddenBlocks / 2;
  const int per_tile = kRowBlocks * splits;            // units of one token tile in s_unit_pre
  const int total_tiles = s_unit_pre[kExpertsLocal] / per_tile;
  const int ks = u % splits;
  const int rest = u / splits;
  const int group_units = total_tiles * kG2BlockGroup;
  const int bg = rest / group_units;
  const int r = rest - bg * group_units;
  int e = 0;
#pragma unroll 1
  while (s_unit_pre[e + 1] / per_tile * kG2BlockGroup <= r) ++e;
  const int cnt = s_cnt[e];
  const int nt = (cnt + 127) / 128;
  const int local = r - s_unit_pre[e] / per_tile * kG2BlockGroup;
  const int bi = local / nt;
  const int tt = local - bi * nt;
  t.e = e;
  t.blk = bg * kG2BlockGroup + bi;
  t.row0 = s_seg[e] + tt * 128;
  t.nvalid = min(128, cnt - tt * 128);
  const int per = kblocks / splits;
  t.kb0 = ks * per;
  t.kb1 = t.kb0 + per;
}

template <bool kG1>
__device__ __forceinline__ void tm_unit(int u, const int* s_unit_pre, const int* s_seg, const int* s_cnt,
                                        int splits, int kblocks, TmTile& t) {
  if constexpr (kG1)
    tm_decode(u, s_unit_pre, s_seg, s_cnt, splits, kblocks, t);
  else
    tm_decode_g2(u, s_unit_pre, s_seg, s_cnt, splits, kblocks, t);
}

}  // namespace

template <bool kG1, int kStages>
__global__ void __launch_bounds__(TmTraits<kG1, kStages>::kThreads, 1)
    moe_gemm_tm_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_a0,
                       const __grid_constant__ CUtensorMap tm_a1, const GemmParams p) {
  using Tr = TmTraits<kG1, kStages>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  float* ring = reinterpret_cast<float*>(smem + Tr::kOffRing);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Tr::kOffBars);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + kStages;
  uint64_t* accf_bar = bars + 2 * kStages;
  uint64_t* acce_bar = accf_bar + 2;
  uint64_t* sfull_bar = acce_bar + 2;
  uint64_t* sempty_bar = sfull_bar + Tr::kScaleSlots;
  uint64_t* ufull_bar = sempty_bar + Tr::kScaleSlots;
  uint64_t* uempty_bar = ufull_bar + Tr::kUnitSlots;
  volatile int* s_units = reinterpret_cast<volatile int*>(smem + Tr::kOffUnits);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + Tr::kOffMisc);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + Tr::kOffMisc + 4);
  int* s_unit_pre = reinterpret_cast<int*>(smem + Tr::kOffUnitPre);
  int* s_seg = reinterpret_cast<int*>(smem + Tr::kOffSeg);
  int* s_cnt = reinterpret_cast<int*>(smem + Tr::kOffCnt);
  float* s_red = reinterpret_cast<float*>(smem + Tr::kOffRed);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // ---------------------------------------------------------------- setup
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_w);
    prefetch_tmap(&tm_a0);
    if (!kG1) prefetch_tmap(&tm_a1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&full_bar[s]), 1);
      mbar_init(smem_u32(&empty_bar[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&accf_bar[b]), 2);   // MMA commit + scale warp
      mbar_init(smem_u32(&acce_bar[b]), Tr::kEpiWarps);
    }
    for (int s = 0; s < Tr::kScaleSlots; ++s) {
      mbar_init(smem_u32(&sfull_bar[s]), 2);
      mbar_init(smem_u32(&sempty_bar[s]), 1);
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
  // Everything above overlaps the previous kernel's tail (programmatic
  // dependent launch); the routing and permutation results are read below.
  pdl_wait();
  pdl_launch_next();
  if (warp == 2) {
    const int lo = p.seg_off[lane];
    const int cnt = p.counts[lane];
    const int base = ((cnt + 127) / 128) * Tr::kRowBlocks;
    // GEMM2 with fewer (expert, block, token tile) units than CTAs: split K
    // 2 or 4 ways (the same choice in every CTA)
    int total = base;
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) total += __shfl_xor_sync(0xffffffffu, total, off);
    int splits = 1;
    if constexpr (kG1) {
      // K-split GEMM1 of few token tiles (partial sums into g1_acc)
      if (p.g1_acc != nullptr) splits = tm_gemm1_splits(total);
    } else {
      if (total > 0 && total < static_cast<int>(gridDim.x)) splits = 2 * total < static_cast<int>(gridDim.x) ? 4 : 2;
    }
    // GEMM2 after a K-split GEMM1: SwiGLU of the g1_acc sums runs here first
    const int g1_units = total / Tr::kRowBlocks * kInterBlocks;
    const int swiglu_phase = !kG1 && p.g1_acc != nullptr && p.grid_sync != nullptr && tm_gemm1_splits(g1_units) > 1;
    int incl = base * splits;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += o;
    }
    s_unit_pre[lane + 1] = incl;
    s_seg[lane] = lo;
    s_cnt[lane] = cnt;
    if (lane == 0) {
      s_unit_pre[0] = 0;
      s_unit_pre[kExpertsLocal + 1] = splits;
      s_seg[kExpertsLocal + 1] = swiglu_phase;   // spare slot of the segment table
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *s_tmem;
  const int total_units = s_unit_pre[kExpertsLocal];

  if (warp == 0) {
    // ======================================================== TMA producer
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(Tr::kRoleRegs));
    int stage = 0, slot = 0, uslot = 0;
    uint32_t ph = 0, sph = 0, uph = 0;
    bool ok = true;
    if (!kG1 && s_seg[kExpertsLocal + 1]) {
      // C (tiles and scales) comes from this grid's SwiGLU phase: wait until
      // every CTA has counted itself on grid_sync
      if (lane == 0) {
        const uint64_t t0 = globaltimer_ns();
        uint32_t spins = 0;
        while (ld_acquire_gpu(p.grid_sync) < static_cast<int>(gridDim.x)) {
          if ((++spins & 63u) == 0u && globaltimer_ns() - t0 > kWaitBudgetNs) {
            atomicOr(p.status, kStatusTimeoutGridSync);
            *s_abort = 1;
            break;
          }
        }
        fence_proxy_async_global();   // C is read through TMA
      }
      __syncwarp();
      if (*s_abort) ok = false;
    }
    while (ok) {
      int u = -1;
      if (lane == 0) u = atomicAdd(p.sched, 1);
      u = __shfl_sync(0xffffffffu, u, 0);
      if (u >= total_units) u = -1;
      // publish the unit (or the end marker -1) to the MMA and epilogue warps
      if (!mbar_wait(smem_u32(&uempty_bar[uslot]), uph ^ 1, s_abort, p.status, kStatusTimeoutProducer)) break;
      if (lane == 0) {
        s_units[uslot] = u;
        mbar_arrive(smem_u32(&ufull_bar[uslot]));
      }
      __syncwarp();
      if (++uslot == Tr::kUnitSlots) { uslot = 0; uph ^= 1; }
      if (u < 0) break;
      TmTile t;
      tm_unit<kG1>(u, s_unit_pre, s_seg, s_cnt, s_unit_pre[kExpertsLocal + 1], Tr::kKBlocks, t);
      int brow0, brow1, wrow0, wrow1;
      if constexpr (kG1) {
        brow0 = t.e * kGemm1Out + t.blk * kBlk;
        brow1 = brow0 + kInter;
        wrow0 = (t.e * kGemm1OutBlocks + t.blk) * kHiddenBlocks;
        wrow1 = (t.e * kGemm1OutBlocks + kInterBlocks + t.blk) * kHiddenBlocks;
      } else {
        brow0 = t.e * kHidden + t.blk * 2 * kBlk;
        brow1 = brow0 + kBlk;
        wrow0 = (t.e * kHiddenBlocks + 2 * t.blk) * kInterBlocks;
        wrow1 = wrow0 + kInterBlocks;
      }
      for (int kb = t.kb0; kb < t.kb1; ++kb) {
        if (!mbar_wait(smem_u32(&empty_bar[stage]), ph ^ 1, s_abort, p.status, kStatusTimeoutProducer) ||
            !mbar_wait(smem_u32(&sempty_bar[slot]), sph ^ 1, s_abort, p.status, kStatusTimeoutProducer)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          uint8_t* st = smem + stage * Tr::kStageBytes;
          const uint32_t fb = smem_u32(&full_bar[stage]);
          const int kx = kb * kBlk;
          mbar_arrive_expect_tx(fb, Tr::kStageBytes);
          tma_load_2d(smem_u32(st), &tm_a0, fb, kx, t.row0);
          if constexpr (!kG1) tma_load_2d(smem_u32(st + Tr::kATileBytes), &tm_a1, fb, kx, t.row0);
          uint8_t* bt = st + Tr::kNumA * Tr::kATileBytes;
          tma_load_2d(smem_u32(bt), &tm_w, fb, kx, brow0);
          tma_load_2d(smem_u32(bt + 128 * 128), &tm_w, fb, kx, brow1);
          float* sp = ring + slot * Tr::kSlotFloats;
          const uint32_t sb = smem_u32(&sfull_bar[slot]);
          mbar_arrive_expect_tx(sb, Tr::BM * 4);
          bulk_load(smem_u32(sp), p.act_scale + static_cast<int64_t>(kb) * p.cap + t.row0, Tr::BM * 4, sb);
          cp_async_4(smem_u32(sp + Tr::BM), p.w_scale + wrow0 + kb);
          cp_async_4(smem_u32(sp + Tr::BM + 1), p.w_scale + wrow1 + kb);
          cp_async_arrive_noinc(sb);
        }
        __syncwarp();
        if (++stage == kStages) { stage = 0; ph ^= 1; }
        if (++slot == Tr::kScaleSlots) { slot = 0; sph ^= 1; }
      }
    }
  } else if (warp == 1) {
    // ========================================================== MMA issuer
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(Tr::kRoleRegs));
    int stage = 0, abuf = 0, uslot = 0;
    uint32_t ph = 0, aph = 0, uph = 0;
    bool ok = true;
    while (ok) {
      if (!mbar_wait(smem_u32(&ufull_bar[uslot]), uph, s_abort, p.status, kStatusTimeoutUnit)) break;
      const int u = s_units[uslot];
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&uempty_bar[uslot]));
      if (++uslot == Tr::kUnitSlots) { uslot = 0; uph ^= 1; }
      if (u < 0) break;
      for (int kb = 0, nkb = Tr::kKBlocks / s_unit_pre[kExpertsLocal + 1]; kb < nkb; ++kb) {
        if (!mbar_wait(smem_u32(&full_bar[stage]), ph, s_abort, p.status, kStatusTimeoutMma) ||
            !mbar_wait(smem_u32(&acce_bar[abuf]), aph ^ 1, s_abort, p.status, kStatusTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t st = smem_u32(smem + stage * Tr::kStageBytes);
          const uint32_t bt = st + Tr::kNumA * Tr::kATileBytes;
          const uint32_t d = tmem_base + abuf * Tr::kAccCols;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t bdesc = sw128_kmajor_desc(bt + 32 * k);
            umma_f8(d, sw128_kmajor_desc(st + 32 * k), bdesc, Tr::kIdesc, k > 0 ? 1u : 0u);
            if constexpr (!kG1) umma_f8(d, sw128_kmajor_desc(st + Tr::kATileBytes + 32 * k), bdesc, Tr::kIdesc, 1u);
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
    // ====================================================== scale combiner
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(Tr::kRoleRegs));
    float* comb = reinterpret_cast<float*>(smem + Tr::kOffComb);
    int slot = 0, abuf = 0, uslot = 0;
    uint32_t sph = 0, aph = 0, uph = 0;
    bool ok = true;
    while (ok) {
      if (!mbar_wait(smem_u32(&ufull_bar[uslot]), uph, s_abort, p.status, kStatusTimeoutUnit)) break;
      const int u = s_units[uslot];
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&uempty_bar[uslot]));
      if (++uslot == Tr::kUnitSlots) { uslot = 0; uph ^= 1; }
      if (u < 0) break;
      for (int kb = 0, nkb = Tr::kKBlocks / s_unit_pre[kExpertsLocal + 1]; kb < nkb; ++kb) {
        // this K block's raw scales have landed, and the epilogue has read
        // the combined scales this buffer held two K blocks ago
        if (!mbar_wait(smem_u32(&sfull_bar[slot]), sph, s_abort, p.status, kStatusTimeoutEpilogue) ||
            !mbar_wait(smem_u32(&acce_bar[abuf]), aph ^ 1, s_abort, p.status, kStatusTimeoutEpilogue)) {
          ok = false;
          break;
        }
        const float* sp = ring + slot * Tr::kSlotFloats;
        const float4 ts = reinterpret_cast<const float4*>(sp)[lane];   // token rows 4*lane .. +3
        const float w0 = sp[Tr::BM], w1 = sp[Tr::BM + 1];
        float4* c0 = reinterpret_cast<float4*>(comb + (abuf * 2) * Tr::BM);
        float4* c1 = reinterpret_cast<float4*>(comb + (abuf * 2 + 1) * Tr::BM);
        c0[lane] = make_float4(ts.x * w0, ts.y * w0, ts.z * w0, ts.w * w0);
        c1[lane] = make_float4(ts.x * w1, ts.y * w1, ts.z * w1, ts.w * w1);
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(smem_u32(&sempty_bar[slot]));
          mbar_arrive(smem_u32(&accf_bar[abuf]));
        }
        if (++slot == Tr::kScaleSlots) { slot = 0; sph ^= 1; }
        if (++abuf == 2) { abuf = 0; aph ^= 1; }
      }
    }
  } else if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(Tr::kRoleRegs));
  } else {
    // ============================================================ epilogue
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(Tr::kEpiRegs));
    const int q = warp & 3;              // TMEM lane quarter: token rows q*32 .. q*32+31
    const int hf = (warp - 4) >> 2;      // column half
    const int r = q * 32 + lane;         // token row inside the tile
    const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
    const float* comb = reinterpret_cast<const float*>(smem + Tr::kOffComb);
    int abuf = 0, uslot = 0;
    uint32_t aph = 0, uph = 0;
    bool ok = true;
    if (!kG1 && s_seg[kExpertsLocal + 1]) {
      // After a K-split GEMM1: C = SwiGLU of the g1_acc sums for every valid
      // (token, expert) row and 128-block, one warp task each over the whole
      // grid; then this CTA counts itself on grid_sync (the producers wait
      // for all CTAs before their first C tile). Valid pair v is row
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
      for (int task = static_cast<int>(blockIdx.x) * Tr::kEpiWarps + (warp - 4); task < pairs * kInterBlocks;
           task += nwarps) {
        const int v = task / kInterBlocks;
        const int e = __popc(__ballot_sync(0xffffffffu, incl <= v));
        const int row = s_seg[e] + v - (__shfl_sync(0xffffffffu, incl, e) - __shfl_sync(0xffffffffu, cnt, e));
        swiglu_quant_row_block(p, row, task % kInterBlocks, lane);
      }
      fence_proxy_async_global();
      __threadfence();
      named_bar_sync(1, 32 * Tr::kEpiWarps);
      if (warp == 4 && lane == 0) red_release_gpu_add(p.grid_sync, 1);
    }
    // GEMM1: acc0 = up, acc1 = gate for intermediate columns hf*64 .. +64.
    // GEMM2: acc0 / acc1 = W2 rows (2*blk + hf)*128 + [0, 64) / [64, 128).
    // Kept as packed pairs (column 2i in the low half) for f32x2 FMAs.
    uint64_t acc0p[32], acc1p[32];
    while (ok) {
      if (!mbar_wait(smem_u32(&ufull_bar[uslot]), uph, s_abort, p.status, kStatusTimeoutUnit)) break;
      const int u = s_units[uslot];
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&uempty_bar[uslot]));
      if (++uslot == Tr::kUnitSlots) { uslot = 0; uph ^= 1; }
      if (u < 0) break;
      TmTile t;
      tm_unit<kG1>(u, s_unit_pre, s_seg, s_cnt, s_unit_pre[kExpertsLocal + 1], Tr::kKBlocks, t);
      const bool valid = r < t.nvalid;
      int my_tok = 0;
      float my_w = 0.f;
      if constexpr (!kG1) {
        if (valid) {
          my_tok = p.perm_row[t.row0 + r];
          my_w = p.perm_w[t.row0 + r];
        }
      }
#pragma unroll
      for (int i = 0; i < 32; ++i) { acc0p[i] = 0ull; acc1p[i] = 0ull; }
      for (int kb = t.kb0; kb < t.kb1; ++kb) {
        // the accumulator of this K block is complete and its combined
        // scales (token scale x weight-block scale) are in `comb`
        if (!mbar_wait(smem_u32(&accf_bar[abuf]), aph, s_abort, p.status, kStatusTimeoutEpilogue)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t tb = lane_base + abuf * Tr::kAccCols;
        const uint32_t col_a = kG1 ? hf * 64 : hf * 128;
        const uint32_t col_b = kG1 ? 128 + hf * 64 : hf * 128 + 64;
        uint32_t v[64];
        tmem_ld32(tb + col_a, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
        tmem_ld32(tb + col_a + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
        // GEMM1: up / gate block scales; GEMM2: this half's W2 block for both
        const float* cb = comb + abuf * 2 * Tr::BM;
        const float s0 = cb[(kG1 ? 0 : hf) * Tr::BM + r];
        const float s1 = kG1 ? cb[Tr::BM + r] : s0;
        const uint64_t s0p = pack_f32x2(__float_as_uint(s0), __float_as_uint(s0));
        const uint64_t s1p = pack_f32x2(__float_as_uint(s1), __float_as_uint(s1));
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) acc0p[i] = ffma_f32x2(pack_f32x2(v[2 * i], v[2 * i + 1]), s0p, acc0p[i]);
        tmem_ld32(tb + col_b, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
        tmem_ld32(tb + col_b + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&acce_bar[abuf]));
        if (++abuf == 2) { abuf = 0; aph ^= 1; }
#pragma unroll
        for (int i = 0; i < 32; ++i) acc1p[i] = ffma_f32x2(pack_f32x2(v[2 * i], v[2 * i + 1]), s1p, acc1p[i]);
      }
      if (!ok) break;
      float acc0[64], acc1[64];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        unpack_f32x2(acc0p[i], acc0[2 * i], acc0[2 * i + 1]);
        unpack_f32x2(acc1p[i], acc1[2 * i], acc1[2 * i + 1]);
      }

      // ------------------------------------------------- final epilogue
      const int64_t row = t.row0 + r;
      if (kG1 && s_unit_pre[kExpertsLocal + 1] > 1) {
        // K-split GEMM1: this K range's fp32 sums of up and gate into g1_acc
        // (GEMM2 applies SwiGLU once all ranges are in)
        if (valid) {
          float* gu = p.g1_acc + row * kGemm1Out + t.blk * kBlk + hf * 64;
          float* gg = gu + kInter;
#pragma unroll
          for (int c = 0; c < 64; c += 4) {
            red_add_v4(gu + c, acc0[c], acc0[c + 1], acc0[c + 2], acc0[c + 3]);
            red_add_v4(gg + c, acc1[c], acc1[c + 1], acc1[c + 2], acc1[c + 3]);
          }
        }
      } else if constexpr (kG1) {
        float m = 0.f;
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          acc0[c] = silu_mul_fast(acc1[c], acc0[c]);
          m = fmaxf(m, fabsf(acc0[c]));
        }
        named_bar_sync(1, 32 * Tr::kEpiWarps);
        s_red[hf * Tr::BM + r] = m;
        named_bar_sync(1, 32 * Tr::kEpiWarps);
        const float amax = fmaxf(s_red[r], s_red[Tr::BM + r]);
        const float inv = amax > 0.f ? 448.0f / amax : 0.f;
        if (valid) {
          if (hf == 0) p.c_scale[static_cast<int64_t>(t.blk) * p.cap + row] = amax * (1.0f / 448.0f);
          uint4* hi_dst = reinterpret_cast<uint4*>(p.c_hi + row * kInter + t.blk * kBlk + hf * 64);
          uint4* lo_dst = reinterpret_cast<uint4*>(p.c_lo + row * kInter + t.blk * kBlk + hf * 64);
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            uint32_t wh[4], wl[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              float x[4], res[4];
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                x[i] = acc0[16 * g + 4 * j + i] * inv;
                res[i] = x[i] - e4m3_round(x[i]);
              }
              wh[j] = pack_e4m3x4(x[0], x[1], x[2], x[3]);
              wl[j] = pack_e4m3x4(res[0], res[1], res[2], res[3]);
            }
            hi_dst[g] = make_uint4(wh[0], wh[1], wh[2], wh[3]);
            lo_dst[g] = make_uint4(wl[0], wl[1], wl[2], wl[3]);
          }
        }
      } else {
        // w * O into the combine rows. Lane l holds 128 consecutive columns
        // of token row r; red.adds from that layout would send 32 scattered
        // 16-byte requests per instruction. Instead each 16-column chunk goes
        // through this warp's staging rows and is read back transposed, so
        // one instruction adds 64 contiguous bytes to each of 8 rows.
        uint8_t* stage_w = smem + Tr::kOffStage + (warp - 4) * Tr::kStageWarpBytes;
        const int rr = lane >> 2;        // row (of 8) this lane reads back
        const int cq = lane & 3;         // its 16-byte column quad
        const float w = valid ? my_w : 0.f;
        int toks[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) toks[j] = __shfl_sync(0xffffffffu, valid ? my_tok : -1, 8 * j + rr);
        float* ybase = p.y_acc + (2 * t.blk + hf) * kBlk + 4 * cq;
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
          const float* a = ch < 4 ? &acc0[16 * ch] : &acc1[16 * (ch - 4)];
          float4* srow = reinterpret_cast<float4*>(stage_w + lane * Tr::kStagePitch);
#pragma unroll
          for (int j = 0; j < 4; ++j)
            srow[j] = make_float4(a[4 * j] * w, a[4 * j + 1] * w, a[4 * j + 2] * w, a[4 * j + 3] * w);
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int row8 = 8 * j + rr;
            const float4 v4 = *reinterpret_cast<const float4*>(stage_w + row8 * Tr::kStagePitch + 16 * cq);
            if (toks[j] >= 0)
              red_add_v4(ybase + static_cast<int64_t>(toks[j]) * kHidden + 16 * ch, v4.x, v4.y, v4.z, v4.w);
          }
          __syncwarp();
        }
      }
    }
  }

  // --------------------------------------------------------------- teardown
  if (*s_abort) {
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

template <bool kG1, int kStages>
static cudaError_t launch_tm(const CUtensorMap& w, const CUtensorMap& a0, const CUtensorMap& a1,
                             const GemmParams& p, int grid, cudaStream_t stream) {
  using Tr = TmTraits<kG1, kStages>;
  auto kern = moe_gemm_tm_kernel<kG1, kStages>;
  static int checked_device = -1;
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (checked_device != dev) {
    err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Tr::kSmemBytes);
    if (err != cudaSuccess) return err;
    // The warpgroup register split is only safe if the block launches with
    // exactly the registers it was sized for.
    cudaFuncAttributes attr;
    err = cudaFuncGetAttributes(&attr, kern);
    if (err != cudaSuccess) return err;
    if (attr.numRegs != Tr::kLaunchRegs) return cudaErrorInvalidConfiguration;
    checked_device = dev;
  }
  return launch_kernel(kern, grid, Tr::kThreads, Tr::kSmemBytes, stream, true, w, a0, a1, p);
}

cudaError_t launch_moe_gemm_tm(bool gemm1, const CUtensorMap& w, const CUtensorMap& a0, const CUtensorMap& a1,
                               const GemmParams& p, int grid, cudaStream_t stream) {
  return gemm1 ? launch_tm<true, 4>(w, a0, a1, p, grid, stream) : launch_tm<false, 3>(w, a0, a1, p, grid, stream);
}

}  // namespace moe
