// Fixed shapes of the operator
// moe_fp8_block_scale_ds_routing_topk8_ng8_kg4_e32_h7168_i2048.
// They restate the reference's constants (solution/cuda/kernel.h:8-23).
#pragma once

namespace moe {

constexpr int kHidden = 7168;           // H
constexpr int kInter = 2048;            // I
constexpr int kGemm1Out = 4096;         // 2 * I (rows [0, I) = up, [I, 2I) = gate)
constexpr int kExpertsGlobal = 256;     // E_global
constexpr int kExpertsLocal = 32;       // E_local
constexpr int kBlk = 128;               // block-scale granularity
constexpr int kHiddenBlocks = 56;       // H / 128
constexpr int kInterBlocks = 16;        // I / 128
constexpr int kGemm1OutBlocks = 32;     // 2I / 128
constexpr int kTopK = 8;
constexpr int kGroups = 8;
constexpr int kGroupSize = 32;
constexpr int kTopKGroups = 4;
// Expert segments of the permuted row space start on multiples of this many
// rows, so every GEMM tile starts 16-byte aligned in the fp32 scale arrays.
constexpr int kSegAlign = 16;

}  // namespace moe
