// SwiGLU of GEMM1 sums and their hi/lo e4m3 quantisation, shared by the
// swap-AB and token-major GEMM kernels.
#pragma once

#include <cuda_fp8.h>
#include <cstdint>

#include "moe_kernels.cuh"
#include "moe_shapes.cuh"

namespace moe {

// silu(gate) * up (solution/cuda/kernel.h:207) with the accurate exponential.
__device__ __forceinline__ float silu_mul(float gate, float up) {
  return gate / (1.0f + expf(-gate)) * up;
}

// SwiGLU of one (row, 128-block) of K-split GEMM1 sums (g1_acc), by one
// warp: C = silu(gate) * up (solution/cuda/kernel.h:207) for intermediate
// columns ib*128 + 4l .. +3 in lane l, written as the e4m3 pair
// C = s * (hi + lo), s = amax / 448 over the block. Same arithmetic as
// swiglu_quant_store.
__device__ __forceinline__ void swiglu_quant_row_block(const GemmParams& p, int row, int ib, int lane) {
  const float* g = p.g1_acc + static_cast<int64_t>(row) * kGemm1Out + ib * kBlk + 4 * lane;
  const float4 up = __ldcg(reinterpret_cast<const float4*>(g));
  const float4 gate = __ldcg(reinterpret_cast<const float4*>(g + kInter));
  const float h[4] = {silu_mul(gate.x, up.x), silu_mul(gate.y, up.y), silu_mul(gate.z, up.z),
                      silu_mul(gate.w, up.w)};
  float amax = fmaxf(fmaxf(fabsf(h[0]), fabsf(h[1])), fmaxf(fabsf(h[2]), fabsf(h[3])));
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
  const float inv = amax > 0.f ? 448.0f / amax : 0.f;
  uint32_t phi = 0, plo = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float x = h[j] * inv;
    const __nv_fp8_e4m3 qh(x);
    const float r = x - static_cast<float>(qh);
    const __nv_fp8_e4m3 ql(r);
    phi |= static_cast<uint32_t>(qh.__x) << (8 * j);
    plo |= static_cast<uint32_t>(ql.__x) << (8 * j);
  }
  const int64_t off = static_cast<int64_t>(row) * kInter + ib * kBlk + 4 * lane;
  *reinterpret_cast<uint32_t*>(p.c_hi + off) = phi;
  *reinterpret_cast<uint32_t*>(p.c_lo + off) = plo;
  if (lane == 0) p.c_scale[static_cast<int64_t>(ib) * p.cap + row] = amax * (1.0f / 448.0f);
}

}  // namespace moe
