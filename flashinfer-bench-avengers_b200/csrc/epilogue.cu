// Element-wise kernels around the grouped GEMMs.
//
// swiglu_quant_kernel   decode path only: after the K-split GEMM1 has summed
//                       its slices into fp32, apply C = silu(gate) * up
//                       (solution/cuda/kernel.h:207 semantics) and write the
//                       hi/lo e4m3 pair with one scale per (row, 128-block).
// finalize_kernel       fp32 combine buffer -> bf16 output (the reference's
//                       final cast, solution/cuda/main.cpp:141).
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cstdint>

#include "moe_kernels.cuh"
#include "moe_ptx.cuh"
#include "moe_shapes.cuh"

namespace moe {

// One warp per (row, 128-block); lane l owns columns 4l .. 4l+3.
__global__ void __launch_bounds__(256) swiglu_quant_kernel(const int* seg_off, const float* g1_acc,
                                                           uint8_t* c_hi, uint8_t* c_lo,
                                                           float* c_scale, int cap) {
  pdl_launch_next();
  pdl_wait();
  const int rows = seg_off[kExpertsLocal];
  const int lane = threadIdx.x & 31;
  const int warps_total = gridDim.x * (blockDim.x >> 5);
  for (int task = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); task < rows * kInterBlocks;
       task += warps_total) {
    const int row = task / kInterBlocks;
    const int ib = task % kInterBlocks;
    const float* g = g1_acc + static_cast<int64_t>(row) * kGemm1Out + ib * kBlk + 4 * lane;
    const float4 up = *reinterpret_cast<const float4*>(g);
    const float4 gate = *reinterpret_cast<const float4*>(g + kInter);
    float h[4];
    const float u[4] = {up.x, up.y, up.z, up.w};
    const float gg[4] = {gate.x, gate.y, gate.z, gate.w};
    float amax = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      h[j] = gg[j] / (1.0f + expf(-gg[j])) * u[j];
      amax = fmaxf(amax, fabsf(h[j]));
    }
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
    *reinterpret_cast<uint32_t*>(c_hi + off) = phi;
    *reinterpret_cast<uint32_t*>(c_lo + off) = plo;
    if (lane == 0) c_scale[static_cast<int64_t>(ib) * cap + row] = amax * (1.0f / 448.0f);
  }
}

// n4 = number of float4 groups (T * 7168 / 4).
__global__ void __launch_bounds__(256) finalize_kernel(const float* y_acc, uint16_t* out, int64_t n4) {
  pdl_launch_next();
  pdl_wait();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4; i += stride) {
    const float4 v = reinterpret_cast<const float4*>(y_acc)[i];
    const __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y);
    const __nv_bfloat162 b = __floats2bfloat162_rn(v.z, v.w);
    uint2 o;
    o.x = *reinterpret_cast<const uint32_t*>(&a);
    o.y = *reinterpret_cast<const uint32_t*>(&b);
    reinterpret_cast<uint2*>(out)[i] = o;
  }
}

}  // namespace moe
