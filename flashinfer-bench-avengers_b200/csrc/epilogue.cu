// Element-wise kernel after the grouped GEMMs.
//
// finalize_kernel       fp32 combine buffer -> bf16 output (the reference's
//                       final cast, solution/cuda/main.cpp:141).
#include <cuda_bf16.h>
#include <cstdint>

#include "moe_kernels.cuh"
#include "moe_ptx.cuh"
#include "moe_shapes.cuh"

namespace moe {

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
