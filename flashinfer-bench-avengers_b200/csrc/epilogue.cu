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

// Combine row r becomes output row slot_tok[r], for the *n_touched rows in
// use; with slot_tok null, all num_tokens rows are converted (row r =
// token r). Output rows of tokens without a combine row (no local
// pick) are not touched here: route_kernel has written their zeros. A CTA
// step covers one 2048-column segment of a row (4 per row); a thread
// converts 8 columns (two float4 loads, one 16-byte store).
__global__ void __launch_bounds__(256) finalize_kernel(const float* y_acc, const int32_t* slot_tok,
                                                       const int* n_touched, uint16_t* out, int num_tokens) {
  pdl_launch_next();
  pdl_wait();
  constexpr int kOcts = kHidden / 8;   // 896 groups of 8 columns per row
  constexpr int kSegs = 4;             // ceil(896 / 256)
  const int rows = slot_tok != nullptr ? min(*n_touched, num_tokens) : num_tokens;
  const int items = rows * kSegs;
  for (int it = blockIdx.x; it < items; it += gridDim.x) {
    const int r = it / kSegs;
    const int j = (it % kSegs) * 256 + threadIdx.x;
    if (j >= kOcts) continue;
    const int t = slot_tok != nullptr ? __ldg(slot_tok + r) : r;
    uint4* orow = reinterpret_cast<uint4*>(out + static_cast<int64_t>(t) * kHidden);
    const float4* yrow = reinterpret_cast<const float4*>(y_acc + static_cast<int64_t>(r) * kHidden);
    {
      const float4 a = yrow[2 * j];
      const float4 b = yrow[2 * j + 1];
      const __nv_bfloat162 p0 = __floats2bfloat162_rn(a.x, a.y);
      const __nv_bfloat162 p1 = __floats2bfloat162_rn(a.z, a.w);
      const __nv_bfloat162 p2 = __floats2bfloat162_rn(b.x, b.y);
      const __nv_bfloat162 p3 = __floats2bfloat162_rn(b.z, b.w);
      orow[j] = make_uint4(*reinterpret_cast<const uint32_t*>(&p0), *reinterpret_cast<const uint32_t*>(&p1),
                           *reinterpret_cast<const uint32_t*>(&p2), *reinterpret_cast<const uint32_t*>(&p3));
    }
  }
}

}  // namespace moe
