// Standalone form of the hidden-state quantiser of hidden_quant.cuh:
// bf16 [T, 7168] -> e4m3 [T, 7168] and fp32 block scales [56, T] (block
// major, the layout the layer reads). One warp per token, 8 tokens per CTA.
// The layer entry point that takes bf16 hidden states does not use it: it
// quantises each row inside its row copy into the permuted buffers.
#include <cstdint>

#include "hidden_quant.cuh"
#include "moe_kernels.cuh"
#include "moe_shapes.cuh"

namespace moe {

__global__ void __launch_bounds__(256) quantize_hidden_kernel(const uint16_t* hidden_bf16, int num_tokens,
                                                              uint8_t* hidden_fp8, float* hidden_scale) {
  const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (t >= num_tokens) return;
  quantize_row_1x128(hidden_bf16 + static_cast<int64_t>(t) * kHidden, hidden_fp8 + static_cast<int64_t>(t) * kHidden,
                     threadIdx.x & 31,
                     [&](int kb, float sc) { hidden_scale[static_cast<int64_t>(kb) * num_tokens + t] = sc; });
}

}  // namespace moe
