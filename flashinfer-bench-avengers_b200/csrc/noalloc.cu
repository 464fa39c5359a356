// Allocation-free entry point: the full MoE layer for small batches with its
// scratch memory in a fixed array inside this library.
//
// Who needs it: callers that may not allocate device memory at call time --
// a runtime whose memory planner reserved every buffer up front and forbids
// cudaMalloc afterwards, host code that has no CUDA allocator of its own to
// hand out a workspace, or a real-time loop where an allocation's latency or
// failure is not acceptable. They pass inputs and the output only.
//
// The scratch is a file-scope __device__ array of kNoAllocScratchBytes. Every
// GPU that loads this library holds one such array until the process exits,
// which is why it is sized for small batches only (num_tokens <=
// MOE_B200_NOALLOC_MAX_TOKENS). In host code the array's name is only a
// host-side stand-in, never a device address: the device address is looked
// up with cudaGetSymbolAddress once per device (on that device's first call,
// with the device current) and handed to the kernels as their workspace.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "../../include/moe_b200.h"

namespace moe {
namespace {

// 24 MiB: the workspace of moe_b200_run for num_tokens <= 16 is 20.9 MiB.
constexpr size_t kNoAllocScratchBytes = MOE_B200_NOALLOC_SCRATCH_BYTES;

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
void* g_scratch_ptr[kMaxDevices] = {};
std::mutex g_scratch_mu;

// Device address of this device's scratch array; nullptr if the lookup fails.
void* scratch_for_current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess) {
      cudaGetLastError();  // clear the error so later calls see a clean state
      return nullptr;
    }
    g_scratch_ptr[dev] = ptr;
  }
  return g_scratch_ptr[dev];
}

}  // namespace
}  // namespace moe

extern "C" int moe_b200_run_noalloc(const float* routing_logits, const void* routing_bias,
                                    int routing_bias_dtype, const void* hidden_states,
                                    const float* hidden_states_scale, const void* gemm1_weights,
                                    const float* gemm1_weights_scale, const void* gemm2_weights,
                                    const float* gemm2_weights_scale, int64_t local_expert_offset,
                                    double routed_scaling_factor, int64_t num_tokens, void* output,
                                    void* stream) {
  if (num_tokens < 0) return MOE_B200_ERR_INVALID_ARGUMENT;
  // Larger batches do not fit the fixed scratch array.
  if (num_tokens > MOE_B200_NOALLOC_MAX_TOKENS) return MOE_B200_ERR_WORKSPACE_TOO_SMALL;
  const size_t need = moe_b200_workspace_bytes(num_tokens);
  if (need == 0 || need > moe::kNoAllocScratchBytes) return MOE_B200_ERR_WORKSPACE_TOO_SMALL;
  if (num_tokens == 0) return MOE_B200_OK;
  void* scratch = moe::scratch_for_current_device();
  if (scratch == nullptr) return MOE_B200_ERR_CUDA;
  // The layer treats its workspace as uninitialised and clears what must
  // start at zero, so the previous call's leftovers in the array are harmless.
  return moe_b200_run(routing_logits, routing_bias, routing_bias_dtype, hidden_states,
                      hidden_states_scale, gemm1_weights, gemm1_weights_scale, gemm2_weights,
                      gemm2_weights_scale, local_expert_offset, routed_scaling_factor, num_tokens,
                      output, scratch, moe::kNoAllocScratchBytes, stream);
}

// The status word of the allocation-free calls sits inside the fixed array,
// at the same offset as in any workspace, so the regular reader applies once
// the array's device address is known.
extern "C" int moe_b200_noalloc_read_status(uint32_t* status, void* stream) {
  if (status == nullptr) return MOE_B200_ERR_INVALID_ARGUMENT;
  void* scratch = moe::scratch_for_current_device();
  if (scratch == nullptr) return MOE_B200_ERR_CUDA;
  return moe_b200_read_status(scratch, status, stream);
}
