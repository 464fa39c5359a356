// Host-side launch interface of the grouped tcgen05 GEMMs (gemm_sm100.cu).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include "moe_kernels.cuh"

namespace moe {

// Launches one grouped GEMM flavour (GemmKind) with token-tile width `bn`
// on `grid` persistent CTAs. Returns cudaErrorInvalidValue for an
// unsupported (kind, bn) pair.
cudaError_t launch_moe_gemm(int kind, int bn, const CUtensorMap& w, const CUtensorMap& b0,
                            const CUtensorMap& b1, const GemmParams& p, int grid,
                            cudaStream_t stream);

bool gemm_config_supported(int kind, int bn);

}  // namespace moe
