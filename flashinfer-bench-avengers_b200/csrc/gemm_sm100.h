// Host-side launch interface of the grouped tcgen05 GEMMs (gemm_sm100.cu).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include "moe_kernels.cuh"

namespace moe {

// Launches one grouped GEMM flavour (GemmKind) with token-tile width `bn`
// on `grid` persistent CTAs. Returns cudaErrorInvalidValue for an
// unsupported (kind, bn) pair. With `early_tables` the kernel reads the
// segment table (and issues its first weight tiles) before waiting for its
// predecessor; that is only correct when the permutation finished before the
// predecessor released its dependents (every kernel between them waits first).
cudaError_t launch_moe_gemm(int kind, int bn, const CUtensorMap& w, const CUtensorMap& b0,
                            const CUtensorMap& b1, const GemmParams& p, int grid,
                            bool early_tables, cudaStream_t stream);

bool gemm_config_supported(int kind, int bn);

// Token-major grouped GEMM (gemm_tm_sm100.cu) for prefill-size batches:
// 128 token rows x 256 weight rows per tile. GEMM1 (gemm1 = true) reads the
// permuted activations through `a0`; GEMM2 reads the hi / lo parts of C
// through `a0` / `a1`. Both token maps must use 128-row boxes.
cudaError_t launch_moe_gemm_tm(bool gemm1, const CUtensorMap& w, const CUtensorMap& a0,
                               const CUtensorMap& a1, const GemmParams& p, int grid,
                               cudaStream_t stream);

}  // namespace moe
