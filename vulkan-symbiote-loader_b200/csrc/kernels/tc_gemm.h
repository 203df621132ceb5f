// Batched decode projections on tcgen05 tensor cores (tc_gemm.cu).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>

#include "../host/kernels.h"
#include "epilogue.cuh"

namespace vsl {

// Device workspace one projection needs: split activations [2*Bp][K] (16-bit), per-CTA
// partials of split row tiles, and one arrival counter per row tile (zero before first use;
// the kernel leaves them zero).
size_t tc_workspace_bytes(int N, int K, int B);
bool tc_supported(int wdtype, int N, int K, int B);

// y = epilogue(x·Wᵀ) for B rows through the tensor cores (activation split + GEMM, two
// launches on `st`). `kind` is an EK_* epilogue; `p` carries its parameters as for the GEMV.
int tc_project(int wdtype, int kind, const GemvParams& p, void* workspace, size_t ws_bytes, int* status,
               cudaStream_t st);

}  // namespace vsl
