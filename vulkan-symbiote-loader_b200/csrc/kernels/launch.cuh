// Host-side launch helpers shared by the kernel translation units.
#pragma once
#include <cuda_runtime.h>

#include "../host/status.h"

namespace vsl {

// Streaming multiprocessor count of the current device (cached per device).
int sm_count();

// Whether kernels are launched with programmatic dependent launch (process-wide switch;
// the engine turns it off when asked to).
bool pdl_enabled();
void set_pdl_enabled(bool on);

// Launch `kernel` on `stream` with the programmatic-stream-serialization attribute, so the
// kernel may begin while its predecessor on the stream drains (it calls pdl_wait() before
// touching the predecessor's outputs).
template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                     Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

inline int launch_status(cudaError_t e, const char* what) {
    if (e != cudaSuccess) return set_error(VSL_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    return VSL_OK;
}

}  // namespace vsl
