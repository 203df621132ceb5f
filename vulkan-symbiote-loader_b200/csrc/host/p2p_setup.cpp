// Host side of the peer-memory all-reduce: each rank allocates its receive buffer, the CUDA IPC
// handles are exchanged with one NCCL all-gather, and every rank opens its peers' buffers.
#include <nccl.h>

#include <cstring>
#include <vector>

#include "../kernels/p2p_allreduce.h"
#include "status.h"

namespace vsl {

int p2p_setup(P2pPeers* out, void** local, void** opened, int rank, int n, int cap, int elem_bytes, void* comm,
              unsigned long long* epoch, int* status, cudaStream_t st) {
    if (n < 2 || n > P2P_MAX_RANKS) return set_error(VSL_ERR_UNSUPPORTED, "p2p: %d ranks", n);
    size_t flag_off = 0;
    const size_t bytes = p2p_buffer_bytes(n, cap, elem_bytes, &flag_off);
    cudaError_t e = cudaMalloc(local, bytes);
    if (e != cudaSuccess) return set_error(VSL_ERR_OOM, "p2p buffer: %s", cudaGetErrorString(e));
    e = cudaMemset(*local, 0, bytes);
    if (e != cudaSuccess) return set_error(VSL_ERR_CUDA, "p2p buffer clear: %s", cudaGetErrorString(e));
    cudaIpcMemHandle_t h;
    e = cudaIpcGetMemHandle(&h, *local);
    if (e != cudaSuccess) return set_error(VSL_ERR_CUDA, "cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
    // exchange the handles: all-gather of n x 64 bytes through a device buffer
    void* dh = nullptr;
    e = cudaMalloc(&dh, (size_t)n * sizeof(h));
    if (e != cudaSuccess) return set_error(VSL_ERR_OOM, "p2p handles: %s", cudaGetErrorString(e));
    std::vector<cudaIpcMemHandle_t> all(n);
    e = cudaMemcpy(static_cast<char*>(dh) + (size_t)rank * sizeof(h), &h, sizeof(h), cudaMemcpyHostToDevice);
    ncclResult_t r = ncclAllGather(static_cast<char*>(dh) + (size_t)rank * sizeof(h), dh, sizeof(h), ncclUint8,
                                   (ncclComm_t)comm, st);
    if (r != ncclSuccess) {
        cudaFree(dh);
        return set_error(VSL_ERR_NCCL, "p2p handle exchange: %s", ncclGetErrorString(r));
    }
    e = cudaStreamSynchronize(st);
    if (e == cudaSuccess) e = cudaMemcpy(all.data(), dh, (size_t)n * sizeof(h), cudaMemcpyDeviceToHost);
    cudaFree(dh);
    if (e != cudaSuccess) return set_error(VSL_ERR_CUDA, "p2p handle exchange: %s", cudaGetErrorString(e));
    P2pPeers p = {};
    p.n = n;
    p.rank = rank;
    p.cap = cap;
    p.slot_bytes = p2p_slot_bytes(cap, elem_bytes);
    p.flag_off = flag_off;
    p.epoch = epoch;
    p.status = status;
    for (int i = 0; i < n; i++) {
        if (i == rank) {
            p.base[i] = *local;
            opened[i] = nullptr;
            continue;
        }
        void* ptr = nullptr;
        e = cudaIpcOpenMemHandle(&ptr, all[i], cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess)
            return set_error(VSL_ERR_CUDA, "cudaIpcOpenMemHandle(rank %d): %s", i, cudaGetErrorString(e));
        p.base[i] = ptr;
        opened[i] = ptr;
    }
    *out = p;
    return VSL_OK;
}

void p2p_teardown(void* local, void** opened, int n) {
    for (int i = 0; i < n; i++)
        if (opened[i]) cudaIpcCloseMemHandle(opened[i]);
    if (local) cudaFree(local);
}

}  // namespace vsl
