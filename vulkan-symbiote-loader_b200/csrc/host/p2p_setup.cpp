// Host side of the peer-memory all-reduce: each rank allocates its receive buffer, the CUDA IPC
// handles are exchanged with one NCCL all-gather, and every rank opens its peers' buffers.
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <thread>
#include <vector>

#include "../kernels/p2p_allreduce.h"
#include "status.h"
#include "watchdog.h"

namespace vsl {

// The handle exchange on the engine's non-blocking communicator: wait (bounded) for the
// enqueue and for the stream, watching the communicator's asynchronous error.
static int exchange_wait(ncclComm_t comm, ncclResult_t r, cudaStream_t st) {
    auto now = [] { return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count(); };
    const double t0 = now(), limit = 120.0;
    while (r == ncclInProgress) {
        if (ncclCommGetAsyncError(comm, &r) != ncclSuccess) break;
        if (r == ncclInProgress && now() - t0 > limit) return set_error(VSL_ERR_TIMEOUT, "p2p handle exchange: timed out");
        std::this_thread::yield();
    }
    if (r != ncclSuccess) return set_error(VSL_ERR_NCCL, "p2p handle exchange: %s", ncclGetErrorString(r));
    cudaError_t qerr = cudaSuccess;
    const int rc = watched_wait(
        [&] {
            const cudaError_t e = cudaStreamQuery(st);
            if (e == cudaSuccess) return StreamPoll::Done;
            if (e == cudaErrorNotReady) return StreamPoll::Pending;
            qerr = e;
            return StreamPoll::Error;
        },
        [&] {
            ncclResult_t ae = ncclSuccess;
            if (ncclCommGetAsyncError(comm, &ae) != ncclSuccess) return true;
            return ae != ncclSuccess && ae != ncclInProgress;
        },
        [] {}, limit, now, [](unsigned long long) { std::this_thread::sleep_for(std::chrono::microseconds(100)); });
    if (rc == VSL_ERR_CUDA) return set_error(rc, "p2p handle exchange: %s", cudaGetErrorString(qerr));
    if (rc) return set_error(rc, "p2p handle exchange: a rank did not take part");
    return VSL_OK;
}

int p2p_setup(P2pPeers* out, void** local, void** opened, int rank, int n, int cap, int elem_bytes, void* comm,
              unsigned long long* epoch, int* status, cudaStream_t st) {
    if (n < 2 || n > P2P_MAX_RANKS) return set_error(VSL_ERR_UNSUPPORTED, "p2p: %d ranks", n);
    const size_t cap_bytes = (size_t)cap * elem_bytes;
    const size_t bytes = p2p_buffer_bytes(n, cap_bytes);
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
    if (e != cudaSuccess) {
        cudaFree(dh);
        return set_error(VSL_ERR_CUDA, "p2p handle staging: %s", cudaGetErrorString(e));
    }
    ncclResult_t r = ncclAllGather(static_cast<char*>(dh) + (size_t)rank * sizeof(h), dh, sizeof(h), ncclUint8,
                                   (ncclComm_t)comm, st);
    if (int rc = exchange_wait((ncclComm_t)comm, r, st)) {
        cudaFree(dh);
        return rc;
    }
    e = cudaMemcpy(all.data(), dh, (size_t)n * sizeof(h), cudaMemcpyDeviceToHost);
    cudaFree(dh);
    if (e != cudaSuccess) return set_error(VSL_ERR_CUDA, "p2p handle exchange: %s", cudaGetErrorString(e));
    P2pPeers p = {};
    p.n = n;
    p.rank = rank;
    p.cap = cap;
    p.slot_bytes = p2p_slot_bytes(cap_bytes);
    p.chunk_words = p2p_chunk_words(cap_bytes);
    p.epoch = epoch;
    p.status = status;
    p.wait_ns = 1000000000ull;  // one second
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
