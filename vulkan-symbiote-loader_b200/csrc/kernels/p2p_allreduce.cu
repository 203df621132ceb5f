// One-shot all-reduce of small tensor-parallel messages over NVLink peer memory.
//
// Row-parallel projections (O, down) leave a partial residual on every rank that must be summed
// (8 KB - 64 KB at decode batch sizes), twice per layer, and the vocab-parallel sampler needs
// the maximum of B packed argmax keys. At these sizes a collective is pure latency, so each
// rank runs one CTA that
//   1. writes its message into slot [parity][rank] of every peer's receive buffer (plain stores
//      to peer memory opened with CUDA IPC, so the copies go straight over NVLink/NVSwitch),
//   2. after a system-scope fence, stores the call's epoch into flag [parity][rank] of every peer,
//   3. waits (bounded: one second, then VSL_ERR_TIMEOUT) until all N flags of its own buffer
//      carry the epoch, and
//   4. reduces the N slots in rank order (so every rank computes the identical result).
// The epoch is a device counter advanced by every call, so a captured CUDA graph replays with
// fresh epochs; receive slots alternate by epoch parity, and a rank can only be one call ahead
// of any peer (it cannot finish call k + 1 before every peer has pushed k + 1, which each does
// after finishing k), so a slot is never overwritten while still being read.
#include <cuda_runtime.h>

#include "common.cuh"
#include "launch.cuh"
#include "p2p_allreduce.h"

namespace vsl {

constexpr int AR_THREADS = 1024;

template <int OP>  // 0: fp32 sum, 1: u64 max
__global__ void __launch_bounds__(AR_THREADS, 1) vsl_p2p_allreduce_kernel(void* data, int n, const P2pPeers peers) {
    __shared__ unsigned long long s_epoch;
    __shared__ int s_ok;
    pdl_wait();
    pdl_launch_dependents();
    const int t = threadIdx.x;
    const int N = peers.n, rank = peers.rank;
    if (t == 0) {
        s_epoch = *peers.epoch + 1;
        s_ok = 1;
    }
    __syncthreads();
    const unsigned long long epoch = s_epoch;
    const int par = (int)(epoch & 1);
    constexpr int ES = OP == 0 ? 4 : 8;
    const size_t slot_bytes = peers.slot_bytes;  // multiple of 256
    // 1. push this rank's message into slot [par][rank] of every rank (16-byte stores where possible)
    const size_t bytes = (size_t)n * ES;
    const size_t n16 = bytes / 16;
    for (int r = 0; r < N; r++) {
        char* dst = static_cast<char*>(peers.base[r]) + ((size_t)par * N + rank) * slot_bytes;
        const uint4* s4 = static_cast<const uint4*>(data);
        for (size_t i = t; i < n16; i += AR_THREADS) reinterpret_cast<uint4*>(dst)[i] = s4[i];
        for (size_t i = n16 * 16 + t * 4; i < bytes; i += (size_t)AR_THREADS * 4)
            *reinterpret_cast<uint32_t*>(dst + i) = *reinterpret_cast<const uint32_t*>(static_cast<const char*>(data) + i);
    }
    __threadfence_system();
    __syncthreads();
    // 2. announce: flag [par][rank] = epoch on every rank
    if (t < N) {
        unsigned long long* f = reinterpret_cast<unsigned long long*>(static_cast<char*>(peers.base[t]) + peers.flag_off) +
                                (size_t)par * N + rank;
        st_release_sys_u64(f, epoch);
    }
    // 3. wait for all N messages of this epoch in the local buffer
    if (t < N) {
        const unsigned long long* f =
            reinterpret_cast<const unsigned long long*>(static_cast<const char*>(peers.base[rank]) + peers.flag_off) +
            (size_t)par * N + t;
        bool ok = ld_acquire_sys_u64(f) == epoch;
        if (!ok) {
            const unsigned long long t0 = globaltimer_ns();
            while (!ok) {
                for (int i = 0; i < 64 && !ok; i++) ok = ld_acquire_sys_u64(f) == epoch;
                if (!ok && globaltimer_ns() - t0 > WAIT_LIMIT_NS) break;
            }
        }
        if (!ok) {
            s_ok = 0;
            set_status(peers.status, VSL_ERR_TIMEOUT);
        }
    }
    __syncthreads();
    if (!s_ok) return;
    __threadfence();
    // 4. reduce the N slots in rank order
    const char* local = static_cast<const char*>(peers.base[rank]) + (size_t)par * N * slot_bytes;
    if (OP == 0) {
        float* x = static_cast<float*>(data);
        const int n4 = n / 4;
        for (int i = t; i < n4; i += AR_THREADS) {
            float4 acc = __ldcg(reinterpret_cast<const float4*>(local) + i);
            for (int r = 1; r < N; r++) {
                const float4 v = __ldcg(reinterpret_cast<const float4*>(local + (size_t)r * slot_bytes) + i);
                acc.x += v.x;
                acc.y += v.y;
                acc.z += v.z;
                acc.w += v.w;
            }
            reinterpret_cast<float4*>(x)[i] = acc;
        }
        for (int i = n4 * 4 + t; i < n; i += AR_THREADS) {
            float acc = __ldcg(reinterpret_cast<const float*>(local) + i);
            for (int r = 1; r < N; r++) acc += __ldcg(reinterpret_cast<const float*>(local + (size_t)r * slot_bytes) + i);
            x[i] = acc;
        }
    } else {
        unsigned long long* x = static_cast<unsigned long long*>(data);
        for (int i = t; i < n; i += AR_THREADS) {
            unsigned long long acc = __ldcg(reinterpret_cast<const unsigned long long*>(local) + i);
            for (int r = 1; r < N; r++) {
                const unsigned long long v = __ldcg(reinterpret_cast<const unsigned long long*>(local + (size_t)r * slot_bytes) + i);
                acc = v > acc ? v : acc;
            }
            x[i] = acc;
        }
    }
    if (t == 0) *peers.epoch = epoch;
}

int p2p_allreduce(const P2pPeers& peers, void* data, int n, int op, cudaStream_t st) {
    if (n <= 0 || n > peers.cap || peers.n < 2 || peers.n > P2P_MAX_RANKS)
        return set_error(VSL_ERR_INVALID, "p2p_allreduce: %d elements (capacity %d) over %d ranks", n, peers.cap, peers.n);
    if ((uintptr_t)data & 15) return set_error(VSL_ERR_INVALID, "p2p_allreduce: message must be 16-byte aligned");
    if (peers.slot_bytes % 256 || peers.slot_bytes < (size_t)n * (op == 0 ? 4 : 8))
        return set_error(VSL_ERR_INVALID, "p2p_allreduce: slot stride %zu", peers.slot_bytes);
    cudaError_t e = op == 0 ? launch_k(vsl_p2p_allreduce_kernel<0>, dim3(1), dim3(AR_THREADS), 0, st, data, n, peers)
                            : launch_k(vsl_p2p_allreduce_kernel<1>, dim3(1), dim3(AR_THREADS), 0, st, data, n, peers);
    return launch_status(e, "p2p allreduce launch");
}

}  // namespace vsl
