// One-shot all-reduce of small tensor-parallel messages over NVLink peer memory.
//
// Row-parallel projections (O, down) leave a partial residual on every rank that must be summed
// (16 KB - 256 KB at decode batch sizes), twice per layer, and the vocab-parallel sampler needs
// the maximum of B packed argmax keys. The reference has no multi-GPU path; this kernel stands
// where ncclAllReduce would after each row-parallel projection. At these sizes a collective is
// pure latency, so the message is cut into chunks (1 KB and up, at most P2P_MAX_CHUNKS) and one
// CTA per chunk, in parallel on as many SMs,
//   1. writes its chunk into slot [parity][rank] of every peer's receive buffer (plain stores
//      to peer memory opened with CUDA IPC, so the copies go straight over NVLink/NVSwitch),
//   2. after a system-scope fence, stores the chunk's epoch into flag [parity][rank][chunk] of
//      every peer,
//   3. waits (bounded by peers.wait_ns, one second in the engine, then VSL_ERR_TIMEOUT) until
//      the N flags [parity][*][chunk] of its own buffer carry the epoch, and
//   4. sums the chunk's N slots in rank order (so every rank computes identical bits).
// Each chunk keeps its own epoch, a device counter advanced by every call that covers the chunk,
// so a captured CUDA graph replays with fresh epochs. Chunk c always covers the same bytes of a
// slot, slots alternate by the chunk's epoch parity, and for one chunk a rank can be at most one
// call ahead of any peer (it cannot finish call k + 1 before every peer has pushed k + 1, which
// each does after finishing k on its stream), so a slot is never overwritten while still read.
// A CTA whose wait times out still advances its epoch, so this rank's counters stay equal to
// those of the ranks whose flags arrived; its chunk is left unreduced and the sticky status
// reports it. Once the status holds VSL_ERR_TIMEOUT (an earlier exchange of the step gave up)
// the call only advances its epochs: the ranks are out of step, the engine reports the failure
// after the step, and each later exchange would otherwise wait out its bound again.
#include <cuda_runtime.h>

#include "common.cuh"
#include "launch.cuh"
#include "p2p_allreduce.h"
#include "trace.cuh"

VSL_TRACE_UNIT(p2p)

namespace vsl {

constexpr int AR_THREADS = 256;

__device__ __forceinline__ unsigned long long* ar_flag(void* base, const P2pPeers& pe, int par, int r, int c) {
    return reinterpret_cast<unsigned long long*>(static_cast<char*>(base) + pe.flag_off) +
           ((size_t)par * pe.n + r) * P2P_MAX_CHUNKS + c;
}

template <int OP>  // 0: fp32 sum, 1: u64 max
__global__ void __launch_bounds__(AR_THREADS) vsl_p2p_allreduce_kernel(void* data, int n, const P2pPeers peers) {
    __shared__ unsigned long long s_epoch;
    VSL_TRACE_ENTRY();
    pdl_wait();
    VSL_TRACE_RELEASED();
    pdl_launch_dependents();
    const int t = threadIdx.x, c = blockIdx.x;
    const int N = peers.n, rank = peers.rank;
    __shared__ int s_failed;
    if (t == 0) {
        s_epoch = peers.epoch[c] + 1;
        s_failed = peers.status && *(volatile int*)peers.status == VSL_ERR_TIMEOUT;
    }
    __syncthreads();
    const unsigned long long epoch = s_epoch;
    if (s_failed) {
        if (t == 0) peers.epoch[c] = epoch;
        VSL_TRACE_EXIT(peers.trace_id, 1002);
        return;
    }
    const int par = (int)(epoch & 1);
    constexpr int ES = OP == 0 ? 4 : 8;
    const size_t bytes = (size_t)n * ES;
    const size_t lo = (size_t)c * peers.chunk_bytes;
    const size_t len = min(bytes, lo + peers.chunk_bytes) - lo;  // > 0: the grid covers the message
    const char* src = static_cast<const char*>(data) + lo;
    const size_t slot = peers.slot_bytes;
    // 1. push this rank's chunk into slot [par][rank] of every rank (16-byte stores, then words)
    const size_t n16 = len / 16, n4 = (len - n16 * 16) / 4;
    for (size_t i = t; i < (size_t)N * n16; i += AR_THREADS) {
        const int r = (int)(i / n16);
        const size_t j = i - (size_t)r * n16;
        char* dst = static_cast<char*>(peers.base[r]) + ((size_t)par * N + rank) * slot + lo;
        reinterpret_cast<uint4*>(dst)[j] = reinterpret_cast<const uint4*>(src)[j];
    }
    for (size_t i = t; i < (size_t)N * n4; i += AR_THREADS) {
        const int r = (int)(i / n4);
        const size_t j = n16 * 4 + (i - (size_t)r * n4);
        char* dst = static_cast<char*>(peers.base[r]) + ((size_t)par * N + rank) * slot + lo;
        reinterpret_cast<uint32_t*>(dst)[j] = reinterpret_cast<const uint32_t*>(src)[j];
    }
    __threadfence_system();
    __syncthreads();
    // 2. announce: flag [par][rank][c] = epoch on every rank
    if (t < N) st_release_sys_u64(ar_flag(peers.base[t], peers, par, rank, c), epoch);
    // 3. wait for the N flags of this chunk in the local buffer
    bool ok = true;
    if (t < N) {
        const unsigned long long* f = ar_flag(peers.base[rank], peers, par, t, c);
        ok = ld_acquire_sys_u64(f) == epoch;
        if (!ok) {
            const unsigned long long t0 = globaltimer_ns();
            while (!ok) {
                for (int i = 0; i < 64 && !ok; i++) ok = ld_acquire_sys_u64(f) == epoch;
                if (!ok && globaltimer_ns() - t0 > peers.wait_ns) break;
            }
        }
    }
    if (__syncthreads_or(!ok)) {
        if (t == 0) {
            set_status(peers.status, VSL_ERR_TIMEOUT);
            peers.epoch[c] = epoch;
        }
        VSL_TRACE_EXIT(peers.trace_id, 1002);
        return;
    }
    __threadfence();
    // 4. reduce the chunk's N slots in rank order
    const char* local = static_cast<const char*>(peers.base[rank]) + (size_t)par * N * slot + lo;
    char* out = static_cast<char*>(data) + lo;
    if (OP == 0) {
        for (size_t i = t; i < n16; i += AR_THREADS) {
            float4 acc = __ldcg(reinterpret_cast<const float4*>(local) + i);
            for (int r = 1; r < N; r++) {
                const float4 v = __ldcg(reinterpret_cast<const float4*>(local + (size_t)r * slot) + i);
                acc.x += v.x;
                acc.y += v.y;
                acc.z += v.z;
                acc.w += v.w;
            }
            reinterpret_cast<float4*>(out)[i] = acc;
        }
        for (size_t i = n16 * 4 + t; i < len / 4; i += AR_THREADS) {
            float acc = __ldcg(reinterpret_cast<const float*>(local) + i);
            for (int r = 1; r < N; r++) acc += __ldcg(reinterpret_cast<const float*>(local + (size_t)r * slot) + i);
            reinterpret_cast<float*>(out)[i] = acc;
        }
    } else {
        for (size_t i = t; i < len / 8; i += AR_THREADS) {
            unsigned long long acc = __ldcg(reinterpret_cast<const unsigned long long*>(local) + i);
            for (int r = 1; r < N; r++) {
                const unsigned long long v = __ldcg(reinterpret_cast<const unsigned long long*>(local + (size_t)r * slot) + i);
                acc = v > acc ? v : acc;
            }
            reinterpret_cast<unsigned long long*>(out)[i] = acc;
        }
    }
    if (t == 0) peers.epoch[c] = epoch;
    VSL_TRACE_EXIT(peers.trace_id, 1000 + OP);
}

int p2p_allreduce(const P2pPeers& peers, void* data, int n, int op, cudaStream_t st) {
    const size_t es = op == 0 ? 4 : 8;
    if (n <= 0 || n > peers.cap || peers.n < 2 || peers.n > P2P_MAX_RANKS || peers.rank < 0 || peers.rank >= peers.n)
        return set_error(VSL_ERR_INVALID, "p2p_allreduce: %d elements (capacity %d) over %d ranks", n, peers.cap, peers.n);
    if (!data || ((uintptr_t)data & 15)) return set_error(VSL_ERR_INVALID, "p2p_allreduce: message must be 16-byte aligned");
    if (!peers.epoch || peers.slot_bytes % 256 || peers.slot_bytes < (size_t)n * es || peers.chunk_bytes % 256 ||
        peers.chunk_bytes == 0)
        return set_error(VSL_ERR_INVALID, "p2p_allreduce: slot stride %zu / chunk %zu", peers.slot_bytes,
                         peers.chunk_bytes);
    const size_t chunks = ((size_t)n * es + peers.chunk_bytes - 1) / peers.chunk_bytes;
    if (chunks > (size_t)P2P_MAX_CHUNKS)
        return set_error(VSL_ERR_INVALID, "p2p_allreduce: %zu chunks exceed %d", chunks, P2P_MAX_CHUNKS);
    P2pPeers pt = peers;
    pt.trace_id = VSL_TRACE_ID();
    cudaError_t e = op == 0 ? launch_k(vsl_p2p_allreduce_kernel<0>, dim3((unsigned)chunks), dim3(AR_THREADS), 0, st,
                                       data, n, pt)
                            : launch_k(vsl_p2p_allreduce_kernel<1>, dim3((unsigned)chunks), dim3(AR_THREADS), 0, st,
                                       data, n, pt);
    return launch_status(e, "p2p allreduce launch");
}

}  // namespace vsl

using vsl::set_error;

extern "C" int vsl_p2p_buffer_size(int n_ranks, size_t cap_bytes, size_t* bytes) {
    if (!bytes || n_ranks < 2 || n_ranks > vsl::P2P_MAX_RANKS || cap_bytes == 0)
        return set_error(VSL_ERR_INVALID, "p2p_buffer_size: %d ranks, %zu bytes", n_ranks, cap_bytes);
    *bytes = vsl::p2p_buffer_bytes(n_ranks, cap_bytes, nullptr);
    return VSL_OK;
}

extern "C" int vsl_p2p_allreduce(void* const* bases, int n_ranks, int rank, size_t cap_bytes, void* data, int n,
                                 int op, uint64_t* epochs, int* status, uint64_t wait_ns, void* stream) {
    if (!bases || n_ranks < 2 || n_ranks > vsl::P2P_MAX_RANKS || rank < 0 || rank >= n_ranks || cap_bytes == 0 ||
        (op != 0 && op != 1) || !epochs || wait_ns == 0)
        return set_error(VSL_ERR_INVALID, "p2p_allreduce: bad arguments (%d ranks, rank %d, op %d)", n_ranks, rank, op);
    vsl::P2pPeers p = {};
    for (int r = 0; r < n_ranks; r++) {
        if (!bases[r] || ((uintptr_t)bases[r] & 255))
            return set_error(VSL_ERR_INVALID, "p2p_allreduce: buffer of rank %d must be 256-byte aligned", r);
        p.base[r] = bases[r];
    }
    const size_t es = op == 0 ? 4 : 8;
    p.n = n_ranks;
    p.rank = rank;
    p.cap = (int)(cap_bytes / es);
    p.slot_bytes = vsl::p2p_slot_bytes(cap_bytes);
    p.chunk_bytes = vsl::p2p_chunk_bytes(cap_bytes);
    vsl::p2p_buffer_bytes(n_ranks, cap_bytes, &p.flag_off);
    p.epoch = reinterpret_cast<unsigned long long*>(epochs);
    p.status = status;
    p.wait_ns = wait_ns;
    return vsl::p2p_allreduce(p, data, n, op, (cudaStream_t)stream);
}
