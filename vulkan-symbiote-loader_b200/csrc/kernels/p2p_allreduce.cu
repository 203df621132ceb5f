// One-shot all-reduce of small tensor-parallel messages over NVLink peer memory.
//
// Row-parallel projections (O, down) leave a partial residual on every rank that must be summed
// (16 KB - 256 KB at decode batch sizes), twice per layer, and the vocab-parallel sampler needs
// the maximum of B packed argmax keys. The reference has no multi-GPU path; this kernel stands
// where ncclAllReduce would after each row-parallel projection. At these sizes a collective is
// pure latency, so the exchange carries its own arrival signal: the message is stored as 8-byte
// words, each a 32-bit piece of the message beside the 32-bit epoch of the call, written by one
// 16-byte store per two pieces. A naturally aligned 8-byte half of such a store is seen whole or
// not at all, so a reader that finds the epoch in a word also finds that word's piece, and no
// memory fence or separate flag is needed between the data and the signal (a system-scope fence
// per call measured 10-13 us of a single exchange's time). The message is cut into chunks (1 KB
// of message and up, at most P2P_MAX_CHUNKS) and one CTA per chunk, in parallel on as many SMs,
//   1. writes its chunk into slot [parity][rank] of every rank's receive buffer (plain stores to
//      peer memory opened with CUDA IPC, so they go straight over NVLink/NVSwitch), then
//   2. reads the chunk's N slots of its own buffer, waiting (bounded by peers.wait_ns, one second
//      in the engine, then VSL_ERR_TIMEOUT) until every word carries the epoch, and sums them in
//      rank order (so every rank computes identical bits).
// Each chunk keeps its own epoch, a device counter advanced by every call that covers the chunk,
// so a captured CUDA graph replays with fresh epochs. Chunk c always covers the same words of a
// slot, slots alternate by the chunk's epoch parity, and for one chunk a rank can be at most one
// call ahead of any peer (it cannot finish call k + 1 before every peer has pushed k + 1, which
// each does after finishing k on its stream), so a slot is never overwritten while still read.
// A CTA whose wait times out still advances its epoch, so this rank's counters stay equal to
// those of the ranks whose words arrived; its chunk is left partly unreduced and the sticky
// status reports it. Once the status holds VSL_ERR_TIMEOUT (an earlier exchange of the step gave
// up) the call only advances its epochs: the ranks are out of step, the engine reports the
// failure after the step, and each later exchange would otherwise wait out its bound again.
#include <cuda_runtime.h>

#include "common.cuh"
#include "launch.cuh"
#include "p2p_allreduce.h"
#include "trace.cuh"

VSL_TRACE_UNIT(p2p)

namespace vsl {

constexpr int AR_THREADS = 256;

// one 16-byte word pair {piece0, tag, piece1, tag}
__device__ __forceinline__ void st_pair(void* p, uint32_t w0, uint32_t w1, uint32_t tag) {
    asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(w0), "r"(tag), "r"(w1), "r"(tag)
                 : "memory");
}
__device__ __forceinline__ uint4 ld_pair(const void* p) {
    uint4 v;
    asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p)
                 : "memory");
    return v;
}
// epoch tag of a word: never 0 (zero-filled buffers hold no arrival) and distinct for 2^31 calls
__device__ __forceinline__ uint32_t ar_tag(unsigned long long epoch) {
    return (uint32_t)(epoch & 0x7fffffffull) | 0x80000000u;
}

template <int OP>  // 0: fp32 sum, 1: u64 max
__global__ void __launch_bounds__(AR_THREADS) vsl_p2p_allreduce_kernel(void* data, int n, const P2pPeers peers) {
    __shared__ unsigned long long s_epoch;
    __shared__ int s_failed;
    VSL_TRACE_ENTRY();
    pdl_wait();
    VSL_TRACE_RELEASED();
    pdl_launch_dependents();
    const int t = threadIdx.x, c = blockIdx.x;
    const int N = peers.n, rank = peers.rank;
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
    const uint32_t tag = ar_tag(epoch);
    const int par = (int)(epoch & 1);
    constexpr int PPE = OP == 0 ? 1 : 2;  // 32-bit pieces per element
    const int nw = n * PPE;
    const int lo = c * peers.chunk_words;                 // even
    const int len = min(nw, lo + peers.chunk_words) - lo;  // > 0: the grid covers the message
    const int npairs = (len + 1) / 2;
    const uint32_t* src = static_cast<const uint32_t*>(data) + lo;
    const size_t slot = peers.slot_bytes;
    // 1. push: the chunk's pieces, two per 16-byte store, into slot [par][rank] of every rank
    for (int i = t; i < N * npairs; i += AR_THREADS) {
        const int r = i / npairs, k = i - r * npairs, j = 2 * k;
        const uint32_t w0 = src[j], w1 = j + 1 < len ? src[j + 1] : 0u;
        st_pair(static_cast<char*>(peers.base[r]) + ((size_t)par * N + rank) * slot + (size_t)(lo + j) * 8, w0, w1,
                tag);
    }
    __syncthreads();  // every piece of `data` read before the sums overwrite it
    // 2. the N slots of this chunk in the local buffer, summed in rank order as they arrive
    const char* local = static_cast<const char*>(peers.base[rank]) + (size_t)par * N * slot + (size_t)lo * 8;
    bool ok = true;
    for (int k = t; k < npairs && ok; k += AR_THREADS) {
        const int j = 2 * k;
        const bool two = j + 1 < len;
        float a0 = 0.0f, a1 = 0.0f;
        unsigned long long m = 0ull;
        for (int r = 0; r < N && ok; r++) {
            const char* p = local + (size_t)r * slot + (size_t)j * 8;
            uint4 v = ld_pair(p);
            if (v.y != tag || (two && v.w != tag)) {
                const unsigned long long t0 = globaltimer_ns();
                while (v.y != tag || (two && v.w != tag)) {
                    for (int it = 0; it < 32 && (v.y != tag || (two && v.w != tag)); it++) v = ld_pair(p);
                    if ((v.y != tag || (two && v.w != tag)) && globaltimer_ns() - t0 > peers.wait_ns) {
                        ok = false;
                        break;
                    }
                }
            }
            if (OP == 0) {
                const float x0 = __uint_as_float(v.x), x1 = __uint_as_float(v.z);
                a0 = r ? a0 + x0 : x0;
                a1 = r ? a1 + x1 : x1;
            } else {
                const unsigned long long key = ((unsigned long long)v.z << 32) | v.x;
                m = (r == 0 || key > m) ? key : m;
            }
        }
        if (!ok) break;
        uint32_t* out = static_cast<uint32_t*>(data) + lo + j;
        if (OP == 0) {
            out[0] = __float_as_uint(a0);
            if (two) out[1] = __float_as_uint(a1);
        } else {
            *reinterpret_cast<unsigned long long*>(out) = m;
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
    if (t == 0) peers.epoch[c] = epoch;
    VSL_TRACE_EXIT(peers.trace_id, 1000 + OP);
}

int p2p_allreduce(const P2pPeers& peers, void* data, int n, int op, cudaStream_t st) {
    const size_t es = op == 0 ? 4 : 8;
    if (n <= 0 || n > peers.cap || peers.n < 2 || peers.n > P2P_MAX_RANKS || peers.rank < 0 || peers.rank >= peers.n)
        return set_error(VSL_ERR_INVALID, "p2p_allreduce: %d elements (capacity %d) over %d ranks", n, peers.cap, peers.n);
    if (!data || ((uintptr_t)data & 15)) return set_error(VSL_ERR_INVALID, "p2p_allreduce: message must be 16-byte aligned");
    const size_t words = (size_t)n * es / 4;
    if (!peers.epoch || peers.slot_bytes % 256 || peers.slot_bytes < (words + 1) / 2 * 16 || peers.chunk_words <= 0 ||
        (peers.chunk_words & 1))
        return set_error(VSL_ERR_INVALID, "p2p_allreduce: slot stride %zu / chunk %d", peers.slot_bytes,
                         peers.chunk_words);
    for (int r = 0; r < peers.n; r++)
        if (!peers.base[r] || ((uintptr_t)peers.base[r] & 255))
            return set_error(VSL_ERR_INVALID, "p2p_allreduce: buffer of rank %d must be 256-byte aligned", r);
    const size_t chunks = (words + peers.chunk_words - 1) / peers.chunk_words;
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
    if (!bytes || n_ranks < 2 || n_ranks > vsl::P2P_MAX_RANKS || cap_bytes == 0 || cap_bytes % 4)
        return set_error(VSL_ERR_INVALID, "p2p_buffer_size: %d ranks, %zu bytes", n_ranks, cap_bytes);
    *bytes = vsl::p2p_buffer_bytes(n_ranks, cap_bytes);
    return VSL_OK;
}

extern "C" int vsl_p2p_allreduce(void* const* bases, int n_ranks, int rank, size_t cap_bytes, void* data, int n,
                                 int op, uint64_t* epochs, int* status, uint64_t wait_ns, void* stream) {
    if (!bases || n_ranks < 2 || n_ranks > vsl::P2P_MAX_RANKS || rank < 0 || rank >= n_ranks || cap_bytes == 0 ||
        cap_bytes % 4 || (op != 0 && op != 1) || !epochs || wait_ns == 0)
        return set_error(VSL_ERR_INVALID, "p2p_allreduce: bad arguments (%d ranks, rank %d, op %d)", n_ranks, rank, op);
    vsl::P2pPeers p = {};
    for (int r = 0; r < n_ranks; r++) p.base[r] = bases[r];
    const size_t es = op == 0 ? 4 : 8;
    p.n = n_ranks;
    p.rank = rank;
    p.cap = (int)(cap_bytes / es);
    p.slot_bytes = vsl::p2p_slot_bytes(cap_bytes);
    p.chunk_words = vsl::p2p_chunk_words(cap_bytes);
    p.epoch = reinterpret_cast<unsigned long long*>(epochs);
    p.status = status;
    p.wait_ns = wait_ns;
    return vsl::p2p_allreduce(p, data, n, op, (cudaStream_t)stream);
}
