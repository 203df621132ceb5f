// One-shot NVLink peer-memory all-reduce for small tensor-parallel messages (p2p_allreduce.cu).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace vsl {

constexpr int P2P_MAX_RANKS = 8;
constexpr int P2P_MAX_CHUNKS = 64;  // CTAs of one call at most (one per chunk of the message)

// Receive buffers of all ranks, as seen from this rank: base[r] points at rank r's buffer
// ([2 parities][n ranks][slot_bytes] of data, then [2][n][P2P_MAX_CHUNKS] u64 flags at
// flag_off bytes). A message is cut into chunks of chunk_bytes, fixed for the buffer, so chunk
// c always covers the same bytes of every slot; one CTA moves and reduces one chunk.
struct P2pPeers {
    void* base[P2P_MAX_RANKS];
    int n, rank;
    int cap;                     // elements per slot
    size_t slot_bytes;           // stride between slots: cap * element size rounded up to 256
    size_t chunk_bytes;          // bytes per chunk (a multiple of 256)
    size_t flag_off;             // byte offset of the flags in every buffer
    unsigned long long* epoch;   // [P2P_MAX_CHUNKS] device call counters of this rank, one per chunk
    int* status;                 // VSL_ERR_TIMEOUT when a peer's message never arrives
    unsigned long long wait_ns;  // bound of the wait for the peers' flags
    unsigned trace_id;           // launch id of the trace build (unused otherwise)
};

// op 0: in-place fp32 sum of n floats; op 1: in-place max of n u64 keys. One launch on `st`.
int p2p_allreduce(const P2pPeers& peers, void* data, int n, int op, cudaStream_t st);

// Buffer geometry for messages of up to cap_bytes over `n` ranks. Every slot starts on a
// 256-byte boundary (the kernel moves 16-byte vectors; a slot of 3 u64 keys is 24 bytes);
// chunks are at least 1 KB and at most P2P_MAX_CHUNKS per message.
inline size_t p2p_slot_bytes(size_t cap_bytes) { return (cap_bytes + 255) / 256 * 256; }
inline size_t p2p_chunk_bytes(size_t cap_bytes) {
    const size_t per = (p2p_slot_bytes(cap_bytes) + P2P_MAX_CHUNKS - 1) / P2P_MAX_CHUNKS;
    const size_t c = (per + 255) / 256 * 256;
    return c < 1024 ? 1024 : c;
}
inline size_t p2p_buffer_bytes(int n, size_t cap_bytes, size_t* flag_off) {
    const size_t off = (size_t)2 * n * p2p_slot_bytes(cap_bytes);
    if (flag_off) *flag_off = off;
    return off + (size_t)2 * n * P2P_MAX_CHUNKS * 8;
}

}  // namespace vsl
