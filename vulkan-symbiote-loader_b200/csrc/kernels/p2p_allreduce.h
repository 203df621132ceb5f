// One-shot NVLink peer-memory all-reduce for small tensor-parallel messages (p2p_allreduce.cu).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace vsl {

constexpr int P2P_MAX_RANKS = 8;
constexpr int P2P_MAX_CHUNKS = 64;  // CTAs of one call at most (one per chunk of the message)

// Receive buffers of all ranks, as seen from this rank: base[r] points at rank r's buffer,
// [2 parities][n ranks][slot_bytes]. A slot holds a message as 8-byte words, each a 32-bit piece
// of the message and the 32-bit epoch of the call that wrote it, so a reader knows a word has
// arrived from the word itself. A message is cut into chunks of chunk_words 32-bit pieces (fixed
// per buffer, so chunk c always covers the same words of every slot); one CTA moves and reduces
// one chunk.
struct P2pPeers {
    void* base[P2P_MAX_RANKS];
    int n, rank;
    int cap;                     // elements per message at most
    size_t slot_bytes;           // bytes per slot: 8 per 32-bit piece of the largest message, rounded up to 256
    int chunk_words;             // 32-bit pieces per chunk (even)
    unsigned long long* epoch;   // [P2P_MAX_CHUNKS] device call counters of this rank, one per chunk
    int* status;                 // VSL_ERR_TIMEOUT when a peer's message never arrives
    unsigned long long wait_ns;  // bound of the wait for the peers' words
    unsigned trace_id;           // launch id of the trace build (unused otherwise)
};

// op 0: in-place fp32 sum of n floats; op 1: in-place max of n u64 keys. One launch on `st`.
int p2p_allreduce(const P2pPeers& peers, void* data, int n, int op, cudaStream_t st);

// Buffer geometry for messages of up to cap_bytes (a multiple of 4) over `n` ranks: slots start on
// 256-byte boundaries; chunks hold at least 256 pieces (1 KB of message) and a message has at most
// P2P_MAX_CHUNKS of them.
inline size_t p2p_slot_bytes(size_t cap_bytes) { return ((cap_bytes / 4 + 1) / 2 * 16 + 255) / 256 * 256; }
inline int p2p_chunk_words(size_t cap_bytes) {
    const size_t words = (cap_bytes / 4 + 1) / 2 * 2;
    size_t per = (words + P2P_MAX_CHUNKS - 1) / P2P_MAX_CHUNKS;
    per = (per + 1) / 2 * 2;
    return (int)(per < 256 ? 256 : per);
}
inline size_t p2p_buffer_bytes(int n, size_t cap_bytes) { return (size_t)2 * n * p2p_slot_bytes(cap_bytes); }

}  // namespace vsl
