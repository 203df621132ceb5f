// One-shot NVLink peer-memory all-reduce for small tensor-parallel messages (p2p_allreduce.cu).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace vsl {

constexpr int P2P_MAX_RANKS = 8;

// Receive buffers of all ranks, as seen from this rank: base[r] points at rank r's buffer
// ([2 parities][n ranks][cap elements] of data, then [2][n] u64 flags at flag_off bytes).
struct P2pPeers {
    void* base[P2P_MAX_RANKS];
    int n, rank;
    int cap;                     // elements per slot
    size_t slot_bytes;           // stride between slots: cap * element size rounded up to 256
    size_t flag_off;             // byte offset of the flags in every buffer
    unsigned long long* epoch;   // device counter of completed calls (this rank)
    int* status;                 // VSL_ERR_TIMEOUT when a peer's message never arrives
};

// A projection's role in a fused tensor-parallel sum (reduce on read, see GemvParams): mode 1
// = row-parallel producer, 2 = consumer whose input is the sum of the ranks' rows (written back
// to x_out); done = this rank's two arrival counters (zero between calls).
struct ArFuse {
    int mode;
    const P2pPeers* peers;
    unsigned int* done;
    float* x_out;
};

// op 0: in-place fp32 sum of n floats; op 1: in-place max of n u64 keys. One launch on `st`.
int p2p_allreduce(const P2pPeers& peers, void* data, int n, int op, cudaStream_t st);

// Buffer bytes for a capacity of `cap` elements of `elem_bytes` over `n` ranks. Every slot starts
// on a 256-byte boundary (the kernel moves 16-byte vectors; a slot of 3 u64 keys is 24 bytes).
inline size_t p2p_slot_bytes(int cap, int elem_bytes) { return ((size_t)cap * elem_bytes + 255) / 256 * 256; }
inline size_t p2p_buffer_bytes(int n, int cap, int elem_bytes, size_t* flag_off) {
    const size_t off = (size_t)2 * n * p2p_slot_bytes(cap, elem_bytes);
    if (flag_off) *flag_off = off;
    return off + (size_t)2 * P2P_MAX_RANKS * 8;
}

}  // namespace vsl
