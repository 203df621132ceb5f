// Program of the fused decode step: an ordered list of phases that one persistent
// cooperative kernel executes per token, with a grid barrier after each phase.
// Shared by the kernel (fused_step.cu) and the engine that builds it (engine.cpp).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace vsl {

enum FsPhaseKind { FS_EMBED = 0, FS_GEMV = 1, FS_ATTN = 2, FS_ATTN_COMBINE = 3, FS_FINAL = 4 };

struct FsPhase {
    int kind;
    int epi;      // projection epilogue (EK_*) for FS_GEMV
    int layer;    // KV cache of FS_GEMV(EK_QKV) / FS_ATTN
    int N, K;     // projection rows and inner dimension
    const void* W;
    const float* x;       // activations [B][K]
    float* y;             // output of STORE / ADD / SWIGLU / LMHEAD
    const float* norm_w;  // RMSNorm weights applied to x first (nullable)
    // tile geometry of the weight stream: tiles of R rows by kc columns (rows longer than kc
    // are cut into n_kc pieces); the consumer warps form 8/cg row groups of 8 rows by cg
    // column groups (see fs_geometry)
    int R, kc, n_kc, cg;
};

struct FsKV {
    void* k;
    void* v;
};

struct FsProgram {
    const FsPhase* phases;
    int n_phases;
    int n_barriers;
    const FsKV* kv;
    int B, d, nh, nkv, hd, wdtype, kvdtype;
    float eps;
    // embedding
    const void* tok_embd;
    int V;
    // paged KV cache, RoPE
    const int32_t* page_table;
    int max_pages, page_size, max_seq;
    const float* rope_cos;
    const float* rope_sin;
    // activations
    float* x;
    float* q;
    float* attn;
    float* att_ws;  // [B][nh][max_chunks][hd + 2]: per-chunk (o, m, l)
    int max_chunks;
    // sampler and bookkeeping
    float* logits;
    int V_local, vocab_offset;
    float inv_temp;
    unsigned long long seed;
    unsigned long long* slots;
    int32_t* ids;
    int32_t* pos;
    int32_t* step;
    const int32_t* forced;
    const int32_t* n_forced;
    int32_t* log;
    int log_cap;
    int32_t* sampled;
    int* status;
    // grid barrier state: arrival counter, its value at the start of the next launch, abort flag
    unsigned long long* bar_counter;
    unsigned long long* bar_epoch;
    int* abort_flag;
    // optional trace: %globaltimer (ns) at kernel start and after every phase barrier,
    // written by CTA 0 ([n_phases + 1] entries; nullptr = off)
    unsigned long long* trace;
};

// Dynamic shared memory of the fused kernel (bytes) and its limits.
constexpr int FS_STAGES = 4;
constexpr int FS_CHUNK = 32768;
constexpr int FS_WORK = 65536;
constexpr int FS_HEAD = 256;
constexpr size_t FS_DYN_SMEM = (size_t)FS_HEAD + (size_t)FS_STAGES * FS_CHUNK + FS_WORK;

// Tile geometry for a projection with K inputs of `es`-byte weights (`vec` weights per 16-byte
// vector). The 8 consumer warps form 8/cg row groups x cg column groups; a warp owns 8 rows
// of a tile and 1/cg of its columns, so every activation it loads from shared memory serves 8
// rows, and its partial sums stay in registers across all pieces of a row (the cross-warp
// reduction runs once per row group, not once per tile).
//   * rows of at least 4 KB: pieces of 4 KB (kc = 4096/es), 8 rows per tile, cg = 8
//     (a warp's slice of a piece is 32 vectors: one per lane);
//   * shorter rows stay whole (one contiguous copy per tile) and cg shrinks so that a slice
//     keeps 32 vectors where the row allows it, with up to 8 * 8/cg rows per 32 KB tile.
// R is even so that row pairs (gate/up, RoPE) never straddle a tile.
inline void fs_geometry(int K, int es, int vec, int* R, int* kc, int* n_kc, int* cg) {
    const int piece = 4096 / es;
    if (K >= piece) {
        *kc = piece;
        *n_kc = (K + piece - 1) / piece;
        *cg = 8;
        *R = 8;
        return;
    }
    int c = 8;
    while (c > 1 && K / c < 32 * vec) c >>= 1;
    const long long row = (long long)K * es;
    int r = 8 * (8 / c);
    if ((long long)r * row > FS_CHUNK) r = (int)(FS_CHUNK / row);
    r &= ~1;
    if (r < 2) r = 2;
    *kc = K;
    *n_kc = 1;
    *cg = c;
    *R = r;
}

int fused_step_launch(const FsProgram& prog, int grid, cudaStream_t st);
int fused_step_max_grid(int* grid);

}  // namespace vsl
