// Split-K flash-decode attention over the paged KV cache (GQA-aware).
//
// Replaces the dense attention of the reference (vk_symbiote/shaders/attention.comp:84-189,
// dispatched from attention_with_weights, VulkanSymbioteEngine.cpp:2440-2584), which makes
// three passes over K per (head, position). Semantics kept: query head h reads KV group
// h*n_kv/n_heads (attention.comp:92), scores are q.k / sqrt(head_dim), softmax with max
// subtraction over positions [0, pos], output = probabilities times V.
//
// Design: one CTA per (split, kv group, sequence). A sequence's positions are cut into at most
// n_splits splits of at least split_min positions, sized from the sequence's current length on the
// device (a short cache takes one split and no combine; a long one spreads over the n_splits CTAs).
// A CTA stages 64-position chunks of K and V (one page-contiguous block each) through a ring of
// shared-memory buffers filled by bulk asynchronous copies (TMA: one copy per chunk of K and of V,
// completion on one mbarrier per buffer; rows land unpadded and every thread reads its 16-byte
// columns in an order rotated by its row, so the score reads stay free of bank conflicts), computes the scores of all G = n_heads/n_kv query heads of its group from
// the same staged K (so a KV page is read from HBM once per group, not once per head), and keeps
// an online softmax (running max / sum, fp32). With 256 threads the scores split each position's
// dot product into four partial sums and the P.V product splits the positions among two (head_dim
// 128) or four (head_dim 64) thread groups, combined once at the end in a fixed order. Splits
// write (max, sum, partial output) to the workspace; the last CTA of a (sequence, group) to
// finish -- found with an atomic counter that it resets to zero -- combines them, so one launch
// does both phases.
#include <cuda_runtime.h>
#include <math_constants.h>

#include <mutex>

#include "common.cuh"
#include "launch.cuh"
#include "trace.cuh"

VSL_TRACE_UNIT(attention)

namespace vsl {

// 256 threads: a chunk's scores and P.V spread over 8 warps. (A 128-thread form capped at 64
// registers, small enough to become resident beside the preceding projection's CTAs, measured
// slower: 16 us per layer against 11-12 us at 7B batch 1.)
constexpr int FD_THREADS = 256;
constexpr int FD_MIN_CTAS = 2;  // two CTAs per SM: a long cache's splits fit in one wave
constexpr int FD_CHUNK = 64;  // positions staged per iteration
constexpr int FD_GMAX = 8;    // query heads per KV group supported
constexpr int FD_PARTS = FD_THREADS / FD_CHUNK;  // partial sums per position score

struct FdParams {
    const float* q;
    const void* k_cache;
    const void* v_cache;
    const int32_t* page_table;
    int max_pages, page_size;
    const int32_t* pos;
    int B, n_heads, n_kv;
    int split_min;   // positions per split at least (a multiple of FD_CHUNK)
    int n_splits;    // splits per (sequence, group) at most: the grid's x
    int max_len;     // positions the caller's cache covers
    float scale;
    float* out;
    float* ws_o;   // [B][n_heads][n_splits][HD]
    float* ws_ml;  // [B][n_heads][n_splits][2]
    int* counters; // [B][n_kv]
    const void* pf_ptr;  // weights of the projection that follows (prefetched into L2)
    size_t pf_bytes;
    int wait_first;      // rows share one sequence's pages (prompt chunk): no cache read before the wait
    SparseMask sp;       // long-context sparse mask (sp.min_len 0: dense)
    int* status;         // VSL_ERR_TIMEOUT if a staging wait ever expires (may be null)
    unsigned trace_id;   // launch id of the trace build (unused otherwise)
};

template <typename KT> struct KvVec;
template <> struct KvVec<float> {
    static constexpr int VEC = 4;
    __device__ __forceinline__ static void widen(const uint4& v, float* f) { WTraits<float>::widen(v, f); }
};
template <> struct KvVec<__half> {
    static constexpr int VEC = 8;
    __device__ __forceinline__ static void widen(const uint4& v, float* f) { WTraits<__half>::widen(v, f); }
};

template <int HD, typename KT>
__host__ __device__ constexpr int fd_row_elems() {
    return HD;  // rows as in the cache (bulk copies of whole chunks); reads rotate their columns
}
template <typename KT>
__host__ __device__ constexpr int fd_stages() {
    return sizeof(KT) == 2 ? 4 : 2;  // chunk buffers in the ring (fp32 rows are twice as large)
}

template <int HD, typename KT>
__host__ __device__ constexpr size_t fd_smem_bytes() {
    return (size_t)fd_stages<KT>() * 2 * FD_CHUNK * fd_row_elems<HD, KT>() * sizeof(KT)  // K and V chunk ring
           + (size_t)2 * FD_GMAX * HD * sizeof(float)                                  // q (padded columns)
           + (size_t)FD_PARTS * FD_GMAX * FD_CHUNK * sizeof(float)                     // score partials
           + (size_t)FD_GMAX * FD_CHUNK * sizeof(float)                                // probabilities
           + (size_t)(FD_THREADS / HD) * FD_GMAX * HD * sizeof(float)                  // P.V group partials
           + (size_t)4 * FD_GMAX * sizeof(float);                                      // m, l, alpha, misc
}

template <int HD, typename KT>
__global__ void __launch_bounds__(FD_THREADS, FD_MIN_CTAS) vsl_flash_decode_kernel(FdParams p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    constexpr int STAGES = fd_stages<KT>();
    constexpr int RE = fd_row_elems<HD, KT>();
    constexpr int VEC = KvVec<KT>::VEC;
    constexpr int VPR = HD / VEC;             // 16-byte vectors per row
    constexpr int NGRP = FD_THREADS / HD;     // position groups of the P.V product
    constexpr int PDIM = HD / FD_PARTS;       // head dimensions per score partial
    static_assert(PDIM % VEC == 0 && FD_THREADS % HD == 0 && (VPR % FD_PARTS) == 0, "attention tiling");
    KT* kv_s = reinterpret_cast<KT*>(smem_raw);  // [STAGES][K, V][CHUNK][RE]
    float* q_s = reinterpret_cast<float*>(kv_s + (size_t)STAGES * 2 * FD_CHUNK * RE);
    // q by 16-byte cache column, each column padded by one float: [GMAX][VPR][VEC + 1], so lanes
    // reading different columns hit different banks
    constexpr int QCOL = VEC + 1, QP = VPR * QCOL;
    float* part_s = q_s + 2 * FD_GMAX * HD;                // [PARTS][GMAX][CHUNK]
    float* p_s = part_s + FD_PARTS * FD_GMAX * FD_CHUNK;   // [GMAX][CHUNK]
    float* ored = p_s + FD_GMAX * FD_CHUNK;                // [NGRP][GMAX][HD]
    float* m_s = ored + NGRP * FD_GMAX * HD;               // [GMAX]
    float* l_s = m_s + FD_GMAX;
    float* a_s = l_s + FD_GMAX;
    __shared__ int is_last;
    __shared__ __align__(8) uint64_t kv_bar[4];  // one per ring buffer: its chunk's copies landed
    VSL_TRACE_ENTRY();

    const int split = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = p.n_heads / p.n_kv;

    // In decode, pos[] and the cache below position pos were written by kernels that finished
    // before the immediate predecessor started, so they are read before griddepcontrol.wait; the
    // predecessor (the QKV projection) writes q and the key/value row at pos. When the rows are
    // consecutive positions of one sequence (a prompt chunk), the predecessor also wrote the
    // rows below pos, so the kernel waits first (wait_first).
    // Positions past the page table or the caller's cache are never read (the QKV kernel has
    // already flagged such a position in the engine's status word).
    const int pos = p.pos[b];
    const int len = min(pos + 1, min(p.max_pages * p.page_size, p.max_len));
    // split length for this sequence's current length: at least split_min, at most n_splits splits
    const int S = max(p.split_min, ((len + p.n_splits - 1) / p.n_splits + FD_CHUNK - 1) / FD_CHUNK * FD_CHUNK);
    // sparse mask: the row attends to [lo, len); splits below lo take no part, the first active
    // split starts at lo's chunk and masks the rows below lo
    const int lo = min(sparse_first(p.sp, pos), len - 1);
    const int s_first = lo / S;
    const int n_total = (len + S - 1) / S;
    const int t_begin = (split < s_first || split >= n_total) ? len : max(split * S, lo & ~(FD_CHUNK - 1));
    if (t_begin >= len) {  // empty split: not counted by the combiner; it only prefetches
        if (p.pf_ptr && tid < 32) {
            const int nblk = gridDim.x * gridDim.y * gridDim.z;
            const int me = (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
            prefetch_share(p.pf_ptr, p.pf_bytes, me, nblk, tid, 32);
        }
        VSL_TRACE_EXIT(p.trace_id, 900);
        return;
    }
    const int t_end = min(len, (split + 1) * S);
    const int n_active = n_total - s_first;  // splits that take part
    const int n_chunks = (t_end - t_begin + FD_CHUNK - 1) / FD_CHUNK;
    const int new_row = pos - t_begin;  // row of the freshly appended position, if in this split
    if (p.wait_first) {
        pdl_wait();
        VSL_TRACE_RELEASED();
    }

    auto chunk_ptrs = [&](int ci, const KT*& kg, const KT*& vg) {
        const int t0 = t_begin + ci * FD_CHUNK;  // t0 % 64 == 0 and page_size % 64 == 0: one page
        const int page = p.page_table[(size_t)b * p.max_pages + t0 / p.page_size];
        const size_t base = (((size_t)page * p.n_kv + g) * p.page_size + (t0 % p.page_size)) * HD;
        kg = reinterpret_cast<const KT*>(p.k_cache) + base;
        vg = reinterpret_cast<const KT*>(p.v_cache) + base;
    };
    // stage chunk ci into ring buffer ci % STAGES: one thread announces the bytes on the buffer's
    // mbarrier and copies the chunk's K and V rows in one bulk copy each (two when the row `skip`,
    // left for later, sits inside the chunk)
    constexpr uint32_t ROW_BYTES = HD * sizeof(KT);  // a multiple of 16
    auto issue = [&](int ci, int skip) {
        if (tid != 0) return;
        const KT* kg;
        const KT* vg;
        chunk_ptrs(ci, kg, vg);
        const int n = min(FD_CHUNK, t_end - (t_begin + ci * FD_CHUNK));
        const int buf = ci % STAGES;
        KT* ks = kv_s + (size_t)(2 * buf) * FD_CHUNK * RE;
        KT* vs = ks + FD_CHUNK * RE;
        const int r = skip - ci * FD_CHUNK;  // row left out, if in [0, n)
        const bool cut = r >= 0 && r < n;
        mbar_arrive_expect_tx(&kv_bar[buf], (uint32_t)(n - (cut ? 1 : 0)) * 2 * ROW_BYTES);
        const int r0 = cut ? r : n;          // rows [0, r0) and [r1, n)
        const int r1 = cut ? r + 1 : n;
        if (r0 > 0) {
            bulk_g2s(ks, kg, (uint32_t)r0 * ROW_BYTES, &kv_bar[buf]);
            bulk_g2s(vs, vg, (uint32_t)r0 * ROW_BYTES, &kv_bar[buf]);
        }
        if (n > r1) {
            bulk_g2s(ks + (size_t)r1 * HD, kg + (size_t)r1 * HD, (uint32_t)(n - r1) * ROW_BYTES, &kv_bar[buf]);
            bulk_g2s(vs + (size_t)r1 * HD, vg + (size_t)r1 * HD, (uint32_t)(n - r1) * ROW_BYTES, &kv_bar[buf]);
        }
    };
    if (tid < STAGES) mbar_init(&kv_bar[tid], 1);
    if (tid == 0) mbar_fence_init();
    __syncthreads();

    // every chunk the ring holds is requested before the wait (older cache rows only)
    const int pre = min(n_chunks, STAGES);
    for (int ci = 0; ci < pre; ci++) issue(ci, new_row);
    int issued = pre;
    bool staged_ok = true;

    if (!p.wait_first) {
        pdl_wait();
        VSL_TRACE_RELEASED();
    }

    // the new row (if it sits in an already-issued chunk) and q, now that the QKV kernel is done;
    // the bulk copies never write that row
    if (new_row >= 0 && new_row < pre * FD_CHUNK) {
        const int ci = new_row / FD_CHUNK, r = new_row % FD_CHUNK;
        const KT* kg;
        const KT* vg;
        chunk_ptrs(ci, kg, vg);
        KT* ks = kv_s + (size_t)(2 * (ci % STAGES)) * FD_CHUNK * RE;
        KT* vs = ks + FD_CHUNK * RE;
        for (int i = tid; i < VPR; i += FD_THREADS) {
            *reinterpret_cast<uint4*>(ks + r * RE + i * VEC) = __ldcg(reinterpret_cast<const uint4*>(kg + (size_t)r * HD + i * VEC));
            *reinterpret_cast<uint4*>(vs + r * RE + i * VEC) = __ldcg(reinterpret_cast<const uint4*>(vg + (size_t)r * HD + i * VEC));
        }
    }
    const int h0 = g * G;
    for (int i = tid; i < G * HD; i += FD_THREADS) {
        const int j = i / HD, d = i - j * HD;
        q_s[j * QP + (d / VEC) * QCOL + d % VEC] = __ldcg(p.q + ((size_t)b * p.n_heads + h0) * HD + i);
    }
    if (tid < FD_GMAX) { m_s[tid] = -CUDART_INF_F; l_s[tid] = 0.0f; }

    const int e_own = tid % HD, grp = tid / HD;  // P.V: output element and position group
    float o_acc[FD_GMAX];
#pragma unroll
    for (int j = 0; j < FD_GMAX; j++) o_acc[j] = 0.0f;

    for (int ci = 0; ci < n_chunks; ci++) {
        const int buf = ci % STAGES;
        const int n = min(FD_CHUNK, t_end - (t_begin + ci * FD_CHUNK));
        // this chunk's copies (bounded wait; all threads decide together to stop)
        const bool late = !mbar_wait(&kv_bar[buf], (uint32_t)((ci / STAGES) & 1));
        if (__syncthreads_or(late)) {
            staged_ok = false;
            break;
        }
        const KT* k_s = kv_s + (size_t)(2 * buf) * FD_CHUNK * RE;
        const KT* v_s = k_s + FD_CHUNK * RE;
        // partial scores: thread (tt, part) covers 1/FD_PARTS of the head dimension of position tt,
        // the 16-byte columns c = (tt + part + FD_PARTS k) mod NCOL: the 8 lanes of a shared-memory
        // phase read 8 different bank groups of their (unpadded) rows
        {
            const int tt = tid & (FD_CHUNK - 1), part = tid / FD_CHUNK;
            if (tt < n) {
                float acc[FD_GMAX];
#pragma unroll
                for (int j = 0; j < FD_GMAX; j++) acc[j] = 0.0f;
                const KT* kr = k_s + tt * RE;
#pragma unroll
                for (int k = 0; k < PDIM / VEC; k++) {
                    const int c = ((tt + part + FD_PARTS * k) % VPR) * VEC;
                    float kf[VEC];
                    KvVec<KT>::widen(*reinterpret_cast<const uint4*>(kr + c), kf);
#pragma unroll
                    for (int j = 0; j < FD_GMAX; j++) {
                        if (j < G) {
#pragma unroll
                            for (int e = 0; e < VEC; e++) acc[j] = fmaf(q_s[j * QP + (c / VEC) * QCOL + e], kf[e], acc[j]);
                        }
                    }
                }
#pragma unroll
                for (int j = 0; j < FD_GMAX; j++)
                    if (j < G) part_s[(part * FD_GMAX + j) * FD_CHUNK + tt] = acc[j];
            }
        }
        __syncthreads();
        // online softmax per head: warp j handles head j
        const int t0 = t_begin + ci * FD_CHUNK;
        for (int j = warp; j < G; j += FD_THREADS / 32) {
            float s0 = -CUDART_INF_F, s1 = -CUDART_INF_F;
            if (lane < n && t0 + lane >= lo) {
                float a = 0.0f;
#pragma unroll
                for (int q = 0; q < FD_PARTS; q++) a += part_s[(q * FD_GMAX + j) * FD_CHUNK + lane];
                s0 = a * p.scale;
            }
            if (lane + 32 < n && t0 + lane + 32 >= lo) {
                float a = 0.0f;
#pragma unroll
                for (int q = 0; q < FD_PARTS; q++) a += part_s[(q * FD_GMAX + j) * FD_CHUNK + lane + 32];
                s1 = a * p.scale;
            }
            const float cmax = warp_max_redux(fmaxf(s0, s1));
            const float m_old = m_s[j];
            const float m_new = fmaxf(m_old, cmax);
            const float e0 = s0 != -CUDART_INF_F ? expf(s0 - m_new) : 0.0f;
            const float e1 = s1 != -CUDART_INF_F ? expf(s1 - m_new) : 0.0f;
            p_s[j * FD_CHUNK + lane] = e0;
            p_s[j * FD_CHUNK + lane + 32] = e1;
            const float csum = warp_sum(e0 + e1);
            if (lane == 0) {
                const float alpha = expf(m_old - m_new);  // 0 on the first chunk (m_old = -inf)
                a_s[j] = alpha;
                l_s[j] = l_s[j] * alpha + csum;
                m_s[j] = m_new;
            }
        }
        __syncthreads();
        // P V: thread (e_own, grp) sums the positions grp, grp + NGRP, ... of the chunk
        {
            float acc[FD_GMAX];
#pragma unroll
            for (int j = 0; j < FD_GMAX; j++) acc[j] = 0.0f;
#pragma unroll 8
            for (int i = 0; i < FD_CHUNK / NGRP; i++) {
                const int tt = grp + i * NGRP;
                if (tt < n) {
                    const float vv = (float)v_s[tt * RE + e_own];
#pragma unroll
                    for (int j = 0; j < FD_GMAX; j++)
                        if (j < G) acc[j] = fmaf(p_s[j * FD_CHUNK + tt], vv, acc[j]);
                }
            }
#pragma unroll
            for (int j = 0; j < FD_GMAX; j++)
                if (j < G) o_acc[j] = o_acc[j] * a_s[j] + acc[j];
        }
        __syncthreads();  // buffer `buf` is free again
        if (issued < n_chunks) {
            issue(issued, -1);
            issued++;
        }
    }
    // The next projection's weights are requested into L2, and its CTAs allowed to start (they
    // request their own heads), only now that this split's cache has landed: issued earlier, those
    // tens of megabytes of prefetches queue in HBM ahead of the few cache chunks attention waits for.
    if (p.pf_ptr && tid < 32) {
        const int nblk = gridDim.x * gridDim.y * gridDim.z;
        const int me = (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
        prefetch_share(p.pf_ptr, p.pf_bytes, me, nblk, tid, 32);
    }
    pdl_launch_dependents();
    if (!staged_ok) {
        // a copy never landed: report it, let the copies still in flight finish (bounded), leave
        set_status(p.status, VSL_ERR_TIMEOUT);
        for (int ci = 0; ci < issued; ci++) mbar_wait(&kv_bar[ci % STAGES], (uint32_t)((ci / STAGES) & 1));
        VSL_TRACE_EXIT(p.trace_id, 904);
        return;
    }

    // ---- combine the position groups (fixed order), then write this split's result ----
#pragma unroll
    for (int j = 0; j < FD_GMAX; j++)
        if (j < G) ored[(grp * FD_GMAX + j) * HD + e_own] = o_acc[j];
    __syncthreads();
    if (tid < HD) {
#pragma unroll
        for (int j = 0; j < FD_GMAX; j++) {
            if (j >= G) continue;
            float o = ored[j * HD + tid];
#pragma unroll
            for (int q = 1; q < NGRP; q++) o += ored[(q * FD_GMAX + j) * HD + tid];
            o_acc[j] = o;
        }
    }
    if (n_active == 1) {  // a single split: its partial is the answer
        if (tid < HD) {
#pragma unroll
            for (int j = 0; j < FD_GMAX; j++)
                if (j < G) p.out[((size_t)b * p.n_heads + h0 + j) * HD + tid] = o_acc[j] / l_s[j];
        }
        VSL_TRACE_EXIT(p.trace_id, 901);
        return;
    }
#pragma unroll
    for (int j = 0; j < FD_GMAX; j++) {
        if (j >= G) continue;
        const size_t row = ((size_t)b * p.n_heads + h0 + j) * p.n_splits + split;
        if (tid < HD) p.ws_o[row * HD + tid] = o_acc[j];
        if (tid == 0) {
            p.ws_ml[row * 2 + 0] = m_s[j];
            p.ws_ml[row * 2 + 1] = l_s[j];
        }
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const int prev = atomicAdd(p.counters + (size_t)b * p.n_kv + g, 1);
        is_last = prev == n_active - 1;
    }
    __syncthreads();
    if (!is_last) {
        VSL_TRACE_EXIT(p.trace_id, 902);
        return;
    }
    __threadfence();
    // ---- combine the active splits of every head in this group ----
    // All G heads at once: the split statistics of a tile of splits are staged in shared memory
    // by all threads (one L2 round trip), then each thread sums its (head, dimension) elements
    // over the tile with eight loads in flight, so the combine costs a few round trips rather
    // than a few per head. Sums run in split order, as a sequential combine would.
    constexpr int EPT = (FD_GMAX * HD + FD_THREADS - 1) / FD_THREADS;  // output elements per thread
    constexpr int TS = (FD_PARTS * FD_GMAX * FD_CHUNK) / FD_GMAX;       // splits per staged tile
    float* cw = part_s;          // [TS][GMAX] exp(m_s - M_j)
    float* cl = ored;            // [TS][GMAX] l_s
    float* mx_s = p_s;           // [GMAX] per-head maxima
    float* l_tot = p_s + FD_GMAX;  // [GMAX] per-head sums
    float* redw = p_s + 2 * FD_GMAX;  // [warps][GMAX]
    const size_t hrow0 = ((size_t)b * p.n_heads + h0) * p.n_splits + s_first;  // head h0 + j: + j * n_splits
    {
        float mx[FD_GMAX];
#pragma unroll
        for (int j = 0; j < FD_GMAX; j++) {
            mx[j] = -CUDART_INF_F;
            if (j < G)
                for (int sp = tid; sp < n_active; sp += FD_THREADS)
                    mx[j] = fmaxf(mx[j], __ldcg(p.ws_ml + (hrow0 + (size_t)j * p.n_splits + sp) * 2));
        }
#pragma unroll
        for (int j = 0; j < FD_GMAX; j++) {
            if (j >= G) break;
            const float m = warp_max_redux(mx[j]);
            if (lane == 0) redw[warp * FD_GMAX + j] = m;
        }
        __syncthreads();
        if (tid < G) {
            float M = redw[tid];
            for (int w = 1; w < FD_THREADS / 32; w++) M = fmaxf(M, redw[w * FD_GMAX + tid]);
            mx_s[tid] = M;
            l_tot[tid] = 0.0f;
        }
    }
    float acc[EPT];
#pragma unroll
    for (int i = 0; i < EPT; i++) acc[i] = 0.0f;
    for (int t0 = 0; t0 < n_active; t0 += TS) {
        const int nt = min(TS, n_active - t0);
        __syncthreads();  // maxima written; the previous tile consumed
#pragma unroll
        for (int j = 0; j < FD_GMAX; j++) {
            if (j >= G) break;
            for (int sp = tid; sp < nt; sp += FD_THREADS) {
                const float2 ml = __ldcg(reinterpret_cast<const float2*>(p.ws_ml + (hrow0 + (size_t)j * p.n_splits + t0 + sp) * 2));
                cw[sp * FD_GMAX + j] = expf(ml.x - mx_s[j]);
                cl[sp * FD_GMAX + j] = ml.y;
            }
        }
        __syncthreads();
        if (tid < G)
            for (int sp = 0; sp < nt; sp++) l_tot[tid] += cl[sp * FD_GMAX + tid] * cw[sp * FD_GMAX + tid];
        // the thread's elements advance together, eight splits at a time: EPT x 8 loads in flight
        const float* src[EPT];
        int jj[EPT];
#pragma unroll
        for (int i = 0; i < EPT; i++) {
            const int e = min(tid + i * FD_THREADS, G * HD - 1);  // past G * HD: a duplicate, not stored
            jj[i] = e / HD;
            src[i] = p.ws_o + (hrow0 + (size_t)jj[i] * p.n_splits + t0) * HD + (e - jj[i] * HD);
        }
        int sp = 0;
        for (; sp + 8 <= nt; sp += 8) {
            float o[EPT][8];
#pragma unroll
            for (int i = 0; i < EPT; i++)
#pragma unroll
                for (int u = 0; u < 8; u++) o[i][u] = __ldcg(src[i] + (size_t)(sp + u) * HD);
#pragma unroll
            for (int i = 0; i < EPT; i++)
#pragma unroll
                for (int u = 0; u < 8; u++) acc[i] += o[i][u] * cw[(sp + u) * FD_GMAX + jj[i]];
        }
        for (; sp < nt; sp++)
#pragma unroll
            for (int i = 0; i < EPT; i++) acc[i] += __ldcg(src[i] + (size_t)sp * HD) * cw[sp * FD_GMAX + jj[i]];
    }
    __syncthreads();  // the last tile's sums are in l_tot
#pragma unroll
    for (int i = 0; i < EPT; i++) {
        const int e = tid + i * FD_THREADS;
        if (e >= G * HD) continue;
        const int j = e / HD, d = e - j * HD;
        p.out[((size_t)b * p.n_heads + h0 + j) * HD + d] = acc[i] / l_tot[j];
    }
    if (tid == 0) p.counters[(size_t)b * p.n_kv + g] = 0;
    VSL_TRACE_EXIT(p.trace_id, 903);
}

// ---------------------------------------------------------------------------------------
// Short caches: one CTA per (sequence, KV group), no split combine.
//
// At a few hundred positions the split-K kernel's cost is its dependent chain (a chunk per CTA,
// then partials through global memory and a last-CTA combine), not bytes. This form stages a
// whole round of positions (256 with fp16 KV, 128 with fp32: four or two 64-position chunks,
// each on its own mbarrier) and processes it at once with 512 threads: every position's score
// in parallel (PARTS threads per position, joined by shuffles), one block-wide maximum and sum,
// then P.V over NG position groups per head dimension, reduced once at the end. Longer caches
// take further rounds with the online softmax; the engine uses this kernel only while the cache
// is at most FS_MAX_LEN positions. Older rows are requested before griddepcontrol.wait, the row
// at pos (written by the predecessor) after it.
// ---------------------------------------------------------------------------------------
// Phase stamps of the trace build (thread 0, first round): [t0, t1] of a phase per CTA
#ifdef VSL_TRACE
#define FS_STAMP(var) const uint64_t var = vsl::trace_now()
#define FS_PHASE(tag, ta, tb) \
    if (tid == 0 && r == 0) vsl_trace_record(p.trace_id, (tag), (ta), (tb))
#else
#define FS_STAMP(var)
#define FS_PHASE(tag, ta, tb)
#endif
constexpr int FS_THREADS = 512;
constexpr int FS_WARPS = FS_THREADS / 32;
template <typename KT>
__host__ __device__ constexpr int fs_chunks() {
    return sizeof(KT) == 2 ? 4 : 2;  // 64-position chunks per round
}
template <int HD, typename KT>
__host__ __device__ constexpr size_t fs_smem_bytes() {
    constexpr int R = fs_chunks<KT>() * FD_CHUNK;
    return (size_t)2 * R * HD * sizeof(KT)                         // K and V of a round
           + (size_t)FD_GMAX * (HD / KvVec<KT>::VEC) * (KvVec<KT>::VEC + 1) * sizeof(float)  // q, padded columns
           + (size_t)FD_GMAX * R * sizeof(float)                    // scores / probabilities
           + (size_t)(FS_THREADS / HD) * FD_GMAX * HD * sizeof(float)  // P.V group partials
           + (size_t)2 * FS_WARPS * FD_GMAX * sizeof(float)          // warp maxima / sums
           + (size_t)4 * FD_GMAX * sizeof(float);                    // m, l, alpha
}

template <int HD, typename KT, int GT>  // GT: query heads per KV group, rounded up to 1, 2, 4 or 8
__global__ void __launch_bounds__(FS_THREADS, 1) vsl_flash_decode_short_kernel(FdParams p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    constexpr int NCH = fs_chunks<KT>();
    constexpr int R = NCH * FD_CHUNK;             // positions per round
    constexpr int PARTS = FS_THREADS / R;         // threads per position score
    constexpr int VEC = KvVec<KT>::VEC;
    constexpr int VPR = HD / VEC;                 // 16-byte vectors per row
    constexpr int NG = FS_THREADS / HD;           // position groups of P.V
    constexpr int QCOL = VEC + 1, QP = VPR * QCOL;
    static_assert(VPR % PARTS == 0 && R % NG == 0, "short attention tiling");
    KT* k_s = reinterpret_cast<KT*>(smem_raw);    // [R][HD]
    KT* v_s = k_s + (size_t)R * HD;               // [R][HD]
    float* q_s = reinterpret_cast<float*>(v_s + (size_t)R * HD);  // [GMAX][VPR][VEC + 1]
    float* s_s = q_s + FD_GMAX * QP;              // [GMAX][R]
    float* ored = s_s + FD_GMAX * R;              // [NG][GMAX][HD]
    float* red = ored + NG * FD_GMAX * HD;        // [2][WARPS][GMAX]
    float* m_s = red + 2 * FS_WARPS * FD_GMAX;    // [GMAX]
    float* l_s = m_s + FD_GMAX;
    float* a_s = l_s + FD_GMAX;
    __shared__ __align__(8) uint64_t bar[4];      // one per chunk of the round
    VSL_TRACE_ENTRY();

    const int g = blockIdx.x, b = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = p.n_heads / p.n_kv;
    const int pos = p.pos[b];
    const int len = min(pos + 1, min(p.max_pages * p.page_size, p.max_len));
    const int lo = min(sparse_first(p.sp, pos), len - 1);
    const int t_begin = lo & ~(FD_CHUNK - 1);
    const int n_rounds = (len - t_begin + R - 1) / R;
    const int new_row = pos - t_begin;  // position of the freshly appended row, relative to t_begin
    constexpr uint32_t ROW_BYTES = HD * sizeof(KT);

    auto chunk_ptrs = [&](int t0, const KT*& kg, const KT*& vg) {
        const int page = p.page_table[(size_t)b * p.max_pages + t0 / p.page_size];
        const size_t base = (((size_t)page * p.n_kv + g) * p.page_size + (t0 % p.page_size)) * HD;
        kg = reinterpret_cast<const KT*>(p.k_cache) + base;
        vg = reinterpret_cast<const KT*>(p.v_cache) + base;
    };
    // round r: chunk c (rows rb .. rb + n) into slot c; `skip` (relative to t_begin) is left out
    auto issue_round = [&](int r, int skip) {
        if (tid != 0) return;
        for (int c = 0; c < NCH; c++) {
            const int t0 = t_begin + r * R + c * FD_CHUNK;
            if (t0 >= len) break;
            const int n = min(FD_CHUNK, len - t0);
            const KT* kg;
            const KT* vg;
            chunk_ptrs(t0, kg, vg);
            KT* ks = k_s + (size_t)c * FD_CHUNK * HD;
            KT* vs = v_s + (size_t)c * FD_CHUNK * HD;
            const int rr = skip - (t0 - t_begin);
            const bool cut = rr >= 0 && rr < n;
            mbar_arrive_expect_tx(&bar[c], (uint32_t)(n - (cut ? 1 : 0)) * 2 * ROW_BYTES);
            const int r0 = cut ? rr : n, r1 = cut ? rr + 1 : n;
            if (r0 > 0) {
                bulk_g2s(ks, kg, (uint32_t)r0 * ROW_BYTES, &bar[c]);
                bulk_g2s(vs, vg, (uint32_t)r0 * ROW_BYTES, &bar[c]);
            }
            if (n > r1) {
                bulk_g2s(ks + (size_t)r1 * HD, kg + (size_t)r1 * HD, (uint32_t)(n - r1) * ROW_BYTES, &bar[c]);
                bulk_g2s(vs + (size_t)r1 * HD, vg + (size_t)r1 * HD, (uint32_t)(n - r1) * ROW_BYTES, &bar[c]);
            }
        }
    };
    if (tid < NCH) mbar_init(&bar[tid], 1);
    if (tid == 0) mbar_fence_init();
    __syncthreads();
    // round 0's older rows do not depend on the predecessor
    issue_round(0, new_row);
    pdl_wait();
    VSL_TRACE_RELEASED();
    FS_STAMP(ts_rel);
    // q and the new row, written by the QKV projection (a position past the cache is never read:
    // the QKV kernel has flagged it in the status word)
    if (pos < len && new_row < R) {
        const int c = new_row / FD_CHUNK, rr = new_row % FD_CHUNK;
        const KT* kg;
        const KT* vg;
        chunk_ptrs(t_begin + c * FD_CHUNK, kg, vg);
        for (int i = tid; i < VPR; i += FS_THREADS) {
            *reinterpret_cast<uint4*>(k_s + ((size_t)c * FD_CHUNK + rr) * HD + i * VEC) =
                __ldcg(reinterpret_cast<const uint4*>(kg + (size_t)rr * HD + i * VEC));
            *reinterpret_cast<uint4*>(v_s + ((size_t)c * FD_CHUNK + rr) * HD + i * VEC) =
                __ldcg(reinterpret_cast<const uint4*>(vg + (size_t)rr * HD + i * VEC));
        }
    }
    const int h0 = g * G;
    for (int i = tid; i < G * HD; i += FS_THREADS) {
        const int j = i / HD, d = i - j * HD;
        q_s[j * QP + (d / VEC) * QCOL + d % VEC] = __ldcg(p.q + ((size_t)b * p.n_heads + h0) * HD + i);
    }
    if (tid < FD_GMAX) {
        m_s[tid] = -CUDART_INF_F;
        l_s[tid] = 0.0f;
    }
    const int d_own = tid % HD, grp = tid / HD;  // P.V: head dimension and position group
    float o_acc[GT];
#pragma unroll
    for (int j = 0; j < GT; j++) o_acc[j] = 0.0f;
    bool staged_ok = true;
    int issued_rounds = 1;
    for (int r = 0; r < n_rounds; r++) {
        const int rb = t_begin + r * R;
        const int n = min(R, len - rb);
        const int nch = (n + FD_CHUNK - 1) / FD_CHUNK;
        bool late = false;
        for (int c = 0; c < nch; c++) late |= !mbar_wait(&bar[c], (uint32_t)(r & 1));
        if (__syncthreads_or(late)) {
            staged_ok = false;
            break;
        }
        FS_STAMP(ts_staged);
        FS_PHASE(2301u, ts_rel, ts_staged);
        // scores: PARTS adjacent threads per position, each over VPR / PARTS 16-byte columns in an
        // order rotated by the position (conflict-free reads of the unpadded rows)
        {
            const int tt = tid / PARTS, part = tid % PARTS;
            float acc[GT];
#pragma unroll
            for (int j = 0; j < GT; j++) acc[j] = 0.0f;
            if (tt < n) {
                const KT* kr = k_s + (size_t)tt * HD;
#pragma unroll
                for (int k = 0; k < VPR / PARTS; k++) {
                    const int cv = (part + PARTS * k + tt) % VPR;
                    float kf[VEC];
                    KvVec<KT>::widen(*reinterpret_cast<const uint4*>(kr + cv * VEC), kf);
#pragma unroll
                    for (int j = 0; j < GT; j++) {
                        if (j < G) {
#pragma unroll
                            for (int e = 0; e < VEC; e++) acc[j] = fmaf(q_s[j * QP + cv * QCOL + e], kf[e], acc[j]);
                        }
                    }
                }
            }
#pragma unroll
            for (int j = 0; j < GT; j++) {
                if (j >= G) break;
#pragma unroll
                for (int o = 1; o < PARTS; o <<= 1) acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], o);
            }
            if (part == 0) {
                const bool valid = tt < n && rb + tt >= lo;
#pragma unroll
                for (int j = 0; j < GT; j++)
                    if (j < G) s_s[j * R + tt] = valid ? acc[j] * p.scale : -CUDART_INF_F;
            }
        }
        __syncthreads();
        FS_STAMP(ts_scores);
        FS_PHASE(2302u, ts_staged, ts_scores);
        // maximum per head over the round
        for (int j = 0; j < G; j++) {
            const float v = tid < R ? s_s[j * R + tid] : -CUDART_INF_F;
            const float mx = warp_max_redux(v);
            if (lane == 0) red[warp * FD_GMAX + j] = mx;
        }
        __syncthreads();
        for (int j = 0; j < G; j++) {
            float cm = -CUDART_INF_F;
#pragma unroll
            for (int w = 0; w < R / 32; w++) cm = fmaxf(cm, red[w * FD_GMAX + j]);
            const float mo = m_s[j];
            const float mn = fmaxf(mo, cm);
            // probabilities in place, their sum per warp
            float e = 0.0f;
            if (tid < R) {
                const float sv = s_s[j * R + tid];
                e = sv != -CUDART_INF_F ? expf(sv - mn) : 0.0f;
                s_s[j * R + tid] = e;
            }
            const float sm = warp_sum(e);
            if (lane == 0) red[(FS_WARPS + warp) * FD_GMAX + j] = sm;
            if (tid == 0) a_s[j] = mo == -CUDART_INF_F ? 0.0f : expf(mo - mn);
        }
        __syncthreads();
        if (tid < G) {
            float sm = 0.0f;
#pragma unroll
            for (int w = 0; w < R / 32; w++) sm += red[(FS_WARPS + w) * FD_GMAX + tid];
            const float mo = m_s[tid];
            float cm = -CUDART_INF_F;
#pragma unroll
            for (int w = 0; w < R / 32; w++) cm = fmaxf(cm, red[w * FD_GMAX + tid]);
            m_s[tid] = fmaxf(mo, cm);
            l_s[tid] = l_s[tid] * a_s[tid] + sm;
        }
        FS_STAMP(ts_soft);
        FS_PHASE(2303u, ts_scores, ts_soft);
        // P.V: thread (d_own, grp) sums positions grp, grp + NG, ... of the round
        {
            float acc[GT];
#pragma unroll
            for (int j = 0; j < GT; j++) acc[j] = 0.0f;
#pragma unroll 4
            for (int i = grp; i < n; i += NG) {
                const float vv = (float)v_s[(size_t)i * HD + d_own];
#pragma unroll
                for (int j = 0; j < GT; j++)
                    if (j < G) acc[j] = fmaf(s_s[j * R + i], vv, acc[j]);
            }
#pragma unroll
            for (int j = 0; j < GT; j++)
                if (j < G) o_acc[j] = o_acc[j] * a_s[j] + acc[j];
        }
        __syncthreads();  // the round's buffers, scores and statistics are consumed
        FS_STAMP(ts_pv);
        FS_PHASE(2304u, ts_soft, ts_pv);
        if (r + 1 < n_rounds) {
            issue_round(r + 1, -1);  // rows after the wait: the new row is already in the cache
            issued_rounds++;
        }
    }
    if (p.pf_ptr && tid < 32) prefetch_share(p.pf_ptr, p.pf_bytes, blockIdx.y * gridDim.x + blockIdx.x,
                                             gridDim.x * gridDim.y, tid, 32);
    pdl_launch_dependents();
    if (!staged_ok) {
        set_status(p.status, VSL_ERR_TIMEOUT);
        // let the copies still in flight land (bounded) before the CTA leaves
        if (tid == 0) {
            const int r = issued_rounds - 1;
            for (int c = 0; c < NCH; c++)
                if (t_begin + r * R + c * FD_CHUNK < len) mbar_wait(&bar[c], (uint32_t)(r & 1));
        }
        __syncthreads();
        VSL_TRACE_EXIT(p.trace_id, 906);
        return;
    }
    // the position groups, in a fixed order
#pragma unroll
    for (int j = 0; j < GT; j++)
        if (j < G) ored[(grp * FD_GMAX + j) * HD + d_own] = o_acc[j];
    __syncthreads();
    for (int i = tid; i < G * HD; i += FS_THREADS) {
        const int j = i / HD, d = i - j * HD;
        float o = ored[j * HD + d];
#pragma unroll
        for (int q = 1; q < NG; q++) o += ored[(q * FD_GMAX + j) * HD + d];
        p.out[((size_t)b * p.n_heads + h0 + j) * HD + d] = o / l_s[j];
    }
    VSL_TRACE_EXIT(p.trace_id, 905);
}

template <int HD, typename KT, int GT>
static int launch_fs_g(const FdParams& p, cudaStream_t st) {
    auto kern = vsl_flash_decode_short_kernel<HD, KT, GT>;
    constexpr size_t smem = fs_smem_bytes<HD, KT>();
    static thread_local int configured_dev = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (configured_dev != dev) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return launch_status(e, "flash_decode_short smem attribute");
        configured_dev = dev;
    }
    FdParams pt = p;
    pt.trace_id = VSL_TRACE_ID();
    return launch_status(launch_k(kern, dim3(p.n_kv, p.B), dim3(FS_THREADS), smem, st, pt), "flash_decode_short launch");
}
template <int HD, typename KT>
static int launch_fs(const FdParams& p, cudaStream_t st) {
    const int G = p.n_heads / p.n_kv;
    if (G <= 1) return launch_fs_g<HD, KT, 1>(p, st);
    if (G <= 2) return launch_fs_g<HD, KT, 2>(p, st);
    if (G <= 4) return launch_fs_g<HD, KT, 4>(p, st);
    return launch_fs_g<HD, KT, 8>(p, st);
}

int flash_decode_short_impl(const float* q, const void* k_cache, const void* v_cache, int kvdtype,
                            const int32_t* page_table, int max_pages, int page_size, const int32_t* pos, int B,
                            int n_heads, int n_kv, int head_dim, int max_len, float* out, cudaStream_t stream,
                            const void* pf_ptr, size_t pf_bytes, const SparseMask* sparse, int* status) {
    if (!q || !k_cache || !v_cache || !page_table || !pos || !out)
        return set_error(VSL_ERR_INVALID, "flash_decode_short: null pointer");
    if (sparse && sparse->min_len > 0 && (sparse->window < 0 || sparse->global_tokens < 0 || sparse->block <= 0))
        return set_error(VSL_ERR_INVALID, "flash_decode_short: sparse mask window %d, global %d, block %d",
                         sparse->window, sparse->global_tokens, sparse->block);
    if (B <= 0 || n_heads <= 0 || n_kv <= 0 || n_heads % n_kv || n_heads / n_kv > FD_GMAX)
        return set_error(VSL_ERR_UNSUPPORTED, "flash_decode_short: heads %d / kv %d (group size <= %d)", n_heads,
                         n_kv, FD_GMAX);
    if (page_size <= 0 || page_size % FD_CHUNK)
        return set_error(VSL_ERR_INVALID, "flash_decode_short: page_size %d must be a multiple of %d", page_size,
                         FD_CHUNK);
    if (max_len <= 0 || max_len > max_pages * page_size)
        return set_error(VSL_ERR_INVALID, "flash_decode_short: max_len %d outside the page table", max_len);
    FdParams p = {};
    p.q = q; p.k_cache = k_cache; p.v_cache = v_cache; p.page_table = page_table; p.max_pages = max_pages;
    p.page_size = page_size; p.pos = pos; p.B = B; p.n_heads = n_heads; p.n_kv = n_kv;
    p.max_len = max_len; p.scale = 1.0f / sqrtf((float)head_dim); p.out = out;
    p.pf_ptr = pf_ptr;
    p.pf_bytes = pf_bytes;
    p.status = status;
    if (sparse) p.sp = *sparse;
    if (kvdtype == VSL_F16) {
        if (head_dim == 128) return launch_fs<128, __half>(p, stream);
        if (head_dim == 64) return launch_fs<64, __half>(p, stream);
    } else if (kvdtype == VSL_F32) {
        if (head_dim == 128) return launch_fs<128, float>(p, stream);
        if (head_dim == 64) return launch_fs<64, float>(p, stream);
    }
    return set_error(VSL_ERR_UNSUPPORTED, "flash_decode_short: head_dim %d / kv dtype %d", head_dim, kvdtype);
}

static size_t align256(size_t n) { return (n + 255) & ~(size_t)255; }

static int fd_splits(int max_len, int split_len) { return (max_len + split_len - 1) / split_len; }
size_t flash_decode_workspace_bytes(int B, int n_heads, int n_kv, int head_dim, int n_splits);

// Workspace: split partials from the front, split counters at the tail (+256 bytes of slack), so
// calls with fewer rows on the same workspace (a prompt pass's last chunk) find their counters
// inside the range every call leaves at zero, never under another call's partials.
static size_t fd_workspace(int B, int n_heads, int n_kv, int head_dim, int n_splits) {
    return align256((size_t)B * n_heads * n_splits * head_dim * sizeof(float)) +
           align256((size_t)B * n_heads * n_splits * 2 * sizeof(float)) +
           align256((size_t)B * n_kv * sizeof(int)) + 256;
}
size_t flash_decode_workspace_bytes(int B, int n_heads, int n_kv, int head_dim, int n_splits) {
    return fd_workspace(B, n_heads, n_kv, head_dim, n_splits);
}
static size_t fd_counters_offset(int B, int n_kv, size_t workspace_bytes) {
    return (workspace_bytes - (size_t)B * n_kv * sizeof(int)) & ~(size_t)255;
}

template <int HD, typename KT>
static int launch_fd(const FdParams& p, cudaStream_t st) {
    auto kern = vsl_flash_decode_kernel<HD, KT>;
    constexpr size_t smem = fd_smem_bytes<HD, KT>();
    static thread_local int configured_dev = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (configured_dev != dev) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return launch_status(e, "flash_decode smem attribute");
        configured_dev = dev;
    }
    dim3 grid(p.n_splits, p.n_kv, p.B);
    FdParams pt = p;
    pt.trace_id = VSL_TRACE_ID();
    return launch_status(launch_k(kern, grid, dim3(FD_THREADS), smem, st, pt), "flash_decode launch");
}

int flash_decode_impl(const float* q, const void* k_cache, const void* v_cache, int kvdtype,
                      const int32_t* page_table, int max_pages, int page_size, const int32_t* pos, int B,
                      int n_heads, int n_kv, int head_dim, int max_len, int split_len, float* out, void* workspace,
                      size_t workspace_bytes, cudaStream_t stream, const void* pf_ptr, size_t pf_bytes,
                      bool shared_pages, const SparseMask* sparse, int n_splits_max, int* status) {
    if (!q || !k_cache || !v_cache || !page_table || !pos || !out || !workspace)
        return set_error(VSL_ERR_INVALID, "flash_decode: null pointer");
    if (sparse && sparse->min_len > 0 && (sparse->window < 0 || sparse->global_tokens < 0 || sparse->block <= 0))
        return set_error(VSL_ERR_INVALID, "flash_decode: sparse mask window %d, global %d, block %d", sparse->window,
                         sparse->global_tokens, sparse->block);
    if (B <= 0 || n_heads <= 0 || n_kv <= 0 || n_heads % n_kv || n_heads / n_kv > FD_GMAX)
        return set_error(VSL_ERR_UNSUPPORTED, "flash_decode: heads %d / kv %d (group size <= %d)", n_heads, n_kv,
                         FD_GMAX);
    if (page_size <= 0 || page_size % FD_CHUNK || split_len <= 0 || split_len % FD_CHUNK)
        return set_error(VSL_ERR_INVALID, "flash_decode: page_size (%d) and split_len (%d) must be multiples of %d",
                         page_size, split_len, FD_CHUNK);
    if (max_len <= 0 || max_len > max_pages * page_size)
        return set_error(VSL_ERR_INVALID, "flash_decode: max_len %d outside the page table", max_len);
    // split_len is the least positions per split; the grid has n_splits_max splits per (sequence,
    // group), or enough to cover max_len with split_len each (then every split is split_len long)
    const int n_splits = n_splits_max > 0 ? n_splits_max : fd_splits(max_len, split_len);
    const size_t need = fd_workspace(B, n_heads, n_kv, head_dim, n_splits);
    if (workspace_bytes < need)
        return set_error(VSL_ERR_INVALID, "flash_decode: workspace %zu bytes < %zu", workspace_bytes, need);
    FdParams p = {};
    p.q = q; p.k_cache = k_cache; p.v_cache = v_cache; p.page_table = page_table; p.max_pages = max_pages;
    p.page_size = page_size; p.pos = pos; p.B = B; p.n_heads = n_heads; p.n_kv = n_kv; p.split_min = split_len;
    p.n_splits = n_splits; p.max_len = max_len; p.scale = 1.0f / sqrtf((float)head_dim); p.out = out;
    char* w = reinterpret_cast<char*>(workspace);
    p.ws_o = reinterpret_cast<float*>(w);
    w += align256((size_t)B * n_heads * n_splits * head_dim * sizeof(float));
    p.ws_ml = reinterpret_cast<float*>(w);
    p.counters = reinterpret_cast<int*>(static_cast<char*>(workspace) + fd_counters_offset(B, n_kv, workspace_bytes));
    p.pf_ptr = pf_ptr;
    p.pf_bytes = pf_bytes;
    p.wait_first = shared_pages ? 1 : 0;
    p.status = status;
    if (sparse) p.sp = *sparse;
    if (kvdtype == VSL_F16) {
        if (head_dim == 128) return launch_fd<128, __half>(p, stream);
        if (head_dim == 64) return launch_fd<64, __half>(p, stream);
    } else if (kvdtype == VSL_F32) {
        if (head_dim == 128) return launch_fd<128, float>(p, stream);
        if (head_dim == 64) return launch_fd<64, float>(p, stream);
    }
    return set_error(VSL_ERR_UNSUPPORTED, "flash_decode: head_dim %d / kv dtype %d", head_dim, kvdtype);
}

}  // namespace vsl

extern "C" int vsl_flash_decode_workspace_size(int B, int n_heads, int n_kv, int head_dim, int max_len,
                                               int split_len, size_t* bytes) {
    if (!bytes || B <= 0 || n_heads <= 0 || n_kv <= 0 || head_dim <= 0 || max_len <= 0 || split_len <= 0)
        return vsl::set_error(VSL_ERR_INVALID, "flash_decode_workspace_size: bad arguments");
    *bytes = vsl::fd_workspace(B, n_heads, n_kv, head_dim, vsl::fd_splits(max_len, split_len));
    return VSL_OK;
}

extern "C" int vsl_flash_decode(const float* q, const void* k_cache, const void* v_cache, int kvdtype,
                                const int32_t* page_table, int max_pages, int page_size, const int32_t* pos, int B,
                                int n_heads, int n_kv, int head_dim, int max_len, int split_len, float* out,
                                void* workspace, size_t workspace_bytes, void* stream) {
    return vsl::flash_decode_impl(q, k_cache, v_cache, kvdtype, page_table, max_pages, page_size, pos, B, n_heads,
                                  n_kv, head_dim, max_len, split_len, out, workspace, workspace_bytes,
                                  (cudaStream_t)stream, nullptr, 0, true, nullptr, 0, nullptr);  // the caller's rows may share pages
}

extern "C" int vsl_flash_decode_short(const float* q, const void* k_cache, const void* v_cache, int kvdtype,
                                      const int32_t* page_table, int max_pages, int page_size, const int32_t* pos,
                                      int B, int n_heads, int n_kv, int head_dim, int max_len, float* out,
                                      const vsl_sparse_mask* mask, int* status, void* stream) {
    vsl::SparseMask m = {};
    if (mask && mask->min_len > 0) m = vsl::SparseMask{mask->min_len, mask->window, mask->global_tokens, mask->block};
    return vsl::flash_decode_short_impl(q, k_cache, v_cache, kvdtype, page_table, max_pages, page_size, pos, B,
                                        n_heads, n_kv, head_dim, max_len, out, (cudaStream_t)stream, nullptr, 0, &m,
                                        status);
}

extern "C" int vsl_flash_decode_sparse(const float* q, const void* k_cache, const void* v_cache, int kvdtype,
                                       const int32_t* page_table, int max_pages, int page_size, const int32_t* pos,
                                       int B, int n_heads, int n_kv, int head_dim, int max_len, int split_len,
                                       float* out, void* workspace, size_t workspace_bytes,
                                       const vsl_sparse_mask* mask, void* stream) {
    vsl::SparseMask m = {};
    if (mask && mask->min_len > 0) m = vsl::SparseMask{mask->min_len, mask->window, mask->global_tokens, mask->block};
    return vsl::flash_decode_impl(q, k_cache, v_cache, kvdtype, page_table, max_pages, page_size, pos, B, n_heads,
                                  n_kv, head_dim, max_len, split_len, out, workspace, workspace_bytes,
                                  (cudaStream_t)stream, nullptr, 0, true, &m, 0, nullptr);
}

// ---------------------------------------------------------------------------------------
// Allocation-free variant.
//
// Some callers cannot let a library call cudaMalloc: hosts whose device memory is owned by
// their own pool or budget (every byte must come from them or be fixed up front), and
// latency-critical loops that cannot afford an allocation's implicit device
// synchronisation or its failure modes mid-run. vsl_flash_decode_noalloc gives them the
// split-K attention without a workspace argument: its scratch is this file-scope device
// array, which exists once per GPU that loads the library and lives until the process exits.
// ---------------------------------------------------------------------------------------
static constexpr size_t FD_STATIC_SCRATCH_BYTES = 4u << 20;  // 4 MiB
static __device__ __align__(256) unsigned char g_fd_static_scratch[FD_STATIC_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_fd_scratch_mu;
void* g_fd_scratch_addr[kMaxDevices] = {};

// Device address of the static scratch on the current device. In host code the array's
// name is only a host-side stand-in, so the address is looked up once per device with that
// device current, and cached for the life of the process (a cudaDeviceReset of that device
// would leave the cached address pointing into the ended context).
int fd_static_scratch(void** out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return vsl::launch_status(e, "flash_decode_noalloc: cudaGetDevice");
    if (dev < 0 || dev >= kMaxDevices)
        return vsl::set_error(VSL_ERR_UNSUPPORTED, "flash_decode_noalloc: device ordinal %d", dev);
    std::lock_guard<std::mutex> lock(g_fd_scratch_mu);
    if (!g_fd_scratch_addr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_fd_static_scratch);
        if (e != cudaSuccess || !p)
            return vsl::set_error(VSL_ERR_CUDA, "flash_decode_noalloc: cudaGetSymbolAddress failed: %s",
                                  cudaGetErrorString(e));
        g_fd_scratch_addr[dev] = p;
    }
    *out = g_fd_scratch_addr[dev];
    return VSL_OK;
}
}  // namespace

extern "C" int vsl_flash_decode_noalloc(const float* q, const void* k_cache, const void* v_cache, int kvdtype,
                                        const int32_t* page_table, int max_pages, int page_size, const int32_t* pos,
                                        int B, int n_heads, int n_kv, int head_dim, int max_len, int split_len,
                                        float* out, void* stream) {
    if (B <= 0 || n_heads <= 0 || n_kv <= 0 || head_dim <= 0 || max_len <= 0 || split_len <= 0)
        return vsl::set_error(VSL_ERR_INVALID, "flash_decode_noalloc: bad arguments");
    const int n_splits = vsl::fd_splits(max_len, split_len);
    const size_t need = vsl::fd_workspace(B, n_heads, n_kv, head_dim, n_splits);
    if (need > FD_STATIC_SCRATCH_BYTES)
        return vsl::set_error(VSL_ERR_UNSUPPORTED,
                              "flash_decode_noalloc: this shape needs %zu bytes of scratch but the static scratch "
                              "holds %zu; use vsl_flash_decode with a caller-owned workspace",
                              need, FD_STATIC_SCRATCH_BYTES);
    void* ws = nullptr;
    int rc = fd_static_scratch(&ws);
    if (rc) return rc;
    // The array keeps whatever the previous call left; the split counters must start at zero.
    const size_t counters_off = vsl::fd_counters_offset(B, n_kv, FD_STATIC_SCRATCH_BYTES);
    cudaError_t e = cudaMemsetAsync(static_cast<unsigned char*>(ws) + counters_off, 0, (size_t)B * n_kv * sizeof(int),
                                    (cudaStream_t)stream);
    if (e != cudaSuccess) return vsl::launch_status(e, "flash_decode_noalloc: clearing the split counters");
    return vsl::flash_decode_impl(q, k_cache, v_cache, kvdtype, page_table, max_pages, page_size, pos, B, n_heads,
                                  n_kv, head_dim, max_len, split_len, out, ws, FD_STATIC_SCRATCH_BYTES,
                                  (cudaStream_t)stream, nullptr, 0, true, nullptr, 0, nullptr);  // the caller's rows may share pages
}
