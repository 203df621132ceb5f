// Long-context decode attention on tcgen05 tensor cores.
//
// Same semantics as vsl_flash_decode_kernel (attention.cu; reference attention.comp:84-189): query
// head h reads KV group h*n_kv/n_heads, scores q.k / sqrt(head_dim), max-subtracted softmax over
// positions [0, pos], output = probabilities times V. Built for caches of thousands of positions
// (fp16 KV, head_dim 128, up to 8 query heads per KV group). Per 128-position chunk:
//   * S^T[128 positions][16] = K[128][128] . Q2[16][128]^T (tcgen05.mma kind::f16, M = 128,
//     N = 16, fp32 in TMEM). Q2 holds the group's query heads as hi/lo fp16 pairs (rows 0..G-1
//     hi, 8..8+G-1 lo, the rest zero), so scores keep ~22 bits of the fp32 query. Positions sit
//     on M because tcgen05 needs M >= 64 and a group has only 4-8 query heads.
//   * online softmax (fp32) by 4 warps, one position per thread (tcgen05.ld of its TMEM row);
//     the probabilities go back to shared memory as hi/lo fp16 rows P2[16][128].
//   * O^T[128 dims][16] = V^T . P2^T on the tensor cores, with the V tile used in place as the
//     MN-major A operand (the TMA layout: positions as rows of 64 dims); a thread (= head dim)
//     folds O into its accumulators one chunk later, so the next chunk's scores and softmax
//     overlap this product.
//   * K and V chunks (two 64-position pages each, 2 x 64-column 128-byte-swizzle atoms) arrive by
//     tensor TMA into a 3-stage ring (192 KB per SM) with separate barriers for the K and the V
//     half of a stage, each filled by its own producer thread: a K half is refilled as soon as its
//     scores are computed, before the softmax and the product of its chunk; rows past the end of
//     a sequence are zeroed in shared memory before the product reads them (0 x garbage).
//   * work split (stream-K): the flattened list of (sequence, KV group, 128-position chunk) is cut
//     into equal ranges over persistent CTAs, whatever the per-sequence lengths; a (sequence,
//     group) shared by several CTAs is merged by the last to finish, in CTA order
//     (deterministic), with an atomic counter it resets to zero.
// Roles: warps 0-3 softmax and accumulation (TMEM lane quarter = warp), warp 4 TMA producers,
// warp 5 TMEM allocation and the single-thread MMA issue. Every wait is bounded (one second) and
// records VSL_ERR_TIMEOUT; the kernel then drains its copies and MMAs and frees its TMEM.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <math_constants.h>

#include <mutex>

#include "common.cuh"
#include "kv_map.h"
#include "launch.cuh"
#include "trace.cuh"

VSL_TRACE_UNIT(attention_tc)

namespace vsl {

constexpr int FT_THREADS = 192;  // 4 softmax warps, TMA producer, MMA issuer
constexpr int FT_CHUNK = 128;                 // positions per chunk (MMA M)
constexpr int FT_HD = 128;
constexpr int FT_GMAX = 8;
constexpr int FT_N = 16;                      // MMA N: 8 hi + 8 lo query rows
constexpr int FT_STAGES = 3;
constexpr int FT_ATOM = 128 * 64 * 2;         // one 64-column swizzle atom of a 128-row tile (16 KB)
constexpr int FT_STAGE = 4 * FT_ATOM;         // K (2 atoms) + V (2 atoms) = 64 KB
constexpr int FT_Q2 = 2 * FT_N * 128;         // 2 atoms of 16 rows x 128 bytes
constexpr int FT_BMAX = 64;
constexpr int FT_P2 = 2 * FT_N * 128;         // P as hi/lo fp16 rows: 2 atoms of 16 rows x 128 bytes
constexpr size_t FT_SMEM = 1024 + (size_t)FT_STAGES * FT_STAGE + FT_Q2 + 2 * (size_t)FT_P2;

struct FtArgs {
    const float* q;          // [B][n_heads][128]
    const int32_t* pos;
    const int32_t* page_table;
    int B, n_heads, n_kv, G, max_len, max_pages, page_size;
    float scale;
    float* out;              // [B][n_heads][128]
    float* ws_o;             // [grid][2][8][128]
    float* ws_ml;            // [grid][2][8][2]
    int* counters;           // [B][n_kv], zero between launches
    int* status;
    uint32_t idesc;     // S MMA: K (A, K-major) . Q2 (B, K-major)
    uint32_t idesc_pv;  // PV MMA: V (A, MN-major) . P2 (B, K-major)
    SparseMask sp;      // long-context sparse mask (sp.min_len 0: dense)
    unsigned trace_id;  // launch id of the trace build (unused otherwise)
};

__device__ __forceinline__ void ft_tma(uint32_t dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void ft_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void ft_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// K-major 128-byte-swizzle operand descriptor (8-row x 128-byte atoms, 1024 bytes apart)
__device__ __forceinline__ uint64_t ft_desc(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
__device__ __forceinline__ int ft_abort(const int* p) { return *reinterpret_cast<const volatile int*>(p); }
// MN-major 128-byte-swizzle operand (the V tile as it lands from TMA: rows = positions = K,
// 64 head dims = M per 128-byte row): atoms of 64 M x 8 K; the next 64 dims sit one 16 KB atom
// further (leading byte offset), the next 8 positions 1024 bytes further (stride byte offset)
__device__ __forceinline__ uint64_t ft_desc_mn(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)(FT_ATOM >> 4) << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
__device__ __forceinline__ void ft_mma(uint32_t d, uint64_t ad, uint64_t bd, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
        "l"(ad), "l"(bd), "r"(idesc), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void ft_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void ft_ld16(uint32_t taddr, uint32_t* r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Flattened work list: for sequence b, n_kv groups x nch[b] chunks, starting at off[b]; chunk ch
// of sequence b covers positions (c0[b] + ch) * 128 onward, of which those below lo[b] are masked
// (the sparse mask's start; c0 = lo = 0 when dense).
struct FtWork {
    int nch[FT_BMAX], len[FT_BMAX], c0[FT_BMAX], lo[FT_BMAX];
    long long off[FT_BMAX + 1];
};

__device__ __forceinline__ long long ft_lo(long long T, int G, int c) { return T * c / G; }
__device__ __forceinline__ int ft_owner(long long T, int G, long long f) { return (int)(((f + 1) * G - 1) / T); }

// cursor over this CTA's chunks: (b, g, ch) of flat index f
struct FtCur {
    long long f;
    int b, g, ch;
};
__device__ __forceinline__ void ft_seek(const FtWork& w, int B, int n_kv, long long f, FtCur& c) {
    c.f = f;
    int b = 0;
    while (b + 1 < B && w.off[b + 1] <= f) b++;
    const long long r = f - w.off[b];
    c.b = b;
    c.g = (int)(r / w.nch[b]);
    c.ch = (int)(r - (long long)c.g * w.nch[b]);
}
__device__ __forceinline__ void ft_next(const FtWork& w, int n_kv, FtCur& c) {
    c.f++;
    if (++c.ch < w.nch[c.b]) return;
    c.ch = 0;
    if (++c.g < n_kv) return;
    c.g = 0;
    c.b++;
}

__global__ void __launch_bounds__(FT_THREADS, 1)
    vsl_flash_decode_tc_kernel(const __grid_constant__ CUtensorMap map_k, const __grid_constant__ CUtensorMap map_v,
                           const __grid_constant__ FtArgs a) {
    VSL_TRACE_ENTRY();
    extern __shared__ unsigned char smem_raw[];
    // K and V halves of a stage have their own barriers: the K half is refilled once the chunk's
    // scores are computed, the V half once its product is
    __shared__ __align__(8) uint64_t full_k[FT_STAGES], full_v[FT_STAGES], empty_k[FT_STAGES], empty_v[FT_STAGES];
    __shared__ __align__(8) uint64_t s_full[2], s_free[2], q_ready;
    __shared__ __align__(8) uint64_t p_ready[2], o_full[2], o_free[2];
    __shared__ uint32_t tmem_s;
    __shared__ int abort_s, last_s;
    __shared__ float red_max[2][4][FT_GMAX], red_sum[4][FT_GMAX];
    __shared__ FtWork wk;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
    const uint32_t ring = base;
    const uint32_t q2 = base + FT_STAGES * FT_STAGE;
    const uint32_t p2 = q2 + FT_Q2;  // two P2 tiles [16 rows][128 positions], K-major, 128-byte swizzle
    const int c = blockIdx.x;

    if (threadIdx.x == 0) {
        for (int s = 0; s < FT_STAGES; s++) {
            mbar_init(&full_k[s], 1);
            mbar_init(&full_v[s], 1);
            mbar_init(&empty_k[s], 1);  // tcgen05.commit after the chunk's scores
            mbar_init(&empty_v[s], 1);  // tcgen05.commit after the chunk's P.V
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&s_full[i], 1);
            mbar_init(&s_free[i], 4);
            mbar_init(&p_ready[i], 4);
            mbar_init(&o_full[i], 1);
            mbar_init(&o_free[i], 4);
        }
        mbar_init(&q_ready, 4);
        mbar_fence_init();
        abort_s = 0;
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_k)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_v)) : "memory");
    }
    if (warp == 5) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_s)), "r"(64)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    pdl_wait();
    VSL_TRACE_RELEASED();
    pdl_launch_dependents();
    if (warp == 0) {  // work list from the current positions
        for (int b = lane; b < a.B; b += 32) {
            int len = __ldcg(a.pos + b) + 1;
            len = len < 1 ? 1 : (len > a.max_len ? a.max_len : len);
            const int lo = sparse_first(a.sp, len - 1);
            wk.len[b] = len;
            wk.lo[b] = lo;
            wk.c0[b] = lo / FT_CHUNK;
            wk.nch[b] = (len + FT_CHUNK - 1) / FT_CHUNK - lo / FT_CHUNK;
        }
        __syncwarp();
        if (lane == 0) {
            long long o = 0;
            for (int b = 0; b < a.B; b++) {
                wk.off[b] = o;
                o += (long long)a.n_kv * wk.nch[b];
            }
            wk.off[a.B] = o;
        }
    }
    ft_fence_before();
    __syncthreads();
    ft_fence_after();
    const uint32_t tmem = tmem_s;
    const long long T = wk.off[a.B];
    // the work is cut over min(gridDim.x, T) CTAs so that every participating CTA owns at least
    // one chunk (the merge counts on each owner of a shared (sequence, group) arriving)
    const int Gc = (long long)gridDim.x < T ? (int)gridDim.x : (int)T;
    const long long f0 = c < Gc ? ft_lo(T, Gc, c) : 0, f1 = c < Gc ? ft_lo(T, Gc, c + 1) : 0;

    if (warp == 4) {
        // ================= TMA producers: lane 0 the K halves, lane 1 the V halves =================
        if (lane < 2) {
            const bool kside = lane == 0;
            uint64_t* fullx = kside ? full_k : full_v;
            uint64_t* emptyx = kside ? empty_k : empty_v;
            const CUtensorMap* map = kside ? &map_k : &map_v;
            const uint32_t half = kside ? 0u : (uint32_t)(2 * FT_ATOM);
            FtCur cu;
            if (f0 < f1) ft_seek(wk, a.B, a.n_kv, f0, cu);
            int s = 0;
            uint32_t epar = 1u;
            long long it = 0;
            bool ok = true;
            for (long long f = f0; f < f1 && ok; f++, it++) {
                if (it >= FT_STAGES && !mbar_wait(&emptyx[s], epar)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(&fullx[s], FT_STAGE / 2);
                const uint32_t st = ring + s * FT_STAGE + half;
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    int p0 = (wk.c0[cu.b] + cu.ch) * FT_CHUNK + h * 64;
                    if (p0 >= wk.len[cu.b]) p0 = 0;  // past the end: any valid page (masked later)
                    const int page = __ldg(a.page_table + (size_t)cu.b * a.max_pages + p0 / a.page_size);
                    const int row = (page * a.n_kv + cu.g) * a.page_size + (p0 % a.page_size);
#pragma unroll
                    for (int at = 0; at < 2; at++)
                        ft_tma(st + at * FT_ATOM + h * (FT_ATOM / 2), map, at * 64, row, &fullx[s]);
                }
                ft_next(wk, a.n_kv, cu);
                if (++s == FT_STAGES) {
                    s = 0;
                    epar ^= 1u;
                }
            }
            if (!ok) {
                set_status(a.status, VSL_ERR_TIMEOUT);
                atomicExch(&abort_s, 1);
            }
            const long long issued = it;
            for (long long u = issued > FT_STAGES ? issued - FT_STAGES : 0; u < issued; u++)
                mbar_wait(&fullx[u % FT_STAGES], (uint32_t)((u / FT_STAGES) & 1));
        }
    } else if (warp == 5) {
        // ================= MMA issue =================
        // per chunk i: S(i) = K . Q2^T into TMEM S[i&1]; PV(i) = V^T . P2(i)^T into TMEM O[i&1]
        // once the softmax warps have written P2(i). S(i+1) is issued before PV(i) when chunk i+1
        // belongs to the same (sequence, group), so scores and products overlap the softmax.
        if (lane == 0) {
            FtCur cs;  // cursor of the next S to issue
            if (f0 < f1) ft_seek(wk, a.B, a.n_kv, f0, cs);
            const long long n = f1 - f0;
            int ss = 0;           // stage of the next S
            uint32_t fpar = 0u;   // its full-barrier parity
            int seg = 0;
            int pb = -1, pg = -1;
            bool ok = true;
            long long s_issued = 0;
            int st_of[2] = {0, 0};      // stage of chunk i (kept for PV(i) and the stage release)
            uint32_t par_of[2] = {0u, 0u};  // and the parity of that use of the stage
            int segpos[2] = {0, 0};     // (b * n_kv + g) of chunk i
            auto issue_s = [&](long long i) -> bool {
                const int key = cs.b * a.n_kv + cs.g;
                if (cs.b != pb || cs.g != pg) {  // new (sequence, group): its query rows must be staged
                    if (!mbar_wait(&q_ready, (uint32_t)(seg & 1))) return false;
                    seg++;
                    pb = cs.b;
                    pg = cs.g;
                }
                if (!mbar_wait(&full_k[ss], fpar)) return false;
                if (i >= 2 && !mbar_wait(&s_free[i & 1], (uint32_t)(((i >> 1) - 1) & 1))) return false;
                ft_fence_after();
                const uint32_t st = ring + ss * FT_STAGE;
#pragma unroll
                for (int at = 0; at < 2; at++) {
                    const uint64_t ad = ft_desc(st + at * FT_ATOM), bd = ft_desc(q2 + at * (FT_Q2 / 2));
#pragma unroll
                    for (int k = 0; k < 4; k++)
                        ft_mma(tmem + (uint32_t)((i & 1) * FT_N), ad + (uint64_t)(2 * k), bd + (uint64_t)(2 * k),
                               a.idesc, (at > 0 || k > 0) ? 1u : 0u);
                }
                ft_commit(&s_full[i & 1]);
                ft_commit(&empty_k[ss]);  // the K half of this stage is no longer read
                st_of[i & 1] = ss;
                par_of[i & 1] = fpar;
                segpos[i & 1] = key;
                if (++ss == FT_STAGES) {
                    ss = 0;
                    fpar ^= 1u;
                }
                ft_next(wk, a.n_kv, cs);
                return true;
            };
            auto issue_pv = [&](long long i) -> bool {
                if (!mbar_wait(&p_ready[i & 1], (uint32_t)((i >> 1) & 1))) return false;
                if (i >= 2 && !mbar_wait(&o_free[i & 1], (uint32_t)(((i >> 1) - 1) & 1))) return false;
                if (!mbar_wait(&full_v[st_of[i & 1]], par_of[i & 1])) return false;
                ft_fence_after();
                const uint32_t vt = ring + st_of[i & 1] * FT_STAGE + 2 * FT_ATOM;
                const uint32_t pt = p2 + (uint32_t)(i & 1) * FT_P2;
#pragma unroll
                for (int k = 0; k < FT_CHUNK / 16; k++) {
                    // V as the MN-major A operand: 16 positions (rows) per step = 2048 bytes
                    const uint64_t ad = ft_desc_mn(vt + (uint32_t)(k * 2048));
                    const uint64_t bd = ft_desc(pt + (uint32_t)((k >> 2) * (FT_P2 / 2))) + (uint64_t)(2 * (k & 3));
                    ft_mma(tmem + (uint32_t)(2 * FT_N + (i & 1) * FT_N), ad, bd, a.idesc_pv, k > 0 ? 1u : 0u);
                }
                ft_commit(&o_full[i & 1]);
                ft_commit(&empty_v[st_of[i & 1]]);  // the V half of this stage is no longer read
                return true;
            };
            if (n > 0) ok = issue_s(0);
            s_issued = ok ? 1 : 0;
            for (long long i = 0; i < n && ok; i++) {
                if (ft_abort(&abort_s)) {
                    ok = false;
                    break;
                }
                // look ahead one S only inside the same (sequence, group): a new one needs the
                // softmax warps to have finished this one first (they stage its query rows)
                if (s_issued == i + 1 && i + 1 < n && cs.b * a.n_kv + cs.g == segpos[i & 1]) {
                    ok = issue_s(i + 1);
                    if (!ok) break;
                    s_issued++;
                }
                ok = issue_pv(i);
                if (!ok) break;
                if (s_issued == i + 1 && i + 1 < n) {
                    ok = issue_s(i + 1);
                    if (!ok) break;
                    s_issued++;
                }
            }
            if (!ok) {
                set_status(a.status, VSL_ERR_TIMEOUT);
                atomicExch(&abort_s, 1);
            }
            // the accumulators must not be freed under a running MMA
            if (n > 0) {
                const long long last = (s_issued > 0 ? s_issued : 1) - 1;
                mbar_wait(&s_full[last & 1], (uint32_t)((last >> 1) & 1));
                mbar_wait(&o_full[last & 1], (uint32_t)((last >> 1) & 1));
            }
        }
        __syncwarp();
    } else {
        // ================= softmax + accumulation (warps 0-3; thread t = position t, dim t) =================
        const int t = threadIdx.x;
        const int G = a.G;
        float m[FT_GMAX], lt[FT_GMAX], o[FT_GMAX], alpha_prev[FT_GMAX];
        unsigned char* smem_g = smem_raw - smem_u32(smem_raw);  // generic pointer of shared address 0
        // P2 rows beyond the group's heads stay zero in both buffers
        for (int i = t; i < 2 * FT_P2 / 16; i += 128)
            *reinterpret_cast<uint4*>(smem_g + p2 + i * 16) = make_uint4(0, 0, 0, 0);
        FtCur cu;
        if (f0 < f1) ft_seek(wk, a.B, a.n_kv, f0, cu);
        long long i = 0;
        int pb = -1, pg = -1;
        int sst = 0;
        uint32_t fpar = 0u;
        // A failed wait (or another role's abort) is carried to the next barrier, a bar.red.or that
        // all four warps take, so they leave the loop together with one barrier per chunk; what
        // runs in between on a failed wait reads stale shared or tensor memory and is discarded.
        bool bad = false;
        for (long long f = f0; f < f1; f++, i++) {
            const int b = cu.b, g = cu.g, ch = cu.ch;
            const int len = wk.len[b];
            const bool seg_start = b != pb || g != pg;
            if (seg_start) {
                // ---- new (sequence, group): reset the softmax state, stage Q2 for the tensor cores ----
#pragma unroll
                for (int j = 0; j < FT_GMAX; j++) {
                    m[j] = -CUDART_INF_F;
                    lt[j] = 0.0f;
                    o[j] = 0.0f;
                    alpha_prev[j] = 1.0f;
                }
                const int r = t >> 4, at = (t >> 3) & 1, cc = t & 7;  // query row r, atom, 16-byte chunk
                uint4 hv = make_uint4(0, 0, 0, 0), lv = make_uint4(0, 0, 0, 0);
                if (r < G) {
                    const float* qr = a.q + ((size_t)b * a.n_heads + (size_t)g * G + r) * FT_HD + at * 64 + cc * 8;
                    const float4 x0 = __ldcg(reinterpret_cast<const float4*>(qr));
                    const float4 x1 = __ldcg(reinterpret_cast<const float4*>(qr) + 1);
                    const float xs[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
                    __half hh[8], ll[8];
#pragma unroll
                    for (int e = 0; e < 8; e++) {
                        hh[e] = __float2half_rn(xs[e]);
                        ll[e] = __float2half_rn(xs[e] - __half2float(hh[e]));
                    }
                    hv = *reinterpret_cast<const uint4*>(hh);
                    lv = *reinterpret_cast<const uint4*>(ll);
                }
                unsigned char* q2p = smem_g + q2 + at * (FT_Q2 / 2);
                *reinterpret_cast<uint4*>(q2p + r * 128 + ((cc ^ (r & 7)) << 4)) = hv;
                *reinterpret_cast<uint4*>(q2p + (r + 8) * 128 + ((cc ^ ((r + 8) & 7)) << 4)) = lv;
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // visible to the tensor cores
                __syncwarp();
                if (lane == 0) mbar_arrive(&q_ready);
                pb = b;
                pg = g;
            }
            // ---- scores of chunk i (TMEM row t) ----
            bad = bad || !mbar_wait(&s_full[i & 1], (uint32_t)((i >> 1) & 1)) || ft_abort(&abort_s);
            ft_fence_after();
            uint32_t r[16];
            ft_ld16(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)((i & 1) * FT_N), r);
            ft_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s_free[i & 1]);
            const int base = (wk.c0[b] + ch) * FT_CHUNK;  // position of TMEM row 0
            const int n_valid = min(FT_CHUNK, len - base);
            const bool past_end = t >= n_valid;
            const bool valid = !past_end && base + t >= wk.lo[b];
            float sc[FT_GMAX];
#pragma unroll
            for (int j = 0; j < FT_GMAX; j++) {
                sc[j] = (j < G && valid) ? (__uint_as_float(r[j]) + __uint_as_float(r[8 + j])) * a.scale : -CUDART_INF_F;
                if (j < G) {
                    const float mx = warp_max_redux(sc[j]);
                    if (lane == 0) red_max[i & 1][warp][j] = mx;  // two buffers: a warp may be a chunk ahead
                }
            }
            if (named_barrier_or(1, 128, bad)) {  // the four warps leave together
                set_status(a.status, VSL_ERR_TIMEOUT);
                atomicExch(&abort_s, 1);
                break;
            }
            float alpha[FT_GMAX];
            const int pc = t >> 6, pcol = t & 63;  // P2 atom and column of position t
            unsigned char* p2p = smem_g + p2 + (uint32_t)(i & 1) * FT_P2 + pc * (FT_P2 / 2) + ((pcol & 7) << 1);
#pragma unroll
            for (int j = 0; j < FT_GMAX; j++) {
                if (j >= G) break;
                const float(&rm)[4][FT_GMAX] = red_max[i & 1];
                const float cm = fmaxf(fmaxf(rm[0][j], rm[1][j]), fmaxf(rm[2][j], rm[3][j]));
                const float mn = fmaxf(m[j], cm);
                // __expf: arguments are <= 0 here, where its error stays a few ulp of the fp32 result
                alpha[j] = __expf(m[j] - mn);
                const float pj = valid ? __expf(sc[j] - mn) : 0.0f;
                m[j] = mn;
                lt[j] = lt[j] * alpha[j] + pj;
                const __half ph = __float2half_rn(pj);
                const __half pl = __float2half_rn(pj - __half2float(ph));
                const int rh = j, rl = j + 8;
                *reinterpret_cast<__half*>(p2p + rh * 128 + ((((pcol >> 3) ^ (rh & 7))) << 4)) = ph;
                *reinterpret_cast<__half*>(p2p + rl * 128 + ((((pcol >> 3) ^ (rl & 7))) << 4)) = pl;
            }
            if (n_valid < FT_CHUNK && past_end) {
                // rows past the sequence end hold whatever the cache had (possibly NaN bit patterns):
                // zero them so that 0 x garbage cannot reach the product
                mbar_wait(&full_v[sst], fpar);  // order after the TMA's writes to this stage
                unsigned char* vrow = smem_g + ring + sst * FT_STAGE + 2 * FT_ATOM + t * 128;
#pragma unroll
                for (int at2 = 0; at2 < 2; at2++)
#pragma unroll
                    for (int c16 = 0; c16 < 8; c16++)
                        *reinterpret_cast<uint4*>(vrow + at2 * FT_ATOM + c16 * 16) = make_uint4(0, 0, 0, 0);
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_ready[i & 1]);
            if (++sst == FT_STAGES) {
                sst = 0;
                fpar ^= 1u;
            }
            // ---- fold PV(i-1) into the output (lagged one chunk: PV(i) overlaps the next softmax) ----
            ft_next(wk, a.n_kv, cu);
            const bool seg_end = f + 1 == f1 || cu.b != b || cu.g != g;
            auto fold = [&](long long k, const float* al) {
                bad = bad || !mbar_wait(&o_full[k & 1], (uint32_t)((k >> 1) & 1)) || ft_abort(&abort_s);
                ft_fence_after();
                uint32_t ov[16];
                ft_ld16(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(2 * FT_N + (k & 1) * FT_N), ov);
                ft_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&o_free[k & 1]);
#pragma unroll
                for (int j = 0; j < FT_GMAX; j++)
                    if (j < G) o[j] = o[j] * al[j] + (__uint_as_float(ov[j]) + __uint_as_float(ov[8 + j]));
            };
            if (!seg_start) fold(i - 1, alpha_prev);
            if (seg_end) fold(i, alpha);
#pragma unroll
            for (int j = 0; j < FT_GMAX; j++) alpha_prev[j] = alpha[j];
            if (!seg_end) continue;
            // ---- end of this CTA's part of (b, g): softmax denominators over the 128 positions ----
#pragma unroll
            for (int j = 0; j < FT_GMAX; j++) {
                if (j >= G) break;
                const float sm = warp_sum(lt[j]);
                if (lane == 0) red_sum[warp][j] = sm;
            }
            if (named_barrier_or(1, 128, bad)) {
                set_status(a.status, VSL_ERR_TIMEOUT);
                atomicExch(&abort_s, 1);
                break;
            }
            float l[FT_GMAX];
#pragma unroll
            for (int j = 0; j < FT_GMAX; j++)
                l[j] = j < G ? (red_sum[0][j] + red_sum[1][j]) + (red_sum[2][j] + red_sum[3][j]) : 1.0f;
            const long long p0 = wk.off[b] + (long long)g * wk.nch[b];
            const int first = ft_owner(T, Gc, p0), lastc = ft_owner(T, Gc, p0 + wk.nch[b] - 1);
            float* out = a.out + ((size_t)b * a.n_heads + (size_t)g * G) * FT_HD + t;
            if (first == lastc) {
#pragma unroll
                for (int j = 0; j < FT_GMAX; j++)
                    if (j < G) out[(size_t)j * FT_HD] = o[j] / l[j];
                named_barrier_sync(1, 128);  // red_sum is reused by the next segment
                continue;
            }
            const int slot = ft_lo(T, Gc, c) >= p0 ? 0 : 1;
            float* wo = a.ws_o + (((size_t)c * 2 + slot) * FT_GMAX) * FT_HD + t;
#pragma unroll
            for (int j = 0; j < FT_GMAX; j++)
                if (j < G) wo[(size_t)j * FT_HD] = o[j];
            if (t < G) {
                float* wml = a.ws_ml + (((size_t)c * 2 + slot) * FT_GMAX + t) * 2;
                float mt = m[0], ltt = l[0];
#pragma unroll
                for (int j = 1; j < FT_GMAX; j++)
                    if (j == t) {
                        mt = m[j];
                        ltt = l[j];
                    }
                wml[0] = mt;
                wml[1] = ltt;
            }
            __threadfence();
            named_barrier_sync(1, 128);
            if (t == 0) last_s = atomicAdd(a.counters + (size_t)b * a.n_kv + g, 1) == lastc - first;
            named_barrier_sync(1, 128);
            if (last_s) {
                __threadfence();
#pragma unroll
                for (int j = 0; j < FT_GMAX; j++) {
                    if (j >= G) break;
                    float M = -CUDART_INF_F;
                    for (int cc2 = first; cc2 <= lastc; cc2++) {
                        const int sl = ft_lo(T, Gc, cc2) >= p0 ? 0 : 1;
                        M = fmaxf(M, __ldcg(a.ws_ml + (((size_t)cc2 * 2 + sl) * FT_GMAX + j) * 2));
                    }
                    float L = 0.0f, O = 0.0f;
                    for (int cc2 = first; cc2 <= lastc; cc2++) {
                        const int sl = ft_lo(T, Gc, cc2) >= p0 ? 0 : 1;
                        const float* ml = a.ws_ml + (((size_t)cc2 * 2 + sl) * FT_GMAX + j) * 2;
                        const float w = expf(__ldcg(ml) - M);
                        L += __ldcg(ml + 1) * w;
                        O += __ldcg(a.ws_o + (((size_t)cc2 * 2 + sl) * FT_GMAX + j) * FT_HD + t) * w;
                    }
                    out[(size_t)j * FT_HD] = O / L;
                }
                if (t == 0) a.counters[(size_t)b * a.n_kv + g] = 0;
            }
            named_barrier_sync(1, 128);  // last_s and red_sum are reused by the next segment
        }
    }

    ft_fence_before();
    __syncthreads();
    if (warp == 5) {
        ft_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(64) : "memory");
    }
    VSL_TRACE_EXIT(a.trace_id, 907u);
}

// ---------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 ft_encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

int kv_tensor_map(CUtensorMap* m, const void* base, long long rows) {
    auto fn = ft_encode_fn();
    if (!fn) return set_error(VSL_ERR_CUDA, "tensor-map encoder unavailable from the driver");
    const cuuint64_t dims[2] = {(cuuint64_t)FT_HD, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)FT_HD * 2};
    const cuuint32_t box[2] = {64, 64};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(VSL_ERR_INVALID, "kv tensor map encode failed (%d)", (int)r);
    return VSL_OK;
}

size_t flash_decode_tc_workspace_bytes(int B, int n_kv) {
    const size_t G = (size_t)sm_count();
    return G * 2 * FT_GMAX * FT_HD * 4 + G * 2 * FT_GMAX * 2 * 4 + (size_t)B * n_kv * 4 + 512;
}

bool flash_decode_tc_supported(int kvdtype, int head_dim, int n_heads, int n_kv, int B, int page_size) {
    return kvdtype == VSL_F16 && head_dim == FT_HD && n_kv > 0 && n_heads % n_kv == 0 && n_heads / n_kv <= FT_GMAX &&
           B >= 1 && B <= FT_BMAX && page_size > 0 && page_size % 64 == 0;
}

int flash_decode_tc_impl(const float* q, const void* k_cache, const void* v_cache, int n_pages,
                         const int32_t* page_table, int max_pages, int page_size, const int32_t* pos, int B,
                         int n_heads, int n_kv, int max_len, float* out, void* workspace, size_t workspace_bytes,
                         int* status, cudaStream_t st, const SparseMask* sparse) {
    if (!flash_decode_tc_supported(VSL_F16, FT_HD, n_heads, n_kv, B, page_size))
        return set_error(VSL_ERR_UNSUPPORTED, "flash_decode_tc: heads %d/%d B %d page %d", n_heads, n_kv, B, page_size);
    if (!q || !k_cache || !v_cache || !page_table || !pos || !out || !workspace || max_len <= 0 ||
        max_len > max_pages * page_size || n_pages <= 0)
        return set_error(VSL_ERR_INVALID, "flash_decode_tc: null pointer, empty pool or max_len outside the page table");
    if (((uintptr_t)k_cache & 15) || ((uintptr_t)v_cache & 15) || ((uintptr_t)q & 15))
        return set_error(VSL_ERR_INVALID, "flash_decode_tc: caches and q must be 16-byte aligned");
    if (workspace_bytes < flash_decode_tc_workspace_bytes(B, n_kv))
        return set_error(VSL_ERR_INVALID, "flash_decode_tc: workspace of %zu bytes needed",
                         flash_decode_tc_workspace_bytes(B, n_kv));
    const int grid = sm_count();
    FtArgs a = {};
    a.q = q;
    a.pos = pos;
    a.page_table = page_table;
    a.B = B;
    a.n_heads = n_heads;
    a.n_kv = n_kv;
    a.G = n_heads / n_kv;
    a.max_len = max_len;
    a.max_pages = max_pages;
    a.page_size = page_size;
    a.scale = 1.0f / sqrtf((float)FT_HD);
    a.out = out;
    char* w = static_cast<char*>(workspace);
    a.ws_o = reinterpret_cast<float*>(w);
    w += (size_t)grid * 2 * FT_GMAX * FT_HD * 4;
    a.ws_ml = reinterpret_cast<float*>(w);
    w += (size_t)grid * 2 * FT_GMAX * 2 * 4;
    a.counters = reinterpret_cast<int*>(w);
    a.status = status;
    a.trace_id = VSL_TRACE_ID();
    if (sparse && sparse->min_len > 0) {
        if (sparse->window < 0 || sparse->global_tokens < 0 || sparse->block <= 0)
            return set_error(VSL_ERR_INVALID, "flash_decode_tc: sparse mask window %d, global %d, block %d",
                             sparse->window, sparse->global_tokens, sparse->block);
        a.sp = *sparse;
    }
    // instruction descriptor (kind::f16): D f32 (bits 4-5 = 1), A/B f16 (0), both K-major,
    // N >> 3 in bits 17-22, M >> 4 in bits 24-28
    a.idesc = (1u << 4) | ((uint32_t)(FT_N >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
    a.idesc_pv = a.idesc | (1u << 15);  // A (V) MN-major
    const long long rows = (long long)n_pages * n_kv * page_size;
    CUtensorMap mk, mv;
    int rc = kv_tensor_map(&mk, k_cache, rows);
    if (rc) return rc;
    rc = kv_tensor_map(&mv, v_cache, rows);
    if (rc) return rc;
    static thread_local int configured_dev = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (configured_dev != dev) {
        cudaError_t e = cudaFuncSetAttribute(vsl_flash_decode_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)FT_SMEM);
        if (e != cudaSuccess) return launch_status(e, "flash_decode_tc smem attribute");
        configured_dev = dev;
    }
    return launch_status(launch_k(vsl_flash_decode_tc_kernel, dim3(grid), dim3(FT_THREADS), FT_SMEM, st, mk, mv, a),
                         "flash_decode_tc launch");
}

}  // namespace vsl

using namespace vsl;

extern "C" int vsl_flash_decode_tc_workspace_size(int B, int n_kv, size_t* bytes) {
    if (!bytes || B <= 0 || B > FT_BMAX || n_kv <= 0)
        return set_error(VSL_ERR_INVALID, "flash_decode_tc_workspace_size: bad arguments");
    *bytes = flash_decode_tc_workspace_bytes(B, n_kv);
    return VSL_OK;
}

extern "C" int vsl_flash_decode_tc(const float* q, const void* k_cache, const void* v_cache, int n_pages,
                                   const int32_t* page_table, int max_pages, int page_size, const int32_t* pos, int B,
                                   int n_heads, int n_kv, int head_dim, int max_len, float* out, void* workspace,
                                   size_t workspace_bytes, void* stream) {
    if (head_dim != FT_HD) return set_error(VSL_ERR_UNSUPPORTED, "flash_decode_tc: head_dim %d (128 only)", head_dim);
    return flash_decode_tc_impl(q, k_cache, v_cache, n_pages, page_table, max_pages, page_size, pos, B, n_heads, n_kv,
                                max_len, out, workspace, workspace_bytes, nullptr, (cudaStream_t)stream, nullptr);
}

extern "C" int vsl_flash_decode_tc_sparse(const float* q, const void* k_cache, const void* v_cache, int n_pages,
                                          const int32_t* page_table, int max_pages, int page_size, const int32_t* pos,
                                          int B, int n_heads, int n_kv, int head_dim, int max_len, float* out,
                                          void* workspace, size_t workspace_bytes, const vsl_sparse_mask* mask,
                                          void* stream) {
    if (head_dim != FT_HD) return set_error(VSL_ERR_UNSUPPORTED, "flash_decode_tc: head_dim %d (128 only)", head_dim);
    SparseMask m = {};
    if (mask && mask->min_len > 0) m = SparseMask{mask->min_len, mask->window, mask->global_tokens, mask->block};
    return flash_decode_tc_impl(q, k_cache, v_cache, n_pages, page_table, max_pages, page_size, pos, B, n_heads, n_kv,
                                max_len, out, workspace, workspace_bytes, nullptr, (cudaStream_t)stream, &m);
}
