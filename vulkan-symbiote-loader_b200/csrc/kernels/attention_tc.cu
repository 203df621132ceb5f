// Long-context decode attention with the score product on tcgen05 tensor cores.
//
// Same semantics as flash_decode_kernel (attention.cu; reference attention.comp:84-189): query
// head h reads KV group h*n_kv/n_heads, scores q.k / sqrt(head_dim), max-subtracted softmax over
// positions [0, pos], output = probabilities times V. Built for caches of thousands of positions
// (fp16 KV, head_dim 128, up to 8 query heads per KV group):
//   * S^T[128 positions][16] = K_chunk[128][128] . Q2[16][128]^T on the tensor cores
//     (tcgen05.mma kind::f16, M = 128, N = 16, K = 16 x 8, fp32 accumulate in TMEM). Q2 holds
//     the group's query heads as hi/lo fp16 pairs (rows 0..G-1 hi, 8..8+G-1 lo, rest zero), so
//     the scores keep ~22 bits of the fp32 query; a thread reads the row of its position with
//     tcgen05.ld and adds the two columns. Positions sit on M because tcgen05 needs M >= 64 and a
//     group has only 4-8 query heads.
//   * softmax (online, fp32) and P.V on the CUDA cores: P.V costs one multiply-add per V byte
//     per head, well under the FMA rate needed at HBM speed; V is read straight from the
//     swizzled stage.
//   * K and V chunks (two 64-position pages each, 2 x 64-column 128-byte-swizzle atoms) arrive by
//     tensor TMA into a 3-stage mbarrier ring (192 KB in flight per SM).
//   * work split (stream-K): the flattened list of (sequence, KV group, 128-position chunk) is cut
//     into gridDim.x equal ranges, one per persistent CTA, whatever the per-sequence lengths; a
//     (sequence, group) shared by several CTAs is merged by the last to finish, in CTA order
//     (deterministic), with an atomic counter it resets to zero.
// Roles: warps 0-3 softmax (TMEM lane quarter = warp), warps 0-7 P.V, warp 8 TMA producer,
// warp 9 TMEM allocation and the single-thread MMA issue. Every wait is bounded (one second) and records
// VSL_ERR_TIMEOUT; the kernel then drains its copies and MMAs and frees its TMEM.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <math_constants.h>

#include <mutex>

#include "common.cuh"
#include "launch.cuh"

namespace vsl {

constexpr int FT_THREADS = 320;  // 8 softmax/P.V warps, TMA producer, MMA issuer
constexpr int FT_CHUNK = 128;                 // positions per chunk (MMA M)
constexpr int FT_HD = 128;
constexpr int FT_GMAX = 8;
constexpr int FT_N = 16;                      // MMA N: 8 hi + 8 lo query rows
constexpr int FT_STAGES = 3;
constexpr int FT_ATOM = 128 * 64 * 2;         // one 64-column swizzle atom of a 128-row tile (16 KB)
constexpr int FT_STAGE = 4 * FT_ATOM;         // K (2 atoms) + V (2 atoms) = 64 KB
constexpr int FT_Q2 = 2 * FT_N * 128;         // 2 atoms of 16 rows x 128 bytes
constexpr int FT_BMAX = 64;
constexpr size_t FT_RED = (size_t)3 * FT_GMAX * FT_HD * 4;  // partial outputs of position quarters 1-3
constexpr size_t FT_SMEM = 1024 + (size_t)FT_STAGES * FT_STAGE + FT_Q2 + (size_t)FT_CHUNK * FT_GMAX * 4 + FT_RED;

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
    uint32_t idesc;
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

// Flattened work list: for sequence b, n_kv groups x nch[b] chunks, starting at off[b].
struct FtWork {
    int nch[FT_BMAX], len[FT_BMAX];
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
    flash_decode_tc_kernel(const __grid_constant__ CUtensorMap map_k, const __grid_constant__ CUtensorMap map_v,
                           const __grid_constant__ FtArgs a) {
    extern __shared__ unsigned char smem_raw[];
    __shared__ __align__(8) uint64_t full[FT_STAGES], empty[FT_STAGES], s_full[2], s_free[2], q_ready;
    __shared__ uint32_t tmem_s;
    __shared__ int abort_s, last_s;
    __shared__ float red_max[4][FT_GMAX], red_sum[4][FT_GMAX];
    __shared__ FtWork wk;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
    const uint32_t ring = base;
    const uint32_t q2 = base + FT_STAGES * FT_STAGE;
    float* Ps = reinterpret_cast<float*>(smem_raw + (q2 + FT_Q2 - smem_u32(smem_raw)));  // [128][8]
    float* red_o = Ps + FT_CHUNK * FT_GMAX;                                                // [3][8][128]
    const int c = blockIdx.x;

    if (threadIdx.x == 0) {
        for (int s = 0; s < FT_STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 8);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&s_full[i], 1);
            mbar_init(&s_free[i], 4);
        }
        mbar_init(&q_ready, 4);
        mbar_fence_init();
        abort_s = 0;
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_k)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_v)) : "memory");
    }
    if (warp == 9) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_s)), "r"(32)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    pdl_wait();
    pdl_launch_dependents();
    if (warp == 0) {  // work list from the current positions
        for (int b = lane; b < a.B; b += 32) {
            int len = __ldcg(a.pos + b) + 1;
            len = len < 1 ? 1 : (len > a.max_len ? a.max_len : len);
            wk.len[b] = len;
            wk.nch[b] = (len + FT_CHUNK - 1) / FT_CHUNK;
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

    if (warp == 8) {
        // ================= TMA producer =================
        if (lane == 0) {
            FtCur cu;
            if (f0 < f1) ft_seek(wk, a.B, a.n_kv, f0, cu);
            int s = 0;
            uint32_t epar = 1u;
            long long it = 0;
            bool ok = true;
            for (long long f = f0; f < f1 && ok; f++, it++) {
                if (it >= FT_STAGES && !mbar_wait(&empty[s], epar)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(&full[s], FT_STAGE);
                const uint32_t st = ring + s * FT_STAGE;
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    int p0 = cu.ch * FT_CHUNK + h * 64;
                    if (p0 >= wk.len[cu.b]) p0 = 0;  // past the end: any valid page (masked later)
                    const int page = __ldg(a.page_table + (size_t)cu.b * a.max_pages + p0 / a.page_size);
                    const int row = (page * a.n_kv + cu.g) * a.page_size + (p0 % a.page_size);
#pragma unroll
                    for (int at = 0; at < 2; at++) {
                        ft_tma(st + at * FT_ATOM + h * (FT_ATOM / 2), &map_k, at * 64, row, &full[s]);
                        ft_tma(st + (2 + at) * FT_ATOM + h * (FT_ATOM / 2), &map_v, at * 64, row, &full[s]);
                    }
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
                mbar_wait(&full[u % FT_STAGES], (uint32_t)((u / FT_STAGES) & 1));
        }
    } else if (warp == 9) {
        // ================= MMA issue =================
        if (lane == 0) {
            FtCur cu;
            if (f0 < f1) ft_seek(wk, a.B, a.n_kv, f0, cu);
            int s = 0, buf = 0, seg = 0;
            uint32_t fpar = 0u;
            long long it = 0;
            bool ok = true;
            int pb = -1, pg = -1;
            for (long long f = f0; f < f1 && ok; f++, it++) {
                if (cu.b != pb || cu.g != pg) {  // new (sequence, group): its query rows must be staged
                    if (!mbar_wait(&q_ready, (uint32_t)(seg & 1))) {
                        ok = false;
                        break;
                    }
                    seg++;
                    pb = cu.b;
                    pg = cu.g;
                }
                if (!mbar_wait(&full[s], fpar) || (it >= 2 && !mbar_wait(&s_free[buf], (uint32_t)(((it >> 1) - 1) & 1))) ||
                    ft_abort(&abort_s)) {
                    ok = false;
                    break;
                }
                ft_fence_after();
                const uint32_t st = ring + s * FT_STAGE;
#pragma unroll
                for (int at = 0; at < 2; at++) {
                    const uint64_t ad = ft_desc(st + at * FT_ATOM), bd = ft_desc(q2 + at * (FT_Q2 / 2));
#pragma unroll
                    for (int k = 0; k < 4; k++)
                        asm volatile(
                            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                            "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem + buf * FT_N),
                            "l"(ad + (uint64_t)(2 * k)), "l"(bd + (uint64_t)(2 * k)), "r"(a.idesc),
                            "r"((at > 0 || k > 0) ? 1u : 0u)
                            : "memory");
                }
                asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                                 smem_u32(&s_full[buf]))
                             : "memory");
                ft_next(wk, a.n_kv, cu);
                buf ^= 1;
                if (++s == FT_STAGES) {
                    s = 0;
                    fpar ^= 1u;
                }
            }
            if (!ok) {
                set_status(a.status, VSL_ERR_TIMEOUT);
                atomicExch(&abort_s, 1);
            }
            if (it > 0) mbar_wait(&s_full[(it - 1) & 1], (uint32_t)(((it - 1) >> 1) & 1));  // last MMAs done
        }
        __syncwarp();
    } else {
        // ================= softmax (warps 0-3) + P.V (warps 0-7) =================
        // warps 0-3: thread t reads TMEM row t (its position in the chunk) and runs the online
        // softmax; all 8 warps then share P.V: thread t owns output dims 2*(t&63), +1 over the
        // position quarter t>>6 of the chunk, with its own partial accumulator (the four quarters
        // are summed in order at the end of a segment)
        const int t = threadIdx.x;
        const bool sm_warp = warp < 4;
        const int dp = t & 63, pq = t >> 6;
        const int G = a.G;
        float m[FT_GMAX], l[FT_GMAX], o0[FT_GMAX], o1[FT_GMAX];
        FtCur cu;
        if (f0 < f1) ft_seek(wk, a.B, a.n_kv, f0, cu);
        int s = 0, buf = 0;
        long long it = 0;
        int pb = -1, pg = -1;
        // V element (position p, dims 2dp..2dp+1) inside a stage: atom dp/32, row p, 16-byte chunk
        // ((2dp mod 64)/8) ^ (p mod 8), byte (2dp mod 8)*2
        const int v_atom = dp >> 5, v_chunk = (dp & 31) >> 2, v_byte = (dp & 3) * 4;
        for (long long f = f0; f < f1; f++, it++) {
            const int b = cu.b, g = cu.g, ch = cu.ch;
            const int len = wk.len[b];
            if (b != pb || g != pg) {
                // ---- new (sequence, group): reset the softmax state, stage Q2 for the tensor cores ----
#pragma unroll
                for (int j = 0; j < FT_GMAX; j++) {
                    m[j] = -CUDART_INF_F;
                    l[j] = 0.0f;
                    o0[j] = 0.0f;
                    o1[j] = 0.0f;
                }
                if (sm_warp) {
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
                    unsigned char* q2p = smem_raw + (q2 - smem_u32(smem_raw)) + at * (FT_Q2 / 2);
                    const int rh = r, rl = r + 8;
                    *reinterpret_cast<uint4*>(q2p + rh * 128 + ((cc ^ (rh & 7)) << 4)) = hv;
                    *reinterpret_cast<uint4*>(q2p + rl * 128 + ((cc ^ (rl & 7)) << 4)) = lv;
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // visible to the tensor cores
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&q_ready);
                }
                pb = b;
                pg = g;
            }
            // ---- scores of this chunk (TMEM row t, warps 0-3) ----
            const int n_valid = min(FT_CHUNK, len - ch * FT_CHUNK);
            const bool valid = t < n_valid;
            float sc[FT_GMAX];
            {
                bool bad = false;
                if (sm_warp) bad = !mbar_wait(&s_full[buf], (uint32_t)((it >> 1) & 1));
                bad = bad || ft_abort(&abort_s);
                // the eight warps leave together (they meet at named barriers further down)
                if (named_barrier_or(1, 256, bad)) {
                    set_status(a.status, VSL_ERR_TIMEOUT);
                    atomicExch(&abort_s, 1);
                    break;
                }
            }
            if (sm_warp) {
                ft_fence_after();
                uint32_t r[16];
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, "
                    "[%16];"
                    : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                      "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
                      "=r"(r[15])
                    : "r"(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(buf * FT_N)));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                ft_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&s_free[buf]);
#pragma unroll
                for (int j = 0; j < FT_GMAX; j++)
                    sc[j] = (j < G && valid) ? (__uint_as_float(r[j]) + __uint_as_float(r[8 + j])) * a.scale
                                             : -CUDART_INF_F;
#pragma unroll
                for (int j = 0; j < FT_GMAX; j++) {
                    if (j >= G) break;
                    const float mx = warp_max(sc[j]);
                    if (lane == 0) red_max[warp][j] = mx;
                }
            }
            named_barrier_sync(1, 256);
            // ---- online softmax: every thread keeps the same running max / sum ----
            float alpha[FT_GMAX];
#pragma unroll
            for (int j = 0; j < FT_GMAX; j++) {
                if (j >= G) break;
                const float cm = fmaxf(fmaxf(red_max[0][j], red_max[1][j]), fmaxf(red_max[2][j], red_max[3][j]));
                const float mn = fmaxf(m[j], cm);
                alpha[j] = expf(m[j] - mn);
                if (sm_warp) {
                    const float pj = valid ? expf(sc[j] - mn) : 0.0f;
                    sc[j] = pj;
                    const float sm = warp_sum(pj);
                    if (lane == 0) red_sum[warp][j] = sm;
                }
                m[j] = mn;
            }
            if (sm_warp) {
                float4* pr = reinterpret_cast<float4*>(Ps + t * FT_GMAX);
                pr[0] = make_float4(sc[0], G > 1 ? sc[1] : 0.f, G > 2 ? sc[2] : 0.f, G > 3 ? sc[3] : 0.f);
                if (G > 4) pr[1] = make_float4(sc[4], G > 5 ? sc[5] : 0.f, G > 6 ? sc[6] : 0.f, G > 7 ? sc[7] : 0.f);
            }
            named_barrier_sync(1, 256);
#pragma unroll
            for (int j = 0; j < FT_GMAX; j++) {
                if (j >= G) break;
                l[j] = l[j] * alpha[j] + (red_sum[0][j] + red_sum[1][j] + red_sum[2][j] + red_sum[3][j]);
            }
            // ---- P.V: dims 2dp, 2dp+1 over positions [32 pq, 32 pq + 32) of the valid ones ----
            {
                const unsigned char* vb = smem_raw + (ring + s * FT_STAGE + 2 * FT_ATOM - smem_u32(smem_raw)) +
                                          v_atom * FT_ATOM + v_byte;
                float a0[FT_GMAX], a1[FT_GMAX];
#pragma unroll
                for (int j = 0; j < FT_GMAX; j++) a0[j] = a1[j] = 0.0f;
                const int pe = min(32 * pq + 32, n_valid);
#pragma unroll 4
                for (int pp = 32 * pq; pp < pe; pp++) {
                    const __half2 vh = *reinterpret_cast<const __half2*>(vb + pp * 128 + ((v_chunk ^ (pp & 7)) << 4));
                    const float2 v = __half22float2(vh);
                    const float4 w0 = *reinterpret_cast<const float4*>(Ps + pp * FT_GMAX);
                    a0[0] = fmaf(w0.x, v.x, a0[0]); a1[0] = fmaf(w0.x, v.y, a1[0]);
                    a0[1] = fmaf(w0.y, v.x, a0[1]); a1[1] = fmaf(w0.y, v.y, a1[1]);
                    a0[2] = fmaf(w0.z, v.x, a0[2]); a1[2] = fmaf(w0.z, v.y, a1[2]);
                    a0[3] = fmaf(w0.w, v.x, a0[3]); a1[3] = fmaf(w0.w, v.y, a1[3]);
                    if (G > 4) {
                        const float4 w1 = *reinterpret_cast<const float4*>(Ps + pp * FT_GMAX + 4);
                        a0[4] = fmaf(w1.x, v.x, a0[4]); a1[4] = fmaf(w1.x, v.y, a1[4]);
                        a0[5] = fmaf(w1.y, v.x, a0[5]); a1[5] = fmaf(w1.y, v.y, a1[5]);
                        a0[6] = fmaf(w1.z, v.x, a0[6]); a1[6] = fmaf(w1.z, v.y, a1[6]);
                        a0[7] = fmaf(w1.w, v.x, a0[7]); a1[7] = fmaf(w1.w, v.y, a1[7]);
                    }
                }
#pragma unroll
                for (int j = 0; j < FT_GMAX; j++) {
                    if (j >= G) break;
                    o0[j] = o0[j] * alpha[j] + a0[j];
                    o1[j] = o1[j] * alpha[j] + a1[j];
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
            if (++s == FT_STAGES) s = 0;
            buf ^= 1;
            // ---- end of this CTA's part of (b, g)? ----
            ft_next(wk, a.n_kv, cu);
            const bool seg_end = f + 1 == f1 || cu.b != b || cu.g != g;
            if (!seg_end) continue;
            // sum the four position quarters in order: quarters 1-3 stage their partials
            if (pq > 0) {
                float* ro = red_o + ((size_t)(pq - 1) * FT_GMAX) * FT_HD + 2 * dp;
#pragma unroll
                for (int j = 0; j < FT_GMAX; j++)
                    if (j < G) *reinterpret_cast<float2*>(ro + (size_t)j * FT_HD) = make_float2(o0[j], o1[j]);
            }
            named_barrier_sync(1, 256);
            const long long p0 = wk.off[b] + (long long)g * wk.nch[b];
            const int first = ft_owner(T, Gc, p0), lastc = ft_owner(T, Gc, p0 + wk.nch[b] - 1);
            float* out = a.out + ((size_t)b * a.n_heads + (size_t)g * G) * FT_HD + 2 * dp;
            const int slot = ft_lo(T, Gc, c) >= p0 ? 0 : 1;
            if (pq == 0) {
#pragma unroll
                for (int j = 0; j < FT_GMAX; j++) {
                    if (j >= G) break;
#pragma unroll
                    for (int q3 = 0; q3 < 3; q3++) {
                        const float2 v = *reinterpret_cast<const float2*>(red_o + ((size_t)q3 * FT_GMAX + j) * FT_HD + 2 * dp);
                        o0[j] += v.x;
                        o1[j] += v.y;
                    }
                }
                if (first == lastc) {
#pragma unroll
                    for (int j = 0; j < FT_GMAX; j++)
                        if (j < G) *reinterpret_cast<float2*>(out + (size_t)j * FT_HD) = make_float2(o0[j] / l[j], o1[j] / l[j]);
                } else {
                    float* wo = a.ws_o + (((size_t)c * 2 + slot) * FT_GMAX) * FT_HD + 2 * dp;
#pragma unroll
                    for (int j = 0; j < FT_GMAX; j++)
                        if (j < G) *reinterpret_cast<float2*>(wo + (size_t)j * FT_HD) = make_float2(o0[j], o1[j]);
                    if (dp < G) {
                        float* wml = a.ws_ml + (((size_t)c * 2 + slot) * FT_GMAX + dp) * 2;
                        float mt = m[0], lt = l[0];
#pragma unroll
                        for (int j = 1; j < FT_GMAX; j++)
                            if (j == dp) {
                                mt = m[j];
                                lt = l[j];
                            }
                        wml[0] = mt;
                        wml[1] = lt;
                    }
                }
            }
            if (first == lastc) {
                named_barrier_sync(1, 256);  // red_o is reused by the next segment
                continue;
            }
            __threadfence();
            named_barrier_sync(1, 256);
            if (t == 0) last_s = atomicAdd(a.counters + (size_t)b * a.n_kv + g, 1) == lastc - first;
            named_barrier_sync(1, 256);
            if (last_s && pq == 0) {
                __threadfence();
#pragma unroll
                for (int j = 0; j < FT_GMAX; j++) {
                    if (j >= G) break;
                    float M = -CUDART_INF_F;
                    for (int cc2 = first; cc2 <= lastc; cc2++) {
                        const int sl = ft_lo(T, Gc, cc2) >= p0 ? 0 : 1;
                        M = fmaxf(M, __ldcg(a.ws_ml + (((size_t)cc2 * 2 + sl) * FT_GMAX + j) * 2));
                    }
                    float L = 0.0f, O0 = 0.0f, O1 = 0.0f;
                    for (int cc2 = first; cc2 <= lastc; cc2++) {
                        const int sl = ft_lo(T, Gc, cc2) >= p0 ? 0 : 1;
                        const float* ml = a.ws_ml + (((size_t)cc2 * 2 + sl) * FT_GMAX + j) * 2;
                        const float w = expf(__ldcg(ml) - M);
                        L += __ldcg(ml + 1) * w;
                        const float2 ov =
                            __ldcg(reinterpret_cast<const float2*>(a.ws_o + (((size_t)cc2 * 2 + sl) * FT_GMAX + j) * FT_HD + 2 * dp));
                        O0 += ov.x * w;
                        O1 += ov.y * w;
                    }
                    *reinterpret_cast<float2*>(out + (size_t)j * FT_HD) = make_float2(O0 / L, O1 / L);
                }
                if (t == 0) a.counters[(size_t)b * a.n_kv + g] = 0;
            }
        }
    }

    ft_fence_before();
    __syncthreads();
    if (warp == 9) {
        ft_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(32) : "memory");
    }
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

// KV cache [rows = n_pages * n_kv * page_size][128] fp16 as 64-row x 64-column boxes, 128-byte swizzle
static int ft_map(CUtensorMap* m, const void* base, long long rows) {
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
                         int* status, cudaStream_t st) {
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
    // instruction descriptor (kind::f16): D f32 (bits 4-5 = 1), A/B f16 (0), both K-major,
    // N >> 3 in bits 17-22, M >> 4 in bits 24-28
    a.idesc = (1u << 4) | ((uint32_t)(FT_N >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
    const long long rows = (long long)n_pages * n_kv * page_size;
    CUtensorMap mk, mv;
    int rc = ft_map(&mk, k_cache, rows);
    if (rc) return rc;
    rc = ft_map(&mv, v_cache, rows);
    if (rc) return rc;
    static thread_local int configured_dev = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (configured_dev != dev) {
        cudaError_t e = cudaFuncSetAttribute(flash_decode_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)FT_SMEM);
        if (e != cudaSuccess) return launch_status(e, "flash_decode_tc smem attribute");
        configured_dev = dev;
    }
    return launch_status(launch_k(flash_decode_tc_kernel, dim3(grid), dim3(FT_THREADS), FT_SMEM, st, mk, mv, a),
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
                                max_len, out, workspace, workspace_bytes, nullptr, (cudaStream_t)stream);
}
