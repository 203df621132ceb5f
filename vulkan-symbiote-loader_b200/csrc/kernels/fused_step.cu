// Fused decode step: one persistent cooperative kernel runs a whole token.
//
// Replaces, for one token, the chain embed -> L x (QKV+RoPE+append, attention, O, gate/up,
// down) -> lm_head -> sample of separate launches (each a full-grid dependency with its own
// launch, ramp-up and tail). Here every SM holds one CTA for the whole token:
//   * warp 8 (producer) streams this CTA's share of EVERY projection's weights, phase after
//     phase, through a ring of 32 KB shared-memory stages with cp.async.bulk (TMA); it never
//     waits for the phase barriers, so the next projection's first tiles are already on chip
//     when the consumers leave a barrier;
//   * warps 0-7 (consumers) run the phases: RMSNorm-staged activations, dot products from the
//     shared-memory stages (8 rows per warp, so each activation read from shared memory serves
//     8 weights), the shared projection epilogues (residual add, SwiGLU, RoPE + KV append,
//     lm_head argmax), chunked attention with a combine phase, and the token bookkeeping;
//     phases are separated by a grid barrier on a global arrival counter.
// Every wait is bounded (one second): on expiry the kernel records VSL_ERR_TIMEOUT, raises the
// abort flag so the other CTAs stop too, and returns. The launch is cooperative, so all CTAs
// are resident and the barrier cannot wait on a CTA that never runs.
#include <cuda_runtime.h>
#include <math_constants.h>

#include <type_traits>

#include "common.cuh"
#include "epilogue.cuh"
#include "fused_step.h"
#include "launch.cuh"

namespace vsl {

constexpr int FS_NCW = 8;                      // consumer warps
constexpr int FS_CT = FS_NCW * 32;             // consumer threads
constexpr int FS_THREADS = FS_CT + 32;         // + producer warp
constexpr int FS_BMAX = 4;                     // activation rows supported
constexpr int FS_RED = 8;                      // slots of the row-group reduction ring

// ---------------------------------------------------------------------------------------
// chunk cursor over the weight stream of this CTA (identical walk in producer and consumers)
// ---------------------------------------------------------------------------------------
struct Cursor {
    int ph;         // phase index (a FS_GEMV phase) or n_phases when done
    int g, c;       // group and piece within the phase
    int rb, re;     // this CTA's rows of the phase
    int n_groups;
    // the phase's geometry, loaded once per phase: the producer must not wait on a global
    // load for every tile it issues
    const char* W;
    int K, R, kc, n_kc;
};

__device__ __forceinline__ void cta_rows(int N, int& rb, int& re) {
    const int U = (N + 1) >> 1;
    const int u0 = (int)(((long long)U * blockIdx.x) / gridDim.x);
    const int u1 = (int)(((long long)U * (blockIdx.x + 1)) / gridDim.x);
    rb = 2 * u0;
    re = min(N, 2 * u1);
}

// first chunk of the first GEMV phase at or after `ph` that gives this CTA any rows
__device__ __forceinline__ void cursor_seek(const FsProgram& P, Cursor& cu, int ph) {
    for (; ph < P.n_phases; ph++) {
        const FsPhase& f = P.phases[ph];
        if (f.kind != FS_GEMV) continue;
        int rb, re;
        cta_rows(f.N, rb, re);
        if (re <= rb) continue;
        cu.ph = ph;
        cu.g = 0;
        cu.c = 0;
        cu.rb = rb;
        cu.re = re;
        cu.n_groups = (re - rb + f.R - 1) / f.R;
        cu.W = reinterpret_cast<const char*>(f.W);
        cu.K = f.K;
        cu.R = f.R;
        cu.kc = f.kc;
        cu.n_kc = f.n_kc;
        return;
    }
    cu.ph = P.n_phases;
}

__device__ __forceinline__ void cursor_next(const FsProgram& P, Cursor& cu) {
    if (++cu.c < cu.n_kc) return;
    cu.c = 0;
    if (++cu.g < cu.n_groups) return;
    cursor_seek(P, cu, cu.ph + 1);
}

__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ int ld_volatile_i32(const int* p) {
    return *reinterpret_cast<const volatile int*>(p);
}

// Bounded wait for phase `par` of an mbarrier. The abort flag lives in global memory (an L2
// round trip), so it is read only every 1024 polls and the time limit every 16: a poll loop
// that read it each time would see a completed phase up to a microsecond late.
__device__ __forceinline__ bool fs_wait(uint64_t* bar, uint32_t par, const int* abort_flag) {
    if (mbar_try_wait(bar, par)) return true;
    const unsigned long long t0 = globaltimer_ns();
    for (unsigned it = 1;; it++) {
        if (mbar_try_wait(bar, par)) return true;
        if ((it & 15u) == 0u) {
            if (globaltimer_ns() - t0 > WAIT_LIMIT_NS) return false;
            if ((it & 1023u) == 0u && ld_volatile_i32(abort_flag)) return false;
        }
    }
}

// ---------------------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------------------
template <typename WT, typename KT, int HD>
__global__ void __launch_bounds__(FS_THREADS, 1) vsl_fused_step_kernel(const __grid_constant__ FsProgram P) {
    extern __shared__ __align__(128) unsigned char smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + FS_STAGES;
    unsigned char* ring = smem + FS_HEAD;
    unsigned char* work = ring + FS_STAGES * FS_CHUNK;
    // cross-warp partial sums of a row group: [group % FS_RED][tile row * cg + column group]
    // [sequence], with an arrival count per row group; the last warp to arrive reduces.
    // A warp runs at most FS_STAGES tiles (so groups) ahead of the slowest one (a ring slot is
    // refilled only when every warp has released it), so FS_RED > FS_STAGES slots never clash.
    __shared__ float red[FS_RED][64][FS_BMAX];
    __shared__ int red_cnt[FS_RED][FS_NCW];
    __shared__ float norm_ss[FS_NCW][FS_BMAX];
    __shared__ unsigned long long best_s[FS_BMAX];
    __shared__ int s_ok;
    __shared__ unsigned long long s_base;

    constexpr int VEC = WTraits<WT>::VEC;
    constexpr int ES = (int)sizeof(WT);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, ct = threadIdx.x;
    const int B = P.B;

    if (threadIdx.x == 0) {
        for (int s = 0; s < FS_STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], FS_NCW);
        }
        mbar_fence_init();
        s_base = *reinterpret_cast<volatile unsigned long long*>(P.bar_epoch);
        s_ok = 1;
    }
    if (threadIdx.x < FS_BMAX) best_s[threadIdx.x] = 0ull;
    if (threadIdx.x < FS_RED * FS_NCW) red_cnt[threadIdx.x / FS_NCW][threadIdx.x % FS_NCW] = 0;
    __syncthreads();
    // a previous launch gave up on a wait: stay idle until the host resets the engine
    if (ld_volatile_i32(P.abort_flag)) return;
    if (P.trace && blockIdx.x == 0 && threadIdx.x == 0) P.trace[0] = globaltimer_ns();

    // =====================================================================================
    // producer warp: the weight stream
    // =====================================================================================
    if (warp == FS_NCW) {
        if (lane == 0) {
            Cursor cu;
            cursor_seek(P, cu, 0);
            for (long long t = 0; cu.ph < P.n_phases; t++) {
                const int s = (int)(t % FS_STAGES);
                if (t >= FS_STAGES) {
                    const bool ok = fs_wait(&empty[s], (uint32_t)(((t / FS_STAGES) - 1) & 1), P.abort_flag);
                    if (!ok) {
                        set_status(P.status, VSL_ERR_TIMEOUT);
                        atomicExch(P.abort_flag, 1);
                        // drain what is in flight before leaving
                        for (long long u = (t > FS_STAGES ? t - FS_STAGES : 0); u < t; u++)
                            mbar_wait(&full[u % FS_STAGES], (uint32_t)((u / FS_STAGES) & 1));
                        return;
                    }
                }
                {
                    const int row0 = cu.rb + cu.g * cu.R;
                    const int nrows = min(cu.R, cu.re - row0);
                    const int kc0 = cu.c * cu.kc;
                    const uint32_t piece = (uint32_t)(min(cu.kc, cu.K - kc0) * ES);
                    const char* src = cu.W + ((size_t)row0 * cu.K + kc0) * ES;
                    unsigned char* dst = ring + (size_t)s * FS_CHUNK;
                    mbar_arrive_expect_tx(&full[s], piece * (uint32_t)nrows);
                    if (cu.n_kc == 1) {
                        bulk_g2s(dst, src, piece * (uint32_t)nrows, &full[s]);  // whole rows: contiguous
                    } else {
                        for (int r = 0; r < nrows; r++)
                            bulk_g2s(dst + (size_t)r * cu.kc * ES, src + (size_t)r * cu.K * ES, piece, &full[s]);
                    }
                }
                cursor_next(P, cu);
                if (cu.ph >= P.n_phases) {
                    // every copy issued must land before this CTA may exit
                    for (long long u = (t + 1 > FS_STAGES ? t + 1 - FS_STAGES : 0); u <= t; u++)
                        mbar_wait(&full[u % FS_STAGES], (uint32_t)((u / FS_STAGES) & 1));
                }
            }
        }
        return;
    }

    // =====================================================================================
    // consumer warps
    // =====================================================================================
    int n_bar = 0;
    auto grid_sync = [&]() -> bool {
        named_barrier_sync(1, FS_CT);
        if (ct == 0) {
            __threadfence();
            atomicAdd(P.bar_counter, 1ull);
            n_bar++;
            const unsigned long long target = s_base + (unsigned long long)n_bar * gridDim.x;
            bool ok = ld_acquire_u64(P.bar_counter) >= target;
            if (!ok) {
                const unsigned long long t0 = globaltimer_ns();
                while (!ok) {
                    for (int i = 0; i < 64 && !ok; i++) ok = ld_acquire_u64(P.bar_counter) >= target;
                    if (!ok && (ld_volatile_i32(P.abort_flag) || globaltimer_ns() - t0 > WAIT_LIMIT_NS)) break;
                }
            }
            if (!ok) {
                set_status(P.status, VSL_ERR_TIMEOUT);
                atomicExch(P.abort_flag, 1);
            }
            __threadfence();
            s_ok = ok ? 1 : 0;
        } else {
            n_bar++;
        }
        named_barrier_sync(1, FS_CT);
        return s_ok != 0;
    };

    // position and KV page of the sequence this thread serves in projection epilogues
    // (lane % B); both stay fixed for the whole step
    int e_pos = 0, e_page = -1;
    if (lane < 4 * B) {
        const int b = lane % B;
        e_pos = __ldcg(P.pos + b);
        if (e_pos >= 0 && e_pos < P.max_pages * P.page_size)
            e_page = __ldcg(P.page_table + (size_t)b * P.max_pages + e_pos / P.page_size);
    }
    int gseq = 0;        // row groups reduced so far (reduction ring position)
    int rs = 0;          // ring stage of the next tile (same walk as the producer)
    uint32_t rpar = 0u;  // its mbarrier phase parity
    float* xs = reinterpret_cast<float*>(work);
    const int steps_now = *P.step;

    for (int ph = 0; ph < P.n_phases; ph++) {
        const FsPhase& f = P.phases[ph];
        if (f.kind == FS_EMBED) {
            // x[b][j] = E[min(id, V-1)][j] for this CTA's slice of j (embedding_lookup.comp:29-40)
            const int j0 = (int)(((long long)P.d * blockIdx.x) / gridDim.x);
            const int j1 = (int)(((long long)P.d * (blockIdx.x + 1)) / gridDim.x);
            for (int b = 0; b < B; b++) {
                int id = __ldcg(P.ids + b);
                id = id < 0 ? 0 : (id > P.V - 1 ? P.V - 1 : id);
                const WT* row = reinterpret_cast<const WT*>(P.tok_embd) + (size_t)id * P.d;
                for (int j = j0 + ct; j < j1; j += FS_CT) P.x[(size_t)b * P.d + j] = WTraits<WT>::load(row, j);
            }
            if (blockIdx.x == 0 && ct < B) P.slots[ct] = 0ull;
        } else if (f.kind == FS_GEMV) {
            int rb, re;
            cta_rows(f.N, rb, re);
            const int K = f.K;
            const int K4 = K / 4;
            // ---- stage activations (RMS-normalised when the phase follows a norm) ----
            // cp.async straight into shared memory, with the norm weights loaded into registers
            // meanwhile: one global round trip. For 16-bit weights (8 per vector) sequence b's
            // activations are stored split: float4 j of the row goes to slot (j & 1) * K/8 + j/2,
            // so the two float4s that meet weight vector v sit at v and K/8 + v and a warp's 32
            // lanes read 512 contiguous bytes each time.
            {
                const int nvec = B * K4;  // float4s in x ([B][K], K % VEC == 0)
                const float4* xg = reinterpret_cast<const float4*>(f.x);
                float4* xs4w = reinterpret_cast<float4*>(xs);
                for (int jj = ct; jj < nvec; jj += FS_CT) {
                    const int b = jj / K4, j = jj - b * K4;
                    const int slot = VEC == 8 ? (j & 1) * (K4 >> 1) + (j >> 1) : j;
                    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(xs4w + b * K4 + slot)),
                                 "l"(xg + jj)
                                 : "memory");
                }
                asm volatile("cp.async.commit_group;" ::: "memory");
                constexpr int MAXW = FS_WORK / 16 / FS_CT;  // norm-weight float4s per thread (K <= 16384)
                float4 nw[MAXW];
                const float4* nw4 = reinterpret_cast<const float4*>(f.norm_w);
                if (nw4) {
#pragma unroll
                    for (int i = 0; i < MAXW; i++)
                        if (ct + i * FS_CT < K4) nw[i] = __ldg(nw4 + ct + i * FS_CT);
                }
                asm volatile("cp.async.wait_group 0;" ::: "memory");
                named_barrier_sync(1, FS_CT);
                if (nw4) {
                    // sum of squares per sequence over this thread's float4s
                    float ss[FS_BMAX] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
                    for (int i = 0; i < MAXW; i++) {
                        const int j = ct + i * FS_CT;
                        if (j < K4) {
                            const int slot = VEC == 8 ? (j & 1) * (K4 >> 1) + (j >> 1) : j;
#pragma unroll
                            for (int b = 0; b < FS_BMAX; b++) {
                                if (b >= B) break;
                                const float4 v = xs4w[b * K4 + slot];
                                ss[b] += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
                            }
                        }
                    }
#pragma unroll
                    for (int b = 0; b < FS_BMAX; b++) {
                        const float s2 = warp_sum(ss[b]);
                        if (lane == 0) norm_ss[warp][b] = s2;
                    }
                    named_barrier_sync(1, FS_CT);
                    float den[FS_BMAX];
#pragma unroll
                    for (int b = 0; b < FS_BMAX; b++) {
                        float s2 = 0.0f;
#pragma unroll
                        for (int w = 0; w < FS_NCW; w++) s2 += norm_ss[w][b];
                        den[b] = sqrtf(s2 / (float)K + P.eps);  // rms_norm.comp:32-34: x / sqrt(var) * w
                    }
#pragma unroll
                    for (int i = 0; i < MAXW; i++) {
                        const int j = ct + i * FS_CT;
                        if (j < K4) {
                            const int slot = VEC == 8 ? (j & 1) * (K4 >> 1) + (j >> 1) : j;
                            const float4 w = nw[i];
#pragma unroll
                            for (int b = 0; b < FS_BMAX; b++) {
                                if (b >= B) break;
                                const float4 v = xs4w[b * K4 + slot];
                                const float dd = den[b];
                                xs4w[b * K4 + slot] =
                                    make_float4(v.x / dd * w.x, v.y / dd * w.y, v.z / dd * w.z, v.w / dd * w.w);
                            }
                        }
                    }
                    named_barrier_sync(1, FS_CT);
                }
            }

            // warp (row group rg, column group cg): tile rows [8 rg, 8 rg + 8), columns
            // [cg/CG, (cg+1)/CG) of every piece
            const int R = f.R, CG = f.cg, kc = f.kc, n_kc = f.n_kc;
            const int rg = warp / CG, cg = warp - rg * CG;
            const int myr = rg * 8;
            const float4* xs4 = reinterpret_cast<const float4*>(xs);
            const int n_groups = re > rb ? (re - rb + R - 1) / R : 0;
            unsigned long long best[FS_BMAX] = {0ull, 0ull, 0ull, 0ull};
            // the tile loop, compiled per batch bound NB (1, 2 or 4) so that the accumulators
            // of the common single-sequence case stay small
            auto tiles = [&](auto nb_tag) -> bool {
                constexpr int NB = decltype(nb_tag)::value;
                            for (int g = 0; g < n_groups; g++) {
                    const int row0 = rb + g * R;
                    const int nrows = min(R, re - row0);
                    const int my_n = nrows - myr;  // rows of this warp in the tile (<= 0: none)
                    // epilogue lanes (one per (pair, sequence) in every warp: the warp that finishes
                    // the row group last runs its epilogue) fetch their residual / RoPE inputs
                    // now, so the loads overlap this group's weight stream
                    const bool epi_lane = lane < 4 * B;
                    const int e_pi = lane / B, e_b = lane - e_pi * B, e_r = myr + 2 * e_pi;
                    const bool e_has1 = e_r + 1 < nrows;
                    EpiPre pre = {0.0f, 0.0f, e_pos, e_page};
                    if (epi_lane && e_r < nrows) {
                        GemvParams ep = {};
                        ep.N = f.N; ep.y = f.y; ep.head_dim = HD; ep.n_heads = P.nh; ep.n_kv = P.nkv;
                        ep.rope_cos = P.rope_cos; ep.rope_sin = P.rope_sin;
                        if (f.epi == EK_ADD) pre = epi_fetch<EK_ADD>(ep, e_b, row0 + e_r, e_has1, e_pos, e_page);
                        else if (f.epi == EK_QKV) pre = epi_fetch<EK_QKV>(ep, e_b, row0 + e_r, e_has1, e_pos, e_page);
                    }
                    float acc[8][NB];
#pragma unroll
                    for (int r = 0; r < 8; r++)
#pragma unroll
                        for (int b = 0; b < NB; b++) acc[r][b] = 0.0f;
                    for (int c = 0; c < n_kc; c++) {
                        const bool ok = fs_wait(&full[rs], rpar, P.abort_flag);
                        if (!ok) {
                            set_status(P.status, VSL_ERR_TIMEOUT);
                            atomicExch(P.abort_flag, 1);
                            return false;
                        }
                        if (my_n > 0) {
                            const int kc0 = c * kc;
                            const int nv = min(kc, K - kc0) / VEC;
                            const int v0 = (nv * cg) / CG, v1 = (nv * (cg + 1)) / CG;
                            const WT* st = reinterpret_cast<const WT*>(ring + (size_t)rs * FS_CHUNK) + (size_t)myr * kc;
                            const int kv0 = kc0 / VEC;
                            for (int v = v0 + lane; v < v1; v += 32) {
                                float xv[NB][VEC];
#pragma unroll
                                for (int b = 0; b < NB; b++) {
                                    if (b >= B) break;
                                    if constexpr (VEC == 8) {
                                        const float4 xa = xs4[b * K4 + kv0 + v], xb = xs4[b * K4 + (K4 >> 1) + kv0 + v];
                                        xv[b][0] = xa.x; xv[b][1] = xa.y; xv[b][2] = xa.z; xv[b][3] = xa.w;
                                        xv[b][4] = xb.x; xv[b][5] = xb.y; xv[b][6] = xb.z; xv[b][7] = xb.w;
                                    } else {
                                        const float4 xa = xs4[b * K4 + kv0 + v];
                                        xv[b][0] = xa.x; xv[b][1] = xa.y; xv[b][2] = xa.z; xv[b][3] = xa.w;
                                    }
                                }
                                // all 8 rows, also past the tile's last row: those read stale but
                                // in-bounds stage memory (rows < 64, row < 4 KB, within the ring +
                                // work area) and their sums are never used
                                uint4 wv[8];
#pragma unroll
                                for (int r = 0; r < 8; r++)
                                    wv[r] = *reinterpret_cast<const uint4*>(st + (size_t)r * kc + (size_t)v * VEC);
#pragma unroll
                                for (int r = 0; r < 8; r++) {
                                    float fw[VEC];
                                    WTraits<WT>::widen(wv[r], fw);
#pragma unroll
                                    for (int b = 0; b < NB; b++) {
                                        if (b >= B) break;
                                        float a = acc[r][b];
#pragma unroll
                                        for (int e = 0; e < VEC; e++) a = fmaf(fw[e], xv[b][e], a);
                                        acc[r][b] = a;
                                    }
                                }
                            }
                        }
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&empty[rs]);
                        if (++rs == FS_STAGES) {
                            rs = 0;
                            rpar ^= 1u;
                        }
                    }
                    // ---- rows complete: lane reduction of the 8 rows at once (after the three
                    // halving exchanges lane L holds row (L>>4&1)*4 + (L>>3&1)*2 + (L>>2&1), summed
                    // over the lanes that share those bits; two more exchanges finish it) ----
                    const int buf = gseq & (FS_RED - 1);
                    gseq++;
                    const int ri = ((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1);
#pragma unroll
                    for (int b = 0; b < NB; b++) {
                        if (b >= B) break;
                        float q[8];
#pragma unroll
                        for (int r = 0; r < 8; r++) q[r] = acc[r][b];
#pragma unroll
                        for (int h = 4, off = 16; h >= 1; h >>= 1, off >>= 1) {
                            const bool up = (lane & off) != 0;
#pragma unroll
                            for (int i = 0; i < h; i++) {
                                const float send = up ? q[i] : q[i + h];
                                const float keep = up ? q[i + h] : q[i];
                                q[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
                            }
                        }
                        float sum = q[0];
                        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
                        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
                        if ((lane & 3) == 0 && myr + ri < R) red[buf][(myr + ri) * CG + cg][b] = sum;
                    }
                    // ---- arrival: the last of the row group's CG warps reduces (no barrier) ----
                    __threadfence_block();
                    __syncwarp();
                    int prev = 0;
                    if (lane == 0) prev = atomicAdd(&red_cnt[buf][rg], 1);
                    prev = __shfl_sync(0xffffffffu, prev, 0);
                    if (prev != CG - 1) continue;
                    __threadfence_block();  // the other warps' partials are visible from here on
                    // ---- pair epilogues: lanes (pair, sequence) of the last warp ----
                    if (epi_lane && e_r < nrows) {
                        float s0 = 0.0f, s1 = 0.0f;
                        for (int j = 0; j < CG; j++) s0 += red[buf][e_r * CG + j][e_b];
                        if (e_has1)
                            for (int j = 0; j < CG; j++) s1 += red[buf][(e_r + 1) * CG + j][e_b];
                        const int r0 = row0 + e_r;
                        GemvParams ep = {};
                        ep.N = f.N; ep.K = K; ep.y = f.y; ep.B = B;
                        ep.n_heads = P.nh; ep.n_kv = P.nkv; ep.head_dim = HD;
                        ep.q_out = P.q; ep.k_cache = P.kv[f.layer].k; ep.v_cache = P.kv[f.layer].v;
                        ep.kvdtype = P.kvdtype; ep.page_size = P.page_size;
                        ep.vocab_offset = P.vocab_offset; ep.inv_temp = P.inv_temp; ep.seed = P.seed;
                        ep.status = P.status;
                        unsigned long long& bb = best[e_b];
                        switch (f.epi) {
                            case EK_STORE: epi_apply<EK_STORE>(ep, pre, e_b, r0, r0 >> 1, e_has1, s0, s1, bb, steps_now); break;
                            case EK_ADD: epi_apply<EK_ADD>(ep, pre, e_b, r0, r0 >> 1, e_has1, s0, s1, bb, steps_now); break;
                            case EK_SWIGLU: epi_apply<EK_SWIGLU>(ep, pre, e_b, r0, r0 >> 1, e_has1, s0, s1, bb, steps_now); break;
                            case EK_QKV: epi_apply<EK_QKV>(ep, pre, e_b, r0, r0 >> 1, e_has1, s0, s1, bb, steps_now); break;
                            default: epi_apply<EK_LMHEAD>(ep, pre, e_b, r0, r0 >> 1, e_has1, s0, s1, bb, steps_now); break;
                        }
                    }
                    __syncwarp();
                    if (lane == 0) red_cnt[buf][rg] = 0;
                }
                return true;
            };
            bool tiles_ok;
            if (B == 1) tiles_ok = tiles(std::integral_constant<int, 1>{});
            else if (B == 2) tiles_ok = tiles(std::integral_constant<int, 2>{});
            else tiles_ok = tiles(std::integral_constant<int, 4>{});
            // a warp whose wait expired has raised the abort flag and skipped its remaining
            // tiles; it still takes part in the barriers below, and the grid barrier then
            // returns false for every consumer warp together
            (void)tiles_ok;
            if (f.epi == EK_LMHEAD) {
#pragma unroll
                for (int b = 0; b < FS_BMAX; b++)
                    if (b < B && best[b]) atomicMax(&best_s[b], best[b]);
                named_barrier_sync(1, FS_CT);
                if (ct < B) {
                    if (best_s[ct]) atomicMax(P.slots + ct, best_s[ct]);
                    best_s[ct] = 0ull;
                }
            }
        } else if (f.kind == FS_ATTN) {
            // chunked attention: item = (b, kv group, 64-position chunk) -> partial (o, m, l)
            // (attention.comp:92,116-189 semantics; combined in the next phase)
            constexpr int RE = HD + 16 / (int)sizeof(KT);
            constexpr int KV = 16 / (int)sizeof(KT);
            KT* ks = reinterpret_cast<KT*>(work);
            KT* vs = ks + 64 * RE;
            float* qs = reinterpret_cast<float*>(vs + 64 * RE);  // [G][HD]
            float* part = qs + 8 * HD;                           // [4][8][64]
            float* pm = part + 4 * 8 * 64;                        // probabilities [8][64]
            float* ml = pm + 8 * 64;                              // m[8], l[8]
            float* op = ml + 16;                                  // [256 / HD][8][HD] partial outputs
            const int G = P.nh / P.nkv;
            const float scale = 1.0f / sqrtf((float)HD);
            int nch[FS_BMAX];
            int total = 0;
            for (int b = 0; b < FS_BMAX; b++) {
                nch[b] = 0;
                if (b < B) {
                    const int len = min(__ldcg(P.pos + b) + 1, min(P.max_seq, P.max_pages * P.page_size));
                    nch[b] = min(P.max_chunks, (len + 63) / 64);
                    total += nch[b] * P.nkv;
                }
            }
            for (int item = blockIdx.x; item < total; item += gridDim.x) {
                int rem = item, b = 0;
                while (rem >= nch[b] * P.nkv) {
                    rem -= nch[b] * P.nkv;
                    b++;
                }
                const int g = rem / nch[b], ch = rem % nch[b];
                const int len = min(__ldcg(P.pos + b) + 1, min(P.max_seq, P.max_pages * P.page_size));
                const int t0 = ch * 64, n = min(64, len - t0);
                const int page = __ldcg(P.page_table + (size_t)b * P.max_pages + t0 / P.page_size);
                const size_t base = (((size_t)page * P.nkv + g) * P.page_size + (t0 % P.page_size)) * HD;
                const KT* kg = reinterpret_cast<const KT*>(P.kv[f.layer].k) + base;
                const KT* vg = reinterpret_cast<const KT*>(P.kv[f.layer].v) + base;
                for (int i = ct; i < n * (HD / KV); i += FS_CT) {
                    const int r = i / (HD / KV), cc = (i % (HD / KV)) * KV;
                    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(ks + r * RE + cc)),
                                 "l"(kg + (size_t)r * HD + cc)
                                 : "memory");
                    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(vs + r * RE + cc)),
                                 "l"(vg + (size_t)r * HD + cc)
                                 : "memory");
                }
                asm volatile("cp.async.commit_group;" ::: "memory");
                const int h0 = g * G;
                for (int i = ct; i < G * HD; i += FS_CT) qs[i] = __ldcg(P.q + ((size_t)b * P.nh + h0) * HD + i);
                asm volatile("cp.async.wait_group 0;" ::: "memory");
                named_barrier_sync(1, FS_CT);
                {  // scores: thread (tt, quarter of the head dimension)
                    const int tt = ct & 63, qt = ct >> 6;
                    if (tt < n) {
                        float a[8];
#pragma unroll
                        for (int j = 0; j < 8; j++) a[j] = 0.0f;
                        const KT* kr = ks + tt * RE;
#pragma unroll
                        for (int e0 = qt * (HD / 4); e0 < (qt + 1) * (HD / 4); e0 += KV) {
                            float kf[KV];
                            if constexpr (sizeof(KT) == 2) WTraits<__half>::widen(*reinterpret_cast<const uint4*>(kr + e0), kf);
                            else WTraits<float>::widen(*reinterpret_cast<const uint4*>(kr + e0), kf);
#pragma unroll
                            for (int j = 0; j < 8; j++)
                                if (j < G)
#pragma unroll
                                    for (int e = 0; e < KV; e++) a[j] = fmaf(qs[j * HD + e0 + e], kf[e], a[j]);
                        }
#pragma unroll
                        for (int j = 0; j < 8; j++)
                            if (j < G) part[(qt * 8 + j) * 64 + tt] = a[j];
                    }
                }
                named_barrier_sync(1, FS_CT);
                if (warp < G) {  // softmax of head `warp` over the chunk
                    const int j = warp;
                    float s0 = -CUDART_INF_F, s1 = -CUDART_INF_F;
                    if (lane < n)
                        s0 = (part[(0 * 8 + j) * 64 + lane] + part[(1 * 8 + j) * 64 + lane] +
                              part[(2 * 8 + j) * 64 + lane] + part[(3 * 8 + j) * 64 + lane]) * scale;
                    if (lane + 32 < n)
                        s1 = (part[(0 * 8 + j) * 64 + lane + 32] + part[(1 * 8 + j) * 64 + lane + 32] +
                              part[(2 * 8 + j) * 64 + lane + 32] + part[(3 * 8 + j) * 64 + lane + 32]) * scale;
                    const float m = warp_max(fmaxf(s0, s1));
                    const float e0 = lane < n ? expf(s0 - m) : 0.0f;
                    const float e1 = lane + 32 < n ? expf(s1 - m) : 0.0f;
                    pm[j * 64 + lane] = e0;
                    pm[j * 64 + lane + 32] = e1;
                    const float l = warp_sum(e0 + e1);
                    if (lane == 0) {
                        ml[j] = m;
                        ml[8 + j] = l;
                    }
                }
                named_barrier_sync(1, FS_CT);
                {  // P V: thread (e, position set)
                    constexpr int SETS = FS_CT / HD;
                    const int e = ct % HD, set = ct / HD;
                    float a[8];
#pragma unroll
                    for (int j = 0; j < 8; j++) a[j] = 0.0f;
                    for (int tt = set; tt < n; tt += SETS) {
                        const float vv = (float)vs[tt * RE + e];
#pragma unroll
                        for (int j = 0; j < 8; j++)
                            if (j < G) a[j] = fmaf(pm[j * 64 + tt], vv, a[j]);
                    }
#pragma unroll
                    for (int j = 0; j < 8; j++)
                        if (j < G) op[(set * 8 + j) * HD + e] = a[j];
                }
                named_barrier_sync(1, FS_CT);
                for (int i = ct; i < G * HD; i += FS_CT) {
                    constexpr int SETS = FS_CT / HD;
                    const int j = i / HD, e = i % HD;
                    float o = 0.0f;
#pragma unroll
                    for (int sset = 0; sset < SETS; sset++) o += op[(sset * 8 + j) * HD + e];
                    float* w = P.att_ws + (((size_t)b * P.nh + h0 + j) * P.max_chunks + ch) * (HD + 2);
                    w[e] = o;
                    if (e == 0) {
                        w[HD] = ml[j];
                        w[HD + 1] = ml[8 + j];
                    }
                }
                named_barrier_sync(1, FS_CT);  // shared buffers are reused by the next item
            }
        } else if (f.kind == FS_ATTN_COMBINE) {
            // one warp per (sequence, head): lanes own HD/32 output elements; chunk partials
            // are read four at a time so their loads overlap
            constexpr int EPL = HD / 32;
            const int n_items = B * P.nh;
            for (int item = blockIdx.x + gridDim.x * warp; item < n_items; item += gridDim.x * FS_NCW) {
                const int b = item / P.nh, h = item % P.nh;
                const int len = min(__ldcg(P.pos + b) + 1, min(P.max_seq, P.max_pages * P.page_size));
                const int nc = min(P.max_chunks, (len + 63) / 64);
                const float* w = P.att_ws + ((size_t)b * P.nh + h) * P.max_chunks * (HD + 2);
                float M = -CUDART_INF_F;
                for (int c = lane; c < nc; c += 32) M = fmaxf(M, __ldcg(w + (size_t)c * (HD + 2) + HD));
                M = warp_max(M);
                float L = 0.0f, o[EPL];
#pragma unroll
                for (int i = 0; i < EPL; i++) o[i] = 0.0f;
#pragma unroll 4
                for (int c = 0; c < nc; c++) {
                    const float* wc = w + (size_t)c * (HD + 2);
                    const float sc = expf(__ldcg(wc + HD) - M);
                    L += __ldcg(wc + HD + 1) * sc;
#pragma unroll
                    for (int i = 0; i < EPL; i++) o[i] += __ldcg(wc + lane + 32 * i) * sc;
                }
#pragma unroll
                for (int i = 0; i < EPL; i++) P.attn[((size_t)b * P.nh + h) * HD + lane + 32 * i] = o[i] / L;
            }
        } else if (f.kind == FS_FINAL) {
            // token bookkeeping: sampled id, next input (forced or sampled), log, positions
            if (blockIdx.x == 0) {
                if (ct < B) {
                    const int b = ct;
                    const unsigned long long sl = __ldcg(P.slots + b);
                    const int32_t sampled = sl ? (int32_t)unpack_argmax_idx(sl) : 0;
                    if (steps_now < P.log_cap) P.log[(size_t)steps_now * B + b] = sampled;
                    P.sampled[b] = sampled;
                    const int nf = *P.n_forced;
                    P.ids[b] = (steps_now + 1 < nf) ? P.forced[(size_t)(steps_now + 1) * B + b] : sampled;
                    const int np = P.pos[b] + 1;
                    if (np > P.max_seq) set_status(P.status, VSL_ERR_BOUNDS);
                    P.pos[b] = np < P.max_seq ? np : P.max_seq;
                }
                named_barrier_sync(1, FS_CT);
                if (ct == 0) {
                    *P.step = steps_now + 1;
                    *P.bar_epoch = s_base + (unsigned long long)P.n_barriers * gridDim.x;
                }
            }
            continue;  // last phase: no barrier
        }
        if (!grid_sync()) return;
        if (P.trace && blockIdx.x == 0 && ct == 0) P.trace[ph + 1] = globaltimer_ns();
    }
}

// ---------------------------------------------------------------------------------------
// host launch
// ---------------------------------------------------------------------------------------
template <typename WT, typename KT, int HD>
static int launch_fs(const FsProgram& prog, int grid, cudaStream_t st) {
    auto kern = vsl_fused_step_kernel<WT, KT, HD>;
    static thread_local int configured_dev = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (configured_dev != dev) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)FS_DYN_SMEM);
        if (e != cudaSuccess) return launch_status(e, "fused step smem attribute");
        int occ = 0;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, FS_THREADS, FS_DYN_SMEM);
        if (e != cudaSuccess) return launch_status(e, "fused step occupancy");
        if (occ < 1) return set_error(VSL_ERR_UNSUPPORTED, "fused step: one CTA does not fit on an SM");
        configured_dev = dev;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(FS_THREADS);
    cfg.dynamicSmemBytes = FS_DYN_SMEM;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return launch_status(cudaLaunchKernelEx(&cfg, kern, prog), "fused step launch");
}

int fused_step_launch(const FsProgram& prog, int grid, cudaStream_t st) {
    if (prog.B < 1 || prog.B > FS_BMAX) return set_error(VSL_ERR_UNSUPPORTED, "fused step: batch %d", prog.B);
    const bool kv16 = prog.kvdtype == VSL_F16;
    if (prog.kvdtype != VSL_F16 && prog.kvdtype != VSL_F32)
        return set_error(VSL_ERR_UNSUPPORTED, "fused step: kv dtype %d", prog.kvdtype);
    // fp32 keys/values of 128-wide heads do not fit the 64 KB attention staging area
#define FS_DISPATCH(WT)                                                                         \
    if (prog.hd == 128 && kv16) return launch_fs<WT, __half, 128>(prog, grid, st);             \
    if (prog.hd == 64) return kv16 ? launch_fs<WT, __half, 64>(prog, grid, st) : launch_fs<WT, float, 64>(prog, grid, st);
    switch (prog.wdtype) {
        case VSL_F16: FS_DISPATCH(__half) break;
        case VSL_BF16: FS_DISPATCH(__nv_bfloat16) break;
        case VSL_F32: FS_DISPATCH(float) break;
        default: break;
    }
#undef FS_DISPATCH
    return set_error(VSL_ERR_UNSUPPORTED, "fused step: weight dtype %d / head_dim %d", prog.wdtype, prog.hd);
}

// Largest cooperative grid: one CTA per SM.
int fused_step_max_grid(int* grid) {
    *grid = sm_count();
    return VSL_OK;
}

}  // namespace vsl
