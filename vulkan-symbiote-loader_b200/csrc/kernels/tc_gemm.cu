// Batched decode projections on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// For batch sizes where a projection y = x·Wᵀ stops being a pure weight stream (B > 4 rows
// of activations), the GEMV kernels would re-stream W once per 4 rows. Here every weight
// tile is read from HBM once and multiplied against all B rows on the tensor cores:
//   D[128 rows of W][2·Bp] = W_tile[128][K] · X2[2·Bp][K]ᵀ        (kind::f16, fp32 accumulate)
// tcgen05 wants both operands in the same 16-bit type, so the fp32 activations are split
// once per projection into x = hi + lo with hi = rn(x), lo = rn(x - hi) in the weight's type
// (X2 = [hi rows; lo rows]); the epilogue adds the two accumulator columns of each row. The
// products of 16-bit values are exact in fp32, so the result matches an fp32-activation GEMV
// to within the ~2^-22 (fp16) / 2^-16 (bf16) relative size of the dropped remainder.
//
// CTA roles (192 threads, one CTA per SM, persistent over a stream-K share of the work):
//   warp 0     TMA producer: W tile (128 x 64, 128-byte swizzle) and X2 tile (2Bp x 64) per
//              k-block into a ring of shared-memory stages (mbarrier complete_tx);
//   warp 1     allocates two TMEM accumulators (2Bp fp32 columns x 128 lanes each, so the
//              MMAs of one segment overlap the epilogue of the previous one) and one lane
//              issues tcgen05.mma (M=128, N=2Bp, K=16; 8 per k-block), committing each stage
//              back to the producer and each finished segment to the epilogue;
//   warps 2-9  epilogue, two warps per TMEM lane quarter on alternate 16-column chunks of the
//              batch: tcgen05.ld of their 32 TMEM lanes (= rows), hi + lo, then either the
//              projection epilogue directly (a segment that covers all of K) or a partial to
//              the workspace plus an arrival on the row tile's counter.
// Split row tiles: at 32 or more activation rows, when each row tile is shared by two or
// more CTAs, they are finished by all of their CTAs together: after its own stream, each contributing CTA waits (bounded) until every
// contributor of the tile has arrived, then sums the partials of its own 1/s share of the
// batch rows in CTA order (deterministic) and runs the epilogue for them. The grid never
// exceeds the SM count and a CTA fills an SM, so all contributors are resident together; a
// CTA waits only after all of its own MMAs are done. Otherwise the sum is short, and the last
// CTA to arrive sums all rows (same order) while the others leave.
// Work split (stream-K): the flattened sequence of (row tile, k-block) pairs is cut into
// gridDim.x equal ranges, one per CTA, so every SM streams the same number of weight bytes.
// Every wait is bounded (one second); on expiry the kernel records VSL_ERR_TIMEOUT, lets its
// copies and MMAs drain (bounded again), frees its TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "epilogue.cuh"
#include "launch.cuh"
#include "tc_gemm.h"
#include "trace.cuh"

VSL_TRACE_UNIT(tc)

namespace vsl {

constexpr int TC_EPI_WARPS = 8;  // two per TMEM lane quarter, each on alternate 16-row chunks of the batch
constexpr int TC_EPI_THREADS = 32 * TC_EPI_WARPS;
constexpr int TC_THREADS = 64 + TC_EPI_THREADS;
constexpr int TC_BM = 128;            // rows of W per tile (MMA M)
constexpr int TC_ATOM = 64;           // k per 128-byte swizzle atom of 16-bit values
constexpr int TC_A_ATOM = TC_BM * TC_ATOM * 2;   // 16 KB of weights per atom
// A stage (one k-block) holds KA atoms of W and of X2: two (128 k) for up to TC_KA1_ROWS - 1
// padded activation rows, one (64 k) from there on, where the X2 tile (2 x 64 B per k) is large
// enough that finer, deeper stages overlap copies and MMAs better.
#ifndef VSL_TC_KA1_ROWS
#define VSL_TC_KA1_ROWS 96
#endif
constexpr int TC_KA1_ROWS = VSL_TC_KA1_ROWS;
// From this many activation rows on, the grid is always one CTA per SM (stream-K), since the
// MMA work of a whole row tile per CTA would outlast its weight stream.
#ifndef VSL_TC_SK_ROWS
#define VSL_TC_SK_ROWS 1024
#endif
constexpr int TC_SK_ROWS = VSL_TC_SK_ROWS;
constexpr int TC_MAX_STAGES = 12;
constexpr int TC_SMEM_BUDGET = 200 * 1024;     // ring bytes (+1 KB alignment slack)

struct TcArgs {
    int N, K, B, Bp;     // rows, inner dimension, batch, batch padded to a multiple of 8
    int n_rt, nkb;       // row tiles, k-blocks
    long long T;         // n_rt * nkb
    int stages, stage_bytes, b_atom, b_bytes;  // X2 bytes per atom and per stage
    uint32_t idesc;      // tcgen05 instruction descriptor
    int tmem_cols;       // columns of one accumulator (two are allocated)
    int dist_fixup;      // split tiles finished by all contributors (else by the last to arrive)
    float* ws;           // [gridDim.x][2][Bp][128] split-tile partials
    int* counters;       // [2][n_rt] arrivals and finished fixups per split row tile (zero between launches)
    int* status;         // VSL_ERR_TIMEOUT on an expired wait (nullable)
    GemvParams ep;       // epilogue parameters (y, residual, RoPE/KV, sampler)
};

// ---------------------------------------------------------------------------------------
// PTX wrappers (tcgen05, tensor TMA)
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void tmap_prefetch(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
__device__ __forceinline__ int ld_abort(const int* p) { return *reinterpret_cast<const volatile int*>(p); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor of a K-major tile in the canonical 128-byte-swizzle layout
// (8-row x 128-byte atoms, 1024 bytes apart): start address >> 4 in bits 0-13, leading byte
// offset (unused for this layout, 16) in 16-29, stride byte offset 1024 in 32-45, descriptor
// version 1 in 46-47, swizzle mode 2 (128 B) in 61-63. The tile base is 1024-byte aligned.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)(16 >> 4) << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// arrive on `bar` once every tcgen05.mma issued so far by this thread has completed
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// two 16-column pieces of this warp's 32 TMEM lanes (the hi and lo accumulator columns of
// the same rows), one wait for both
__device__ __forceinline__ void tmem_ld16x2(uint32_t ta, uint32_t tb, float* va, float* vb) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%32];\n\t"
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%33];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(ta), "r"(tb)
        : "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) {
        va[i] = __uint_as_float(r[i]);
        vb[i] = __uint_as_float(r[16 + i]);
    }
}

// ---------------------------------------------------------------------------------------
// stream-K partition: CTA c owns flat k-blocks [lo(c), lo(c+1)), lo(c) = c*T/G
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ long long sk_lo(long long T, int G, int c) { return T * c / G; }
// CTA whose range holds flat k-block f
__device__ __forceinline__ int sk_owner(long long T, int G, long long f) { return (int)(((f + 1) * G - 1) / T); }

struct Segment {
    int rt, kb0, kb1;
    bool full;   // covers all k-blocks of the row tile
    int slot;    // workspace slot of a split segment: 0 = first of this CTA, 1 = last
};

__device__ __forceinline__ bool next_segment(const TcArgs& a, long long& f, long long f1, long long f0, Segment& s) {
    if (f >= f1) return false;
    s.rt = (int)(f / a.nkb);
    s.kb0 = (int)(f - (long long)s.rt * a.nkb);
    const long long rem = f1 - f;
    s.kb1 = (long long)(a.nkb - s.kb0) < rem ? a.nkb : s.kb0 + (int)rem;
    s.full = s.kb0 == 0 && s.kb1 == a.nkb;
    s.slot = f == f0 ? 0 : 1;
    f += s.kb1 - s.kb0;
    return true;
}

// ---------------------------------------------------------------------------------------
// activation split: X2[b] = rn(xn), X2[Bp + b] = rn(xn - X2[b]), xn = RMSNorm(x[b]) or x[b]
// One CTA per row. A row of up to XS_VEC x 1024 values is read once, as float4 per thread and
// step, and kept in registers for both the sum of squares and the split; longer rows are read
// twice. K % 8 == 0 (tc_supported), so rows and their halves stay 16- and 8-byte aligned.
// ---------------------------------------------------------------------------------------
constexpr int XS_VEC = 12;

// norm weights of 4-value group j (any alignment)
__device__ __forceinline__ float4 xs_w4(const float* nw, bool nw4, int j) {
    if (nw4) return __ldg(reinterpret_cast<const float4*>(nw) + j);
    return make_float4(__ldg(nw + 4 * j), __ldg(nw + 4 * j + 1), __ldg(nw + 4 * j + 2), __ldg(nw + 4 * j + 3));
}

template <typename WT>
__device__ __forceinline__ void xs_emit(WT* hi, WT* lo, int j, float4 t, bool norm, float4 w4, float den) {
    float e[4] = {t.x, t.y, t.z, t.w};
    if (norm) {
        const float w[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
        for (int q = 0; q < 4; q++) e[q] = e[q] / den * w[q];  // rms_norm.comp:32-34: x / sqrt(var) * w
    }
    WT h[4], l[4];
#pragma unroll
    for (int q = 0; q < 4; q++) {
        if constexpr (std::is_same<WT, __half>::value) {
            h[q] = __float2half_rn(e[q]);
            l[q] = __float2half_rn(e[q] - __half2float(h[q]));
        } else {
            h[q] = __float2bfloat16_rn(e[q]);
            l[q] = __float2bfloat16_rn(e[q] - __bfloat162float(h[q]));
        }
    }
    *reinterpret_cast<uint2*>(hi + 4 * (size_t)j) = *reinterpret_cast<const uint2*>(h);
    *reinterpret_cast<uint2*>(lo + 4 * (size_t)j) = *reinterpret_cast<const uint2*>(l);
}

template <typename WT>
__global__ void __launch_bounds__(256) vsl_xsplit_kernel(const float* __restrict__ x, int K, const float* __restrict__ nw,
                                                     float eps, int Bp, WT* __restrict__ x2, unsigned trace_id) {
    __shared__ float red[8];
    const int b = blockIdx.x;
    VSL_TRACE_ENTRY();
    const int n4 = K / 4;
    const bool in_regs = n4 <= XS_VEC * 256;
    const bool nw4 = ((uintptr_t)nw & 15) == 0;
    // the norm weights are not written by the previous kernel: requested before its end
    float4 w[XS_VEC];
    if (in_regs && nw) {
#pragma unroll
        for (int i = 0; i < XS_VEC; i++) {
            const int j = threadIdx.x + i * 256;
            if (j < n4) w[i] = xs_w4(nw, nw4, j);
        }
    }
    pdl_wait();
    VSL_TRACE_RELEASED();
    pdl_launch_dependents();
    const float4* xr = reinterpret_cast<const float4*>(x + (size_t)b * K);
    float4 v[XS_VEC];
    float ss = 0.0f;
    if (in_regs) {
#pragma unroll
        for (int i = 0; i < XS_VEC; i++) {
            const int j = threadIdx.x + i * 256;
            v[i] = j < n4 ? __ldcg(xr + j) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
        if (nw) {
#pragma unroll
            for (int i = 0; i < XS_VEC; i++) ss += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
        }
    } else if (nw) {
        for (int j = threadIdx.x; j < n4; j += 256) {
            const float4 t = __ldcg(xr + j);
            ss += t.x * t.x + t.y * t.y + t.z * t.z + t.w * t.w;
        }
    }
    float den = 1.0f;
    if (nw) {
        ss = warp_sum(ss);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
        __syncthreads();
        float s = 0.0f;
#pragma unroll
        for (int w = 0; w < 8; w++) s += red[w];
        den = sqrtf(s / (float)K + eps);
    }
    WT* hi = x2 + (size_t)b * K;
    WT* lo = x2 + (size_t)(Bp + b) * K;
    const float4 one = make_float4(1.0f, 1.0f, 1.0f, 1.0f);
    if (in_regs) {
#pragma unroll
        for (int i = 0; i < XS_VEC; i++) {
            const int j = threadIdx.x + i * 256;
            if (j < n4) xs_emit(hi, lo, j, v[i], nw != nullptr, nw ? w[i] : one, den);
        }
    } else {
        for (int j = threadIdx.x; j < n4; j += 256)
            xs_emit(hi, lo, j, __ldcg(xr + j), nw != nullptr, nw ? xs_w4(nw, nw4, j) : one, den);
    }
    VSL_TRACE_EXIT(trace_id, 2100u);
}

// ---------------------------------------------------------------------------------------
// the GEMM
// ---------------------------------------------------------------------------------------
// Epilogue of up to TC_EB activation rows b0.. for this thread's weight row: v[j] is the
// finished sum for row `row`, sequence b0 + j. Rows pair up within a warp (lane parity = row
// parity) and both lanes of a pair work on the pair: the even lane on the chunk's first TC_EB/2
// sequences, the odd lane on the rest, each given its partner's sums by one shuffle per
// sequence. The positions and KV pages of the sequences (EK_QKV) come from shared memory, staged
// once per CTA; the remaining global inputs of the half-chunk (residuals, RoPE terms) are
// requested before any is used, so a half-chunk costs one memory round trip.
constexpr int TC_EB = 16;
constexpr int TC_EH = TC_EB / 2;

// Global inputs of a chunk's epilogue for this lane's half of the sequences (residual pair or
// RoPE terms; positions and pages stay in shared memory until the epilogue applies).
struct TcPre {
    float a0, a1;
};
template <int EK>
__device__ __forceinline__ void tc_epi_fetch(const TcArgs& a, const int* s_pos, const int* s_page, int b0, int b_end,
                                             int row, TcPre* pre) {
    const int lane = threadIdx.x & 31;
    const int r0 = row & ~1;  // the pair's first row
    const int jb = (lane & 1) ? TC_EH : 0;
    const int nb = b_end - b0 < TC_EB ? b_end - b0 : TC_EB;
    const bool has1 = r0 + 1 < a.N;
    if (r0 >= a.N) return;
    if constexpr (EK == EK_QKV) {
        // RoPE terms of the pair at each sequence's position (q and k rows only); the table row
        // of a position comes staged from shared memory
        const int hd = a.ep.head_dim;
        if (r0 >= (a.ep.n_heads + a.ep.n_kv) * hd) return;
        const int rc = (r0 % hd) >> 1;
#pragma unroll
        for (int i = 0; i < TC_EH; i++) {
            const int b = b0 + jb + i;
            if (jb + i < nb && s_page[b] >= 0) {
                const size_t t = (size_t)s_pos[b] + rc;  // s_pos holds pos * head_dim / 2 here
                pre[i] = TcPre{__ldg(a.ep.rope_cos + t), __ldg(a.ep.rope_sin + t)};
            }
        }
        return;
    }
#pragma unroll
    for (int i = 0; i < TC_EH; i++) {
        if (jb + i < nb) {
            const int b = b0 + jb + i;
            int pos = 0, page = 0;
            if (EK == EK_QKV) {
                pos = s_pos[b];
                page = s_page[b];
            }
            const EpiPre e = epi_fetch<EK>(a.ep, b, r0, has1, pos, page);
            pre[i] = TcPre{e.a0, e.a1};
        }
    }
}

// The epilogue of a chunk given its fetched inputs.
template <int EK>
__device__ __forceinline__ void tc_epi_apply(const TcArgs& a, const int* s_pos, const int* s_page, const int* s_kvrow,
                                             int b0, int b_end, int row, const float* v, const TcPre* pre, int step) {
    const int lane = threadIdx.x & 31;
    const bool odd = lane & 1;
    const int r0 = row & ~1;
    // own[i] / mate[i]: this lane's and its partner's sums for sequence b0 + jb + i
    float own[TC_EH], mate[TC_EH];
#pragma unroll
    for (int i = 0; i < TC_EH; i++) {
        own[i] = odd ? v[TC_EH + i] : v[i];
        mate[i] = __shfl_xor_sync(0xffffffffu, odd ? v[i] : v[TC_EH + i], 1);
    }
    const int jb = odd ? TC_EH : 0;
    const bool act = r0 < a.N;
    const bool has1 = r0 + 1 < a.N;
    const int nb = b_end - b0 < TC_EB ? b_end - b0 : TC_EB;
    if constexpr (EK == EK_QKV) {
        // q rows: rotated pair into q_out; k rows: rotated pair, v rows: as is, into the
        // sequence's KV page (s_page: page, -1 outside the cache; s_kvrow: the row of KV group 0
        // for the position)
        if (!act) return;
        const GemvParams& p = a.ep;
        const int hd = p.head_dim, qd = p.n_heads * hd, kvd = p.n_kv * hd;
        const int el = r0 % hd;
        const bool is_q = r0 < qd, is_v = r0 >= qd + kvd;
        const int g = is_q ? 0 : (is_v ? r0 - qd - kvd : r0 - qd) / hd;
        void* cache = is_v ? p.v_cache : p.k_cache;
#pragma unroll
        for (int i = 0; i < TC_EH; i++) {
            if (jb + i >= nb) continue;
            const int b = b0 + jb + i;
            if (s_page[b] < 0) {
                if (p.status) atomicCAS(p.status, 0, VSL_ERR_BOUNDS);
                continue;
            }
            const float s0 = odd ? mate[i] : own[i], s1 = odd ? own[i] : mate[i];
            float o0 = s0, o1 = s1;
            if (!is_v) {  // rotate q and k: adjacent pair (el, el + 1)
                o0 = __fsub_rn(__fmul_rn(s0, pre[i].a0), __fmul_rn(s1, pre[i].a1));
                o1 = __fadd_rn(__fmul_rn(s0, pre[i].a1), __fmul_rn(s1, pre[i].a0));
            }
            if (is_q) {
                *reinterpret_cast<float2*>(p.q_out + (size_t)b * qd + r0) = make_float2(o0, o1);
            } else {
                const size_t idx = ((size_t)s_kvrow[b] + (size_t)g * p.page_size) * hd + el;
                if (p.kvdtype == VSL_F16)
                    *reinterpret_cast<__half2*>(static_cast<__half*>(cache) + idx) = __floats2half2_rn(o0, o1);
                else if (p.kvdtype == VSL_BF16)
                    *reinterpret_cast<__nv_bfloat162*>(static_cast<__nv_bfloat16*>(cache) + idx) =
                        __floats2bfloat162_rn(o0, o1);
                else
                    *reinterpret_cast<float2*>(static_cast<float*>(cache) + idx) = make_float2(o0, o1);
            }
        }
        return;
    }
    unsigned long long best[EK == EK_LMHEAD ? TC_EH : 1];
#pragma unroll
    for (int i = 0; i < (EK == EK_LMHEAD ? TC_EH : 1); i++) best[i] = 0ull;
    if (act) {
#pragma unroll
        for (int i = 0; i < TC_EH; i++) {
            if (jb + i < nb) {
                unsigned long long bb = 0ull;
                const float s0 = odd ? mate[i] : own[i], s1 = odd ? own[i] : mate[i];
                const int b = b0 + jb + i;
                const EpiPre e = {pre[i].a0, pre[i].a1, EK == EK_QKV ? s_pos[b] : 0, EK == EK_QKV ? s_page[b] : 0};
                epi_apply<EK>(a.ep, e, b, r0, r0 >> 1, has1, s0, s1, bb, step);
                if (EK == EK_LMHEAD) best[EK == EK_LMHEAD ? i : 0] = bb;
            }
        }
    }
    if (EK == EK_LMHEAD) {
        // sequence b0 + jb + i: the maximum over the lanes of this parity
#pragma unroll
        for (int i = 0; i < TC_EH; i++) {
            unsigned long long bb = best[EK == EK_LMHEAD ? i : 0];
#pragma unroll
            for (int o = 16; o > 1; o >>= 1) {
                const unsigned long long t = __shfl_xor_sync(0xffffffffu, bb, o);
                bb = t > bb ? t : bb;
            }
            if (lane < 2 && bb && jb + i < nb) atomicMax(a.ep.slots + b0 + jb + i, bb);
        }
    }
}

template <int EK>
__device__ __forceinline__ void tc_epilogue_chunk(const TcArgs& a, const int* s_pos, const int* s_page,
                                                  const int* s_kvrow, int b0, int b_end, int row, const float* v,
                                                  int step) {
    TcPre pre[TC_EH];
    tc_epi_fetch<EK>(a, s_pos, s_page, b0, b_end, row, pre);
    tc_epi_apply<EK>(a, s_pos, s_page, s_kvrow, b0, b_end, row, v, pre, step);
}

// Sum of the partials of split row tile rt from CTAs first..lastc (in CTA order: the result
// does not depend on arrival order) for activation rows [bs0, bs1), then the epilogue.
template <int EK>
__device__ __forceinline__ void tc_fixup_rows(const TcArgs& a, const int* s_pos, const int* s_page, const int* s_kvrow,
                                              int G, int rt, int first, int lastc, int bs0, int bs1, int row, int rloc,
                                              int step, int hb) {
    for (int b0 = bs0 + hb * TC_EB; b0 < bs1; b0 += 2 * TC_EB) {
        // TC_EB rows x 2 CTAs of loads are in flight per thread (two warps share each row)
        float v[TC_EB];
#pragma unroll
        for (int j = 0; j < TC_EB; j++) v[j] = 0.0f;
        for (int c0 = first; c0 <= lastc; c0 += 2) {
            float t[2][TC_EB];
#pragma unroll
            for (int u = 0; u < 2; u++) {
                const int cc = c0 + u;
                if (cc <= lastc) {
                    const int slot = sk_lo(a.T, G, cc) >= (long long)rt * a.nkb ? 0 : 1;
                    const float* src = a.ws + (((size_t)cc * 2 + slot) * a.Bp + b0) * TC_BM + rloc;
#pragma unroll
                    for (int j = 0; j < TC_EB; j++) t[u][j] = b0 + j < bs1 ? __ldcg(src + (size_t)j * TC_BM) : 0.0f;
                }
            }
#pragma unroll
            for (int u = 0; u < 2; u++)
                if (c0 + u <= lastc)
#pragma unroll
                    for (int j = 0; j < TC_EB; j++) v[j] += t[u][j];
        }
        tc_epilogue_chunk<EK>(a, s_pos, s_page, s_kvrow, b0, bs1, row, v, step);
    }
}

template <int EK, int KA>
__global__ void __launch_bounds__(TC_THREADS, 1)
    vsl_tc_gemm_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x,
                   const __grid_constant__ TcArgs a) {
    extern __shared__ unsigned char smem_raw[];
    __shared__ __align__(8) uint64_t full[TC_MAX_STAGES], empty[TC_MAX_STAGES];
    __shared__ __align__(8) uint64_t tmem_full[2], tmem_empty[2];
    __shared__ uint32_t tmem_base_s;
    __shared__ int abort_s;
    __shared__ int last_s;
    // EK_QKV, per sequence: RoPE table row (pos * head_dim / 2), KV page (-1: outside the cache)
    // and the cache row of KV group 0 at the position
    __shared__ int s_pos[EK == EK_QKV ? TC_MAX_BATCH : 1], s_page[EK == EK_QKV ? TC_MAX_BATCH : 1],
        s_kvrow[EK == EK_QKV ? TC_MAX_BATCH : 1];

    VSL_TRACE_ENTRY();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t ring = (smem_u32(smem_raw) + 1023u) & ~1023u;
    const int G = gridDim.x, c = blockIdx.x;
    const long long f0 = sk_lo(a.T, G, c), f1 = sk_lo(a.T, G, c + 1);
    const int S = a.stages;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&tmem_full[i], 1);
            mbar_init(&tmem_empty[i], TC_EPI_WARPS);
        }
        mbar_fence_init();
        abort_s = 0;
        tmap_prefetch(&map_w);
        tmap_prefetch(&map_x);
    }
    if (warp == 1) {  // two TMEM accumulators: 128 lanes x tmem_cols fp32 columns each
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_s)),
                     "r"(2 * a.tmem_cols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base_s;

    if (warp == 0) {
        // ================= producer =================
        if (lane == 0) {
            const uint32_t tx = (uint32_t)(TC_A_ATOM * KA + a.b_bytes);
            long long it = 0;
            // weights do not depend on the previous kernel: the first stages' W tiles are
            // requested before griddepcontrol.wait, their X2 tiles after it
            long long f = f0;
            Segment sg;
            int pre = 0;
            {
                long long g = f0;
                Segment s2;
                while (pre < S && next_segment(a, g, f1, f0, s2))
                    for (int kb = s2.kb0; kb < s2.kb1 && pre < S; kb++, pre++) {
                        mbar_arrive_expect_tx(&full[pre], tx);
#pragma unroll
                        for (int at = 0; at < KA; at++)
                            tma_load_2d(ring + pre * a.stage_bytes + at * TC_A_ATOM, &map_w, (kb * KA + at) * TC_ATOM,
                                        s2.rt * TC_BM, &full[pre]);
                    }
            }
            pdl_wait();
            VSL_TRACE_RELEASED();
            pdl_launch_dependents();
            bool ok = true;
            // stage index and the parity of its empty-barrier phase advance incrementally (a
            // 64-bit division per k-block costs more issue slots than the rest of the loop)
            int s = 0;
            uint32_t epar = 1u;  // the first lap finds every stage free
            while (ok && next_segment(a, f, f1, f0, sg)) {
                for (int kb = sg.kb0; kb < sg.kb1; kb++, it++) {
                    if (it >= pre) {
                        if (it >= S && !mbar_wait(&empty[s], epar)) {
                            ok = false;
                            break;
                        }
                        mbar_arrive_expect_tx(&full[s], tx);
#pragma unroll
                        for (int at = 0; at < KA; at++)
                            tma_load_2d(ring + s * a.stage_bytes + at * TC_A_ATOM, &map_w, (kb * KA + at) * TC_ATOM,
                                        sg.rt * TC_BM, &full[s]);
                    }
#pragma unroll
                    for (int at = 0; at < KA; at++)
                        tma_load_2d(ring + s * a.stage_bytes + TC_A_ATOM * KA + at * a.b_atom, &map_x,
                                    (kb * KA + at) * TC_ATOM, 0, &full[s]);
                    if (++s == S) {
                        s = 0;
                        epar ^= 1u;
                    }
                }
            }
            if (!ok) {
                set_status(a.status, VSL_ERR_TIMEOUT);
                atomicExch(&abort_s, 1);
            }
            // every copy issued must land before the CTA may exit
            const long long issued = it > pre ? it : pre;
            for (long long u = issued > S ? issued - S : 0; u < issued; u++) mbar_wait(&full[u % S], (uint32_t)((u / S) & 1));
        }
    } else if (warp == 1) {
        // ================= MMA issuer =================
        if (lane == 0) {
            pdl_wait();
            pdl_launch_dependents();
            long long f = f0, it = 0;
            int si = 0, s = 0;
            uint32_t fpar = 0u;
            Segment sg;
            bool ok = true;
            bool committed = false;
            while (ok && next_segment(a, f, f1, f0, sg)) {
                const int buf = si & 1;
                // accumulator buf was last used by segment si - 2
                if (si >= 2 && !mbar_wait(&tmem_empty[buf], (uint32_t)(((si >> 1) - 1) & 1))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t acc = tmem + (uint32_t)(buf * a.tmem_cols);
                for (int kb = sg.kb0; kb < sg.kb1; kb++, it++) {
                    if (!mbar_wait(&full[s], fpar) || (((int)it & 15) == 0 && ld_abort(&abort_s))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = ring + s * a.stage_bytes, sb = sa + TC_A_ATOM * KA;
#pragma unroll
                    for (int at = 0; at < KA; at++) {
                        const uint64_t ad = sw128_desc(sa + at * TC_A_ATOM), bd = sw128_desc(sb + at * a.b_atom);
#pragma unroll
                        for (int k = 0; k < TC_ATOM / 16; k++)  // +32 bytes per 16 values inside the atom
                            tc_mma(acc, ad + (uint64_t)(2 * k), bd + (uint64_t)(2 * k), a.idesc,
                                   (kb > sg.kb0 || at > 0 || k > 0) ? 1u : 0u);
                    }
                    tc_commit(&empty[s]);  // frees the stage once these MMAs have read it
                    if (++s == S) {
                        s = 0;
                        fpar ^= 1u;
                    }
                }
                if (!ok) break;
                tc_commit(&tmem_full[buf]);
                committed = true;
                si++;
            }
            if (!ok) {
                set_status(a.status, VSL_ERR_TIMEOUT);
                atomicExch(&abort_s, 1);
            }
            // the accumulator must not be freed under a running MMA
            if (committed) mbar_wait(&tmem_full[(si - 1) & 1], (uint32_t)(((si - 1) >> 1) & 1));
        }
        __syncwarp();
    } else {
        // ================= epilogue warps =================
        pdl_wait();
        pdl_launch_dependents();
        const int q = warp & 3;          // TMEM lane quarter this warp may access
        const int hb = (warp - 2) >> 2;  // chunks b0 = 16 (2 j + hb) of the batch
        const int rloc = q * 32 + lane;
        const int et = threadIdx.x - 64;  // 0..TC_EPI_THREADS - 1
        int step = 0;
        if (EK == EK_LMHEAD && a.ep.inv_temp > 0.0f) step = *a.ep.step_counter;
        if (EK == EK_QKV) {  // positions and KV pages of the sequences, once per CTA
            for (int b = et; b < a.B; b += TC_EPI_THREADS) {
                int pos, page;
                epi_pos_page(a.ep, b, pos, page);
                s_pos[b] = pos * (a.ep.head_dim >> 1);
                s_page[b] = page;
                s_kvrow[b] = page < 0 ? 0 : page * a.ep.n_kv * a.ep.page_size + pos % a.ep.page_size;
            }
            named_barrier_sync(1, TC_EPI_THREADS);
        }
        long long f = f0;
        int si = 0;
        Segment sg;
        int n_split = 0, split_rt[2] = {0, 0};  // split tiles of this CTA: only its first and last segment
        bool aborted = false;
        while (next_segment(a, f, f1, f0, sg)) {
            const int buf = si & 1;
            {
                // the epilogue warps leave together (they meet at named barriers below)
                const bool bad = !mbar_wait(&tmem_full[buf], (uint32_t)((si >> 1) & 1)) || ld_abort(&abort_s);
                if (named_barrier_or(1, TC_EPI_THREADS, bad)) {
                    set_status(a.status, VSL_ERR_TIMEOUT);
                    atomicExch(&abort_s, 1);
                    aborted = true;
                    break;
                }
            }
            tc_fence_after();
#ifdef VSL_TRACE
            const uint64_t te0 = vsl::trace_now();
#endif
            const int row = sg.rt * TC_BM + rloc;
            float* wsp = a.ws + ((size_t)c * 2 + sg.slot) * a.Bp * TC_BM;
            const uint32_t tl = tmem + (uint32_t)(buf * a.tmem_cols) + ((uint32_t)(q * 32) << 16);
            for (int b0 = hb * TC_EB; b0 < a.B; b0 += 2 * TC_EB) {
                float hi[TC_EB], lo[TC_EB];
                tmem_ld16x2(tl + (uint32_t)b0, tl + (uint32_t)(a.Bp + b0), hi, lo);
#pragma unroll
                for (int i = 0; i < TC_EB; i++) hi[i] += lo[i];
                if (sg.full) {
                    tc_epilogue_chunk<EK>(a, s_pos, s_page, s_kvrow, b0, a.B, row, hi, step);
                } else {
#pragma unroll
                    for (int i = 0; i < TC_EB; i++)
                        if (b0 + i < a.B) wsp[(size_t)(b0 + i) * TC_BM + rloc] = hi[i];
                }
            }
            // accumulator read: hand TMEM back to the MMA warp
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tmem_empty[buf]);
#ifdef VSL_TRACE
            if (et == 0 && si == 0) vsl_trace_record(a.ep.trace_id, 2090u + EK, te0, vsl::trace_now());
#endif
            si++;
            if (!sg.full) {
                // partial written: arrive on the row tile (release after the CTA's stores)
                __threadfence();
                named_barrier_sync(1, TC_EPI_THREADS);
                if (a.dist_fixup) {
                    if (et == 0) atomicAdd(a.counters + sg.rt, 1);
                    split_rt[n_split++] = sg.rt;
                } else {
                    const int first = sk_owner(a.T, G, (long long)sg.rt * a.nkb);
                    const int lastc = sk_owner(a.T, G, (long long)sg.rt * a.nkb + a.nkb - 1);
                    if (et == 0) last_s = atomicAdd(a.counters + sg.rt, 1) == lastc - first ? 1 : 0;
                    named_barrier_sync(1, TC_EPI_THREADS);
                    if (last_s) {
                        __threadfence();
                        tc_fixup_rows<EK>(a, s_pos, s_page, s_kvrow, G, sg.rt, first, lastc, 0, a.B, row, rloc, step, hb);
                        if (et == 0) a.counters[sg.rt] = 0;
                    }
                }
            }
        }
        // fixup of the split tiles: contributor k of s sums batch rows [B k / s, B (k + 1) / s)
        for (int i = 0; i < n_split && !aborted; i++) {
            const int rt = split_rt[i];
            const int first = sk_owner(a.T, G, (long long)rt * a.nkb);
            const int lastc = sk_owner(a.T, G, (long long)rt * a.nkb + a.nkb - 1);
            const int ns = lastc - first + 1, k = c - first;
            bool bad = false;
            if (et == 0) {
                const volatile int* cnt = a.counters + rt;
                bool ok = *cnt >= ns;
                if (!ok) {
                    const unsigned long long t0 = globaltimer_ns();
                    while (!ok) {
                        for (int r = 0; r < 32 && !ok; r++) ok = *cnt >= ns;
                        if (!ok && (globaltimer_ns() - t0 > WAIT_LIMIT_NS || ld_abort(&abort_s))) break;
                    }
                }
                bad = !ok;
            }
            if (named_barrier_or(1, TC_EPI_THREADS, bad)) {
                set_status(a.status, VSL_ERR_TIMEOUT);
                atomicExch(&abort_s, 1);
                break;
            }
            __threadfence();
            tc_fixup_rows<EK>(a, s_pos, s_page, s_kvrow, G, rt, first, lastc, (int)((long long)a.B * k / ns),
                              (int)((long long)a.B * (k + 1) / ns), rt * TC_BM + rloc, rloc, step, hb);
            // the last contributor through here clears the tile's counters for the next launch
            // (every contributor has seen all arrivals by now)
            if (et == 0) {
                const int prev = atomicAdd(a.counters + a.n_rt + rt, 1);
                if (prev == ns - 1) {
                    a.counters[rt] = 0;
                    a.counters[a.n_rt + rt] = 0;
                }
            }
        }
    }

    // ---- teardown: the allocating warp frees TMEM once every role is done with it ----
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * a.tmem_cols)
                     : "memory");
    }
    VSL_TRACE_EXIT(a.ep.trace_id, (unsigned)(2000 + EK * 10 + KA));
}

// ---------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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

// 2-D tensor map over a row-major [rows][cols] 16-bit matrix, box = box_rows x 64 columns,
// 128-byte swizzle (the canonical K-major tcgen05 operand layout), zero fill out of bounds.
static int make_map(CUtensorMap* m, const void* base, int wdtype, int rows, int cols, int box_rows) {
    auto fn = encode_fn();
    if (!fn) return set_error(VSL_ERR_CUDA, "tensor-map encoder unavailable from the driver");
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    const cuuint32_t box[2] = {(cuuint32_t)TC_ATOM, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(m, wdtype == VSL_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                    const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(VSL_ERR_INVALID, "tensor map encode failed (%d) rows=%d cols=%d", (int)r, rows, cols);
    return VSL_OK;
}

static int pad_batch(int B) { return (B + 7) / 8 * 8; }
size_t tc_split_rows(int B) { return (size_t)pad_batch(B); }

size_t tc_workspace_bytes(int N, int K, int B) {
    const int Bp = pad_batch(B);
    const int G = sm_count();
    const size_t x2 = (size_t)2 * Bp * K * 2;
    const size_t ws = (size_t)G * 2 * Bp * TC_BM * sizeof(float);
    const size_t cnt = (size_t)2 * ((N + TC_BM - 1) / TC_BM) * sizeof(int);
    auto up = [](size_t v) { return (v + 1023) / 1024 * 1024; };
    return up(x2) + up(ws) + up(cnt);
}

bool tc_supported(int wdtype, int N, int K, int B) {
    // shapes at least one tile in each direction (TMA boxes are 128 rows x 64 columns) and
    // 16-byte row pitches (tensor-map strides)
    return (wdtype == VSL_F16 || wdtype == VSL_BF16) && B >= 1 && B <= TC_MAX_BATCH && N >= TC_BM && K >= TC_ATOM &&
           (K % 8) == 0;
}

template <int EK, int KA>
static int launch_tc(const TcArgs& a, const CUtensorMap& mw, const CUtensorMap& mx, int grid, size_t smem,
                     cudaStream_t st) {
    auto kern = vsl_tc_gemm_kernel<EK, KA>;
    static thread_local int configured_dev = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (configured_dev != dev) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             TC_SMEM_BUDGET + 1024);
        if (e != cudaSuccess) return launch_status(e, "tc gemm smem attribute");
        configured_dev = dev;
    }
    return launch_status(launch_k(kern, dim3(grid), dim3(TC_THREADS), smem, st, mw, mx, a), "tc gemm launch");
}

int tc_project(int wdtype, int kind, const GemvParams& p, void* workspace, size_t ws_bytes, int* status,
               cudaStream_t st) {
    if (!tc_supported(wdtype, p.N, p.K, p.B))
        return set_error(VSL_ERR_UNSUPPORTED, "tc gemm: dtype %d N=%d K=%d B=%d", wdtype, p.N, p.K, p.B);
    if (((uintptr_t)p.W & 15) || ((uintptr_t)p.x & 15))
        return set_error(VSL_ERR_INVALID, "tc gemm: weights and activations must be 16-byte aligned");
    const size_t need = tc_workspace_bytes(p.N, p.K, p.B);
    if (!workspace || ws_bytes < need || ((uintptr_t)workspace & 1023))
        return set_error(VSL_ERR_INVALID, "tc gemm: workspace of %zu bytes (1 KB aligned) needed", need);

    TcArgs a = {};
    a.N = p.N;
    a.K = p.K;
    a.B = p.B;
    a.Bp = pad_batch(p.B);
    a.n_rt = (p.N + TC_BM - 1) / TC_BM;
    const int ka = a.Bp >= TC_KA1_ROWS ? 1 : 2;
    a.nkb = (p.K + TC_ATOM * ka - 1) / (TC_ATOM * ka);
    a.T = (long long)a.n_rt * a.nkb;
    const int n = 2 * a.Bp;  // MMA N (multiple of 16)
    a.b_atom = n * TC_ATOM * 2;  // n % 16 == 0: a multiple of 2 KB, so every atom stays 1 KB aligned
    a.b_bytes = a.b_atom * ka;
    a.stage_bytes = TC_A_ATOM * ka + a.b_bytes;
    a.stages = TC_SMEM_BUDGET / a.stage_bytes;
    if (a.stages > TC_MAX_STAGES) a.stages = TC_MAX_STAGES;
    a.tmem_cols = 32;
    while (a.tmem_cols < n) a.tmem_cols <<= 1;
    const uint32_t fmt = wdtype == VSL_BF16 ? 1u : 0u;
    // instruction descriptor (kind::f16): D f32 (bits 4-5 = 1), A/B format (bits 7-9, 10-12),
    // both K-major (bits 15, 16 = 0), N >> 3 in bits 17-22, M >> 4 in bits 24-28
    a.idesc = (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(TC_BM >> 4) << 24);

    unsigned char* w8 = static_cast<unsigned char*>(workspace);
    auto up = [](size_t v) { return (v + 1023) / 1024 * 1024; };
    void* x2 = p.x_presplit && p.x2_in ? const_cast<void*>(p.x2_in) : static_cast<void*>(w8);
    if (((uintptr_t)x2 & 15) || (p.x2_out && (kind != EK_SWIGLU || ((uintptr_t)p.x2_out & 15))))
        return set_error(VSL_ERR_INVALID, "tc gemm: split activations must be 16-byte aligned (output: SwiGLU only)");
    const size_t x2b = up((size_t)2 * a.Bp * p.K * 2);
    const int G0 = sm_count();
    a.ws = reinterpret_cast<float*>(w8 + x2b);
    // the arrival counters sit at the tail of the workspace whatever the shape of the call, so
    // calls of different shapes sharing one workspace (sized for the largest N and K together)
    // never write split activations or partials over another shape's counters
    const size_t cnt_bytes = (size_t)2 * a.n_rt * sizeof(int);
    a.counters = reinterpret_cast<int*>(w8 + ((ws_bytes - cnt_bytes) & ~(size_t)1023));
    a.status = status;
    a.ep = p;
    a.ep.status = status;
    a.ep.trace_id = VSL_TRACE_ID();

    // With at most one row tile per SM, the grid is a multiple of the tile count: every tile is
    // split into the same number of k ranges and no CTA straddles two tiles (fewer partial
    // segments and fixups; 12288 x 4096 at 64 rows: 28.6 us on 96 CTAs against 40.2 us on 148).
    // Otherwise stream-K spreads the k-blocks evenly over every SM.
    int grid = G0;
    if (a.n_rt <= G0 && a.Bp < TC_SK_ROWS) grid = a.n_rt * (G0 / a.n_rt);
    if ((long long)grid > a.T) grid = (int)a.T;
    // many contributors per split tile (at least two CTAs per row tile) and a long sum
    a.dist_fixup = a.B >= 32 && 2 * a.n_rt <= grid ? 1 : 0;

    CUtensorMap mw, mx;
    int rc = make_map(&mw, p.W, wdtype, p.N, p.K, TC_BM);
    if (rc) return rc;
    rc = make_map(&mx, x2, wdtype, n, p.K, n);
    if (rc) return rc;

    // activation split (+ RMSNorm), unless the producing kernel wrote the split tile already
    cudaError_t e = cudaSuccess;
    if (p.x_presplit)
        ;
    else if (wdtype == VSL_BF16)
        e = launch_k(vsl_xsplit_kernel<__nv_bfloat16>, dim3(p.B), dim3(256), 0, st, p.x, p.K, p.norm_w, p.eps, a.Bp,
                     static_cast<__nv_bfloat16*>(x2), (unsigned)VSL_TRACE_ID());
    else
        e = launch_k(vsl_xsplit_kernel<__half>, dim3(p.B), dim3(256), 0, st, p.x, p.K, p.norm_w, p.eps, a.Bp,
                     static_cast<__half*>(x2), (unsigned)VSL_TRACE_ID());
    rc = launch_status(e, "tc activation split");
    if (rc) return rc;

    const size_t smem = (size_t)a.stages * a.stage_bytes + 1024;
    switch (kind) {
        case EK_STORE:
            return ka == 1 ? launch_tc<EK_STORE, 1>(a, mw, mx, grid, smem, st)
                           : launch_tc<EK_STORE, 2>(a, mw, mx, grid, smem, st);
        case EK_ADD:
            return ka == 1 ? launch_tc<EK_ADD, 1>(a, mw, mx, grid, smem, st)
                           : launch_tc<EK_ADD, 2>(a, mw, mx, grid, smem, st);
        case EK_SWIGLU:
            return ka == 1 ? launch_tc<EK_SWIGLU, 1>(a, mw, mx, grid, smem, st)
                           : launch_tc<EK_SWIGLU, 2>(a, mw, mx, grid, smem, st);
        case EK_QKV:
            return ka == 1 ? launch_tc<EK_QKV, 1>(a, mw, mx, grid, smem, st)
                           : launch_tc<EK_QKV, 2>(a, mw, mx, grid, smem, st);
        default:
            return ka == 1 ? launch_tc<EK_LMHEAD, 1>(a, mw, mx, grid, smem, st)
                           : launch_tc<EK_LMHEAD, 2>(a, mw, mx, grid, smem, st);
    }
}

}  // namespace vsl

using namespace vsl;

extern "C" int vsl_skinny_gemm_tc_workspace_size(int N, int K, int B, size_t* bytes) {
    if (!bytes || N <= 0 || K <= 0 || B <= 0 || B > TC_MAX_BATCH)
        return set_error(VSL_ERR_INVALID, "tc workspace: bad shape N=%d K=%d B=%d", N, K, B);
    *bytes = tc_workspace_bytes(N, K, B);
    return VSL_OK;
}

extern "C" int vsl_skinny_gemm_tc(int wdtype, const void* W, int N, int K, const float* x, int B, float* y,
                                  int epilogue, const float* norm_w, float eps, void* workspace,
                                  size_t workspace_bytes, void* stream) {
    if (!W || !x || !y) return set_error(VSL_ERR_INVALID, "tc gemm: null pointer");
    if (epilogue != VSL_EPI_STORE && epilogue != VSL_EPI_ADD && epilogue != VSL_EPI_SWIGLU)
        return set_error(VSL_ERR_INVALID, "tc gemm: unknown epilogue %d", epilogue);
    if (epilogue == VSL_EPI_SWIGLU && (N & 1))
        return set_error(VSL_ERR_INVALID, "tc gemm: SwiGLU needs interleaved gate/up rows (N even), N=%d", N);
    GemvParams p = {};
    p.W = W; p.N = N; p.K = K; p.x = x; p.B = B; p.y = y; p.norm_w = norm_w; p.eps = eps;
    const int kind = epilogue == VSL_EPI_ADD ? EK_ADD : epilogue == VSL_EPI_SWIGLU ? EK_SWIGLU : EK_STORE;
    return tc_project(wdtype, kind, p, workspace, workspace_bytes, nullptr, (cudaStream_t)stream);
}
