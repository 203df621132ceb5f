// Prompt attention on tcgen05 tensor cores: one query block per CTA.
//
// A prompt chunk is up to 128 consecutive positions of one sequence whose K and V rows the
// chunk's QKV projection has just appended to the paged cache. Row r (position pos[r]) attends
// causally to positions [first(r), pos[r]] of the cache (first = 0 unless the long-context
// sparse mask applies), with the semantics of the decode kernels (attention.cu, attention_tc.cu;
// reference attention.comp:84-189 run once per prompt token): scores q.k / sqrt(head_dim),
// max-subtracted softmax, probabilities times V. One CTA takes one query head and a block of
// 128 rows, so the K and V of each 128-position chunk are read once for the whole block rather
// than once per row:
//   * S[128 rows][128 positions] = Q2 . K^T (tcgen05.mma kind::f16, M = N = 128, fp32 in TMEM),
//     with the fp32 query split into fp16 hi and lo tiles that accumulate into the same scores
//     (about 22 bits of the query survive);
//   * online softmax (fp32) by 8 warps, two per TMEM lane quarter: a thread takes one query row
//     (its TMEM lane) and half of the chunk's 128 score columns, read with one 64-column TMEM
//     load (the row maximum is combined with the partner warp through shared memory), and
//     writes its half of the row back as fp16 hi/lo tiles P2;
//   * PV[128 rows][128 dims] = P2 . V (V as the MN-major B operand, in place as it lands from
//     TMA) into TMEM; each thread folds its half of the row's dims into fp32 registers with the
//     softmax rescale.
// K and V of a chunk arrive by tensor TMA (two 64-position pages x two 64-column 128-byte-swizzle
// atoms each) into single K and V tiles with their own barriers, so the next chunk's K loads
// while this chunk's softmax runs. The next chunk's scores are issued before this chunk's
// product. Rows past the cache end are zeroed in the V tile before the product (0 x garbage);
// rows of K past the end give scores that the mask drops.
// Roles: warps 0-7 softmax and accumulation (TMEM lane quarter = warp % 4, column half =
// warp / 4), warp 8 TMA producer, warp 9 TMEM allocation and the single-thread MMA issue. Every wait is bounded (one second)
// and records VSL_ERR_TIMEOUT; the kernel then drains its copies and MMAs and frees its TMEM.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <math_constants.h>

#include <climits>
#include <type_traits>

#include "common.cuh"
#include "kv_map.h"
#include "launch.cuh"
#include "trace.cuh"

VSL_TRACE_UNIT(prefill)

// Phase stamps of the trace build: one extra record per CTA and phase, [t0, t1] of the phase
#ifdef VSL_TRACE
#define FP_STAMP(var) const uint64_t var = vsl::trace_now()
#define FP_PHASE(tag, ta, tb) vsl_trace_record(a.trace_id, (tag), (ta), (tb))
#else
#define FP_STAMP(var)
#define FP_PHASE(tag, ta, tb)
#endif

namespace vsl {

constexpr int FP_SM_WARPS = 8;         // softmax warps
constexpr int FP_THREADS = 32 * FP_SM_WARPS + 64;  // + TMA producer, MMA issuer
constexpr int FP_SM_THREADS = 32 * FP_SM_WARPS;
constexpr int FP_ROWS = 128;           // query rows per CTA (MMA M)
constexpr int FP_CHUNK = 128;          // positions per chunk
constexpr int FP_HD = 128;
constexpr int FP_ATOM = 128 * 64 * 2;  // one 64-column swizzle atom of a 128-row tile (16 KB)
constexpr int FP_TILE = 2 * FP_ATOM;   // a 128 x 128 16-bit tile
// shared memory: Q hi, Q lo, K, V, P hi, P lo
constexpr size_t FP_SMEM = 1024 + 6 * (size_t)FP_TILE;
constexpr uint32_t FP_TMEM_COLS = 512;  // S[2] at columns 0 and 128, PV at 256
constexpr int FP_OST = FP_HD + 4;       // fp32 row stride of the staged output (padded, 16-byte aligned)
static_assert((size_t)FP_ROWS * FP_OST * 4 <= 3 * (size_t)FP_TILE, "staged output fits the Q and K tiles");

struct FpArgs {
    const float* q;             // [P][n_heads][128]
    const int32_t* pos;         // [P] positions of the rows
    const int32_t* page_row;    // the sequence's page-table row
    int P, n_heads, n_kv, G, max_len, max_pages, page_size;
    float scale;
    float* out;                 // [P][n_heads][128]
    int* status;
    uint32_t idesc_s;           // Q2 (A, K-major) . K (B, K-major)
    uint32_t idesc_pv;          // P2 (A, K-major) . V (B, MN-major)
    SparseMask sp;
    long long kv_rows;          // rows of the pool's tensor map (n_pages * n_kv * page_size)
    unsigned trace_id;          // launch id of the trace build (unused otherwise)
    void* x2;                   // non-null: write the split activations of the next projection instead of out
    int x2_bf16, x2_rows;       // their type; row of the first lo row
};

// Eight values of row `rb` of the next projection's split activations (hi row rb, lo row
// x2_rows + rb) at columns [k0, k0 + 8), from shared memory, as 16-bit hi and residual lo.
template <typename T>
__device__ __forceinline__ void fp_store_split8(const FpArgs& a, size_t rb, size_t k0, const float* v) {
    const size_t K = (size_t)a.n_heads * FP_HD;
    const float4 v0 = *reinterpret_cast<const float4*>(v), v1 = *reinterpret_cast<const float4*>(v + 4);
    const float x[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    T h[8], l[8];
#pragma unroll
    for (int e = 0; e < 8; e++) {
        if constexpr (std::is_same<T, __half>::value) {
            h[e] = __float2half_rn(x[e]);
            l[e] = __float2half_rn(x[e] - __half2float(h[e]));
        } else {
            h[e] = __float2bfloat16_rn(x[e]);
            l[e] = __float2bfloat16_rn(x[e] - __bfloat162float(h[e]));
        }
    }
    *reinterpret_cast<uint4*>(static_cast<T*>(a.x2) + rb * K + k0) = *reinterpret_cast<const uint4*>(h);
    *reinterpret_cast<uint4*>(static_cast<T*>(a.x2) + ((size_t)a.x2_rows + rb) * K + k0) =
        *reinterpret_cast<const uint4*>(l);
}

__device__ __forceinline__ void fp_tma(uint32_t dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void fp_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fp_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// K-major 128-byte-swizzle operand (8-row x 128-byte atoms, 1024 bytes apart)
__device__ __forceinline__ uint64_t fp_desc(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// MN-major 128-byte-swizzle operand: the V tile as TMA lands it (rows = positions = K, 64 head
// dims = N per 128-byte row); the next 64 dims sit one 16 KB atom further (leading byte offset),
// the next 8 positions 1024 bytes further (stride byte offset)
__device__ __forceinline__ uint64_t fp_desc_mn(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)(FP_ATOM >> 4) << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
__device__ __forceinline__ void fp_mma(uint32_t d, uint64_t ad, uint64_t bd, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
        "l"(ad), "l"(bd), "r"(idesc), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void fp_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
// 64 consecutive fp32 columns of this warp's 32 TMEM lanes, one load and one wait
__device__ __forceinline__ void fp_ld64(uint32_t taddr, float* v) {
    uint32_t r[64];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%64];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
          "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
          "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
          "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
          "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 64; i++) v[i] = __uint_as_float(r[i]);
}
// 8 consecutive fp32 columns of this warp's 32 TMEM lanes
__device__ __forceinline__ void fp_ld8(uint32_t taddr, float* v) {
    uint32_t r[8];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 8; i++) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ int fp_abort(const int* p) { return *reinterpret_cast<const volatile int*>(p); }
// byte offset of 16-bit column `col` (0..127) of row `r` in a 128 x 128 K-major swizzled tile
__device__ __forceinline__ uint32_t fp_off(int r, int col) {
    return (uint32_t)((col >> 6) * FP_ATOM + (r >> 3) * 1024 + (r & 7) * 128 + ((((col & 63) >> 3) ^ (r & 7)) << 4) +
                      (col & 7) * 2);
}

__global__ void __launch_bounds__(FP_THREADS, 1)
    vsl_prefill_attention_kernel(const __grid_constant__ CUtensorMap map_k, const __grid_constant__ CUtensorMap map_v,
                                 const __grid_constant__ FpArgs a) {
    VSL_TRACE_ENTRY();
    extern __shared__ unsigned char smem_raw[];
    __shared__ __align__(8) uint64_t k_full, k_empty, v_full, v_empty, s_full[2], s_free[2], q_ready, p_ready, o_full,
        o_free;
    __shared__ uint32_t tmem_s;
    __shared__ int abort_s, len_s, lo_s;
    __shared__ float red_m[2][2][FP_ROWS], red_l[2][FP_ROWS];  // row maxima (by chunk parity) and sums per half

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
    const uint32_t qt = base, kt = base + 2 * FP_TILE, vt = base + 3 * FP_TILE, pt = base + 4 * FP_TILE;
    unsigned char* smem_g = smem_raw - smem_u32(smem_raw);  // generic pointer of shared address 0
    const int h = blockIdx.x, g = h / a.G;
    const int r0 = blockIdx.y * FP_ROWS;

    if (threadIdx.x == 0) {
        mbar_init(&k_full, 1);
        mbar_init(&k_empty, 1);
        mbar_init(&v_full, 1);
        mbar_init(&v_empty, 1);
        for (int i = 0; i < 2; i++) {
            mbar_init(&s_full[i], 1);
            mbar_init(&s_free[i], FP_SM_WARPS);
        }
        mbar_init(&q_ready, FP_SM_WARPS);
        mbar_init(&p_ready, FP_SM_WARPS);
        mbar_init(&o_full, 1);
        mbar_init(&o_free, FP_SM_WARPS);
        mbar_fence_init();
        abort_s = 0;
        len_s = 0;
        lo_s = INT_MAX;
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_k)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_v)) : "memory");
    }
    if (warp == FP_SM_WARPS + 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_s)),
                     "r"(FP_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    // q, K and V of this chunk are written by the preceding projection
    pdl_wait();
    VSL_TRACE_RELEASED();
    __syncthreads();
    // dense mask: chunk 0 starts at position 0 whatever the rows' positions, so the producer
    // requests its K and V now, before the block's length is known (pages of positions past the
    // cache end give rows that are masked (K) or zeroed (V) later; entries outside the page
    // table's row or the pool fall back to row 0 of the pool)
    const bool early = a.sp.min_len <= 0;
    if (early && warp == FP_SM_WARPS && lane == 0) {
        for (int kv = 0; kv < 2; kv++) {
            uint64_t* full = kv ? &v_full : &k_full;
            mbar_arrive_expect_tx(full, FP_TILE);
#pragma unroll
            for (int hh = 0; hh < 2; hh++) {
                const int pi = (hh * 64) / a.page_size;
                const int page = pi < a.max_pages ? __ldg(a.page_row + pi) : 0;
                long long row = ((long long)page * a.n_kv + g) * a.page_size + (hh * 64) % a.page_size;
                if (row < 0 || row + 64 > a.kv_rows) row = 0;
#pragma unroll
                for (int at = 0; at < 2; at++)
                    fp_tma((kv ? vt : kt) + at * FP_ATOM + hh * (FP_ATOM / 2), kv ? &map_v : &map_k, at * 64, (int)row,
                           full);
            }
        }
    }
    // this thread's query row: position, first attended position; the block's cache length and
    // lowest first position
    int pr = -1, first = INT_MAX;
    const int row = threadIdx.x & (FP_ROWS - 1);
    if (threadIdx.x < FP_SM_THREADS && r0 + row < a.P) {
        pr = __ldg(a.pos + r0 + row);
        pr = pr < 0 ? 0 : (pr >= a.max_len ? a.max_len - 1 : pr);
        first = sparse_first(a.sp, pr);
        if (threadIdx.x < FP_ROWS) {
            atomicMax(&len_s, pr + 1);
            atomicMin(&lo_s, first);
        }
    }
    fp_fence_before();
    __syncthreads();
    fp_fence_after();
    const uint32_t tmem = tmem_s;
    const int len = len_s;                          // >= 1: row 0 of the block exists
    const int c0 = (lo_s == INT_MAX ? 0 : lo_s) / FP_CHUNK;
    const int n = (len + FP_CHUNK - 1) / FP_CHUNK - c0;  // chunks of the block

    if (warp == FP_SM_WARPS) {
        // ================= TMA producer: K(i) and V(i) into single tiles =================
        if (lane == 0) {
            int issued_k = early ? 1 : 0, issued_v = early ? 1 : 0;  // chunk 0 already requested
            bool ok = true;
            for (int i = early ? 1 : 0; i < n && ok; i++) {
                for (int kv = 0; kv < 2 && ok; kv++) {
                    uint64_t* full = kv ? &v_full : &k_full;
                    uint64_t* empty = kv ? &v_empty : &k_empty;
                    if (i > 0 && !mbar_wait(empty, (uint32_t)((i - 1) & 1))) {
                        ok = false;
                        break;
                    }
                    if (fp_abort(&abort_s)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(full, FP_TILE);
                    const uint32_t dst = kv ? vt : kt;
#pragma unroll
                    for (int hh = 0; hh < 2; hh++) {
                        int p0 = (c0 + i) * FP_CHUNK + hh * 64;
                        if (p0 >= len) p0 = 0;  // past the end: any valid page (masked or zeroed later)
                        const int page = __ldg(a.page_row + p0 / a.page_size);
                        const int row = (page * a.n_kv + g) * a.page_size + (p0 % a.page_size);
#pragma unroll
                        for (int at = 0; at < 2; at++)
                            fp_tma(dst + at * FP_ATOM + hh * (FP_ATOM / 2), kv ? &map_v : &map_k, at * 64, row, full);
                    }
                    if (kv) issued_v++;
                    else issued_k++;
                }
            }
            if (!ok) {
                set_status(a.status, VSL_ERR_TIMEOUT);
                atomicExch(&abort_s, 1);
            }
            // no copy may still be landing when the CTA leaves
            if (issued_k > 0) mbar_wait(&k_full, (uint32_t)((issued_k - 1) & 1));
            if (issued_v > 0) mbar_wait(&v_full, (uint32_t)((issued_v - 1) & 1));
        }
    } else if (warp == FP_SM_WARPS + 1) {
        // ================= MMA issue =================
        if (lane == 0) {
            FP_STAMP(tm0);
            bool ok = mbar_wait(&q_ready, 0u);
            FP_STAMP(tm_q);
            FP_PHASE(2205u, tm0, tm_q);
            int s_issued = 0, pv_issued = 0;
            auto issue_s = [&](int i) -> bool {
                if (!mbar_wait(&k_full, (uint32_t)(i & 1))) return false;
                if (i >= 2 && !mbar_wait(&s_free[i & 1], (uint32_t)(((i >> 1) - 1) & 1))) return false;
                fp_fence_after();
#pragma unroll
                for (int hl = 0; hl < 2; hl++)
#pragma unroll
                    for (int at = 0; at < 2; at++) {
                        const uint64_t ad = fp_desc(qt + hl * FP_TILE + at * FP_ATOM), bd = fp_desc(kt + at * FP_ATOM);
#pragma unroll
                        for (int k = 0; k < 4; k++)
                            fp_mma(tmem + (uint32_t)((i & 1) * FP_CHUNK), ad + (uint64_t)(2 * k), bd + (uint64_t)(2 * k),
                                   a.idesc_s, (hl | at | k) ? 1u : 0u);
                    }
                fp_commit(&s_full[i & 1]);
                fp_commit(&k_empty);  // K(i) is no longer read
                s_issued++;
                return true;
            };
            auto issue_pv = [&](int i) -> bool {
                if (!mbar_wait(&p_ready, (uint32_t)(i & 1))) return false;
                if (!mbar_wait(&v_full, (uint32_t)(i & 1))) return false;
                if (i >= 1 && !mbar_wait(&o_free, (uint32_t)((i - 1) & 1))) return false;
                fp_fence_after();
#pragma unroll
                for (int hl = 0; hl < 2; hl++)
#pragma unroll
                    for (int k = 0; k < FP_CHUNK / 16; k++) {
                        const uint64_t ad =
                            fp_desc(pt + hl * FP_TILE + (uint32_t)((k >> 2) * FP_ATOM)) + (uint64_t)(2 * (k & 3));
                        const uint64_t bd = fp_desc_mn(vt + (uint32_t)(k * 2048));
                        fp_mma(tmem + 2 * FP_CHUNK, ad, bd, a.idesc_pv, (hl | k) ? 1u : 0u);
                    }
                fp_commit(&o_full);
                fp_commit(&v_empty);  // V(i) and P2(i) are no longer read
                pv_issued++;
                return true;
            };
            if (ok && n > 0) ok = issue_s(0);
            FP_STAMP(tm_s);
            FP_PHASE(2206u, tm_q, tm_s);  // waits for K(0), then issues S(0)
            for (int i = 0; i < n && ok; i++) {
                if (fp_abort(&abort_s)) {
                    ok = false;
                    break;
                }
                if (i + 1 < n) {
                    ok = issue_s(i + 1);
                    if (!ok) break;
                }
                ok = issue_pv(i);
            }
            if (!ok) {
                set_status(a.status, VSL_ERR_TIMEOUT);
                atomicExch(&abort_s, 1);
            }
            // the accumulators must not be freed under a running MMA
            if (s_issued > 0) mbar_wait(&s_full[(s_issued - 1) & 1], (uint32_t)(((s_issued - 1) >> 1) & 1));
            if (pv_issued > 0) mbar_wait(&o_full, (uint32_t)((pv_issued - 1) & 1));
        }
        __syncwarp();
    } else {
        // ===== softmax + accumulation (warps 0-7; row = TMEM lane, hc = half of the columns) =====
        const int t = row;            // query row = TMEM lane
        const int hc = warp >> 2;     // score columns / head dims [64 hc, 64 hc + 64)
        const int th = threadIdx.x;   // 0..255
        FP_STAMP(ts_setup);
        // ---- stage Q2: rows of this head as fp16 hi / lo, 128-byte swizzle ----
        {
            const size_t qs = (size_t)a.n_heads * FP_HD;
            const int col = 4 * lane;
#pragma unroll 8
            for (int k = 0; k < FP_ROWS / FP_SM_WARPS; k++) {
                const int r = warp + FP_SM_WARPS * k;
                float4 x = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                if (r0 + r < a.P)
                    x = __ldcg(reinterpret_cast<const float4*>(a.q + (size_t)(r0 + r) * qs + (size_t)h * FP_HD + col));
                const float xs[4] = {x.x, x.y, x.z, x.w};
                __half hh[4], ll[4];
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    hh[e] = __float2half_rn(xs[e]);
                    ll[e] = __float2half_rn(xs[e] - __half2float(hh[e]));
                }
                const uint32_t o = fp_off(r, col);
                *reinterpret_cast<uint2*>(smem_g + qt + o) = *reinterpret_cast<const uint2*>(hh);
                *reinterpret_cast<uint2*>(smem_g + qt + FP_TILE + o) = *reinterpret_cast<const uint2*>(ll);
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // visible to the tensor cores
            __syncwarp();
            if (lane == 0) mbar_arrive(&q_ready);
        }
        FP_STAMP(ts_q);
        if (th == 0) FP_PHASE(2201u, ts_setup, ts_q);
        constexpr int HALF = FP_CHUNK / 2;  // == FP_HD / 2
        float o[HALF];
#pragma unroll
        for (int j = 0; j < HALF; j++) o[j] = 0.0f;
        float m = -CUDART_INF_F, l = 0.0f;  // l: this half's share of the row sum
        bool failed = false;
        const uint32_t lane_base = ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)(hc * HALF);
        for (int i = 0; i < n; i++) {
            {
                const bool bad = !mbar_wait(&s_full[i & 1], (uint32_t)((i >> 1) & 1)) || fp_abort(&abort_s);
                if (named_barrier_or(1, FP_SM_THREADS, bad)) {  // the softmax warps leave together
                    failed = true;
                    break;
                }
            }
            fp_fence_after();
            FP_STAMP(ts_s);
            const int cb = (c0 + i) * FP_CHUNK + hc * HALF;  // position of this half's score column 0
            const int jlo = first - cb, jhi = pr - cb;       // valid columns: jlo <= j <= jhi
            const uint32_t ts = tmem + lane_base + (uint32_t)((i & 1) * FP_CHUNK);
            // the row's maximum over its valid columns (both halves)
            float sv[HALF];  // this half's scores, read once
            fp_ld64(ts, sv);
            float cm = -CUDART_INF_F;
#pragma unroll
            for (int j = 0; j < HALF; j++)
                if (j >= jlo && j <= jhi) cm = fmaxf(cm, sv[j] * a.scale);
            red_m[i & 1][hc][t] = cm;
            named_barrier_sync(1, FP_SM_THREADS);
            cm = fmaxf(cm, red_m[i & 1][hc ^ 1][t]);
            FP_STAMP(ts_m);
            if (th == 0 && i == 0) FP_PHASE(2207u, ts_s, ts_m);
            const float mn = fmaxf(m, cm);
            const float alpha = mn == -CUDART_INF_F ? 1.0f : expf(m - mn);
            // probabilities, as fp16 hi / lo halves of the row of P2 (P2 of the previous chunk has
            // been read: its product completed before that chunk's fold below)
            // (a rolled loop over 8-column groups, re-reading the scores from TMEM: the code runs
            // once per chunk, and a compact body measured faster than the fully unrolled form
            // working from registers, 6.2 against 9.9 us)
            float ls = 0.0f;
#pragma unroll 1
            for (int c8 = 0; c8 < HALF / 8; c8++) {
                float v[8];
                fp_ld8(ts + (uint32_t)(c8 * 8), v);
                __half ph[8], pl[8];
#pragma unroll
                for (int e = 0; e < 8; e++) {
                    const int j = c8 * 8 + e;
                    const float p = (j >= jlo && j <= jhi) ? expf(v[e] * a.scale - mn) : 0.0f;
                    ls += p;
                    ph[e] = __float2half_rn(p);
                    pl[e] = __float2half_rn(p - __half2float(ph[e]));
                }
                const uint32_t off = fp_off(t, hc * HALF + c8 * 8);
                *reinterpret_cast<uint4*>(smem_g + pt + off) = *reinterpret_cast<const uint4*>(ph);
                *reinterpret_cast<uint4*>(smem_g + pt + FP_TILE + off) = *reinterpret_cast<const uint4*>(pl);
            }
            fp_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s_free[i & 1]);
            m = mn;
            l = l * alpha + ls;
            const int ccb = (c0 + i) * FP_CHUNK;  // position of V row 0
            if (ccb + FP_CHUNK > len) {
                // V rows past the cache end hold whatever the pool had (possibly NaN bit
                // patterns): zero them so that 0 x garbage cannot reach the product (thread th
                // clears half `th / 128` of V row `th % 128`)
                const bool bad = !mbar_wait(&v_full, (uint32_t)(i & 1));
                if (named_barrier_or(1, FP_SM_THREADS, bad)) {
                    failed = true;
                    break;
                }
                const int vr = th & (FP_CHUNK - 1), at = th >> 7;
                if (ccb + vr >= len) {
#pragma unroll
                    for (int c = 0; c < 8; c++)
                        *reinterpret_cast<uint4*>(smem_g + vt + at * FP_ATOM + (vr >> 3) * 1024 + (vr & 7) * 128 +
                                                  c * 16) = make_uint4(0, 0, 0, 0);
                }
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_ready);
            // the next projection's CTAs may start once the first chunk's probabilities are out
            // (earlier, their weight requests delayed this kernel's K and V: 24.7 against 22.1 us)
            if (i == 0) pdl_launch_dependents();
            FP_STAMP(ts_p);
            if (th == 0 && i == 0) FP_PHASE(2202u, ts_s, ts_p);
            // ---- fold PV(i) into this half of the row's accumulators ----
            {
                const bool bad = !mbar_wait(&o_full, (uint32_t)(i & 1)) || fp_abort(&abort_s);
                if (named_barrier_or(1, FP_SM_THREADS, bad)) {
                    failed = true;
                    break;
                }
            }
            fp_fence_after();
            FP_STAMP(ts_o);
            if (th == 0 && i == 0) FP_PHASE(2203u, ts_p, ts_o);
            {
                float v[HALF];
                fp_ld64(tmem + lane_base + (uint32_t)(2 * FP_CHUNK), v);
#pragma unroll
                for (int j = 0; j < HALF; j++) o[j] = o[j] * alpha + v[j];
            }
            fp_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&o_free);
        }
        if (failed) {
            set_status(a.status, VSL_ERR_TIMEOUT);
            atomicExch(&abort_s, 1);
        } else {
            red_l[hc][t] = l;
            named_barrier_sync(1, FP_SM_THREADS);
            // the normalised rows go through shared memory (the Q and K tiles are free: the last
            // scores and product are done) and out with coalesced stores by all 256 threads, in
            // a rolled loop (straight-line stores from each thread's registers measured slower)
            float* ost = reinterpret_cast<float*>(smem_g + qt);  // [128][FP_OST] fp32
            const float inv = pr >= 0 ? 1.0f / (red_l[0][t] + red_l[1][t]) : 0.0f;  // > 0: pr is attended
            float* orow = ost + t * FP_OST + hc * HALF;
#pragma unroll
            for (int j = 0; j < HALF; j += 4)
                *reinterpret_cast<float4*>(orow + j) = make_float4(o[j] * inv, o[j + 1] * inv, o[j + 2] * inv, o[j + 3] * inv);
            named_barrier_sync(1, FP_SM_THREADS);
            const int nrows = min(FP_ROWS, a.P - r0);
            if (a.x2) {
#pragma unroll 1
                for (int it = th; it < nrows * 16; it += FP_SM_THREADS) {  // 16 threads per row, 8 columns each
                    const int r = it >> 4, c8 = (it & 15) * 8;
                    if (a.x2_bf16)
                        fp_store_split8<__nv_bfloat16>(a, (size_t)(r0 + r), (size_t)h * FP_HD + c8, ost + r * FP_OST + c8);
                    else
                        fp_store_split8<__half>(a, (size_t)(r0 + r), (size_t)h * FP_HD + c8, ost + r * FP_OST + c8);
                }
            } else {
#pragma unroll 1
                for (int it = th; it < nrows * 32; it += FP_SM_THREADS) {  // 32 threads per row, 4 columns each
                    const int r = it >> 5, c4 = (it & 31) * 4;
                    *reinterpret_cast<float4*>(a.out + ((size_t)(r0 + r) * a.n_heads + h) * FP_HD + c4) =
                        *reinterpret_cast<const float4*>(ost + r * FP_OST + c4);
                }
            }
            FP_STAMP(ts_end);
            if (th == 0) FP_PHASE(2204u, ts_setup, ts_end);
        }
    }

    fp_fence_before();
    __syncthreads();
    if (warp == FP_SM_WARPS + 1) {
        fp_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(FP_TMEM_COLS) : "memory");
    }
    VSL_TRACE_EXIT(a.trace_id, 2200u);
}

bool flash_prefill_supported(int kvdtype, int head_dim, int n_heads, int n_kv, int page_size) {
    return kvdtype == VSL_F16 && head_dim == FP_HD && n_kv > 0 && n_heads % n_kv == 0 && page_size > 0 &&
           page_size % 64 == 0;
}

int flash_prefill_impl(const float* q, const void* k_cache, const void* v_cache, int n_pages, const int32_t* page_row,
                       int max_pages, int page_size, const int32_t* pos, int P, int n_heads, int n_kv, int max_len,
                       float* out, int* status, cudaStream_t st, const SparseMask* sparse, void* x2, int x2_bf16,
                       int x2_rows) {
    if (!flash_prefill_supported(VSL_F16, FP_HD, n_heads, n_kv, page_size))
        return set_error(VSL_ERR_UNSUPPORTED, "flash_prefill: heads %d/%d page %d", n_heads, n_kv, page_size);
    if (!q || !k_cache || !v_cache || !page_row || !pos || (!out && !x2) || P <= 0 || max_len <= 0 ||
        max_len > max_pages * page_size || n_pages <= 0)
        return set_error(VSL_ERR_INVALID, "flash_prefill: null pointer, no rows or max_len outside the page table");
    if (((uintptr_t)k_cache & 15) || ((uintptr_t)v_cache & 15) || ((uintptr_t)q & 15) || ((uintptr_t)out & 15) ||
        ((uintptr_t)x2 & 15))
        return set_error(VSL_ERR_INVALID, "flash_prefill: caches, q and out must be 16-byte aligned");
    if (x2 && x2_rows < P) return set_error(VSL_ERR_INVALID, "flash_prefill: split tile of %d rows for %d", x2_rows, P);
    FpArgs a = {};
    a.q = q;
    a.pos = pos;
    a.page_row = page_row;
    a.P = P;
    a.n_heads = n_heads;
    a.n_kv = n_kv;
    a.G = n_heads / n_kv;
    a.max_len = max_len;
    a.max_pages = max_pages;
    a.page_size = page_size;
    a.scale = 1.0f / sqrtf((float)FP_HD);
    a.out = out;
    a.status = status;
    a.trace_id = VSL_TRACE_ID();
    a.x2 = x2;
    a.x2_bf16 = x2_bf16;
    a.x2_rows = x2_rows;
    if (sparse && sparse->min_len > 0) {
        if (sparse->window < 0 || sparse->global_tokens < 0 || sparse->block <= 0)
            return set_error(VSL_ERR_INVALID, "flash_prefill: sparse mask window %d, global %d, block %d",
                             sparse->window, sparse->global_tokens, sparse->block);
        a.sp = *sparse;
    }
    // instruction descriptor (kind::f16): D f32 (bits 4-5 = 1), A/B f16 (0), N >> 3 in bits
    // 17-22, M >> 4 in bits 24-28; bit 16 marks B as MN-major (V in the product)
    a.idesc_s = (1u << 4) | ((uint32_t)(FP_CHUNK >> 3) << 17) | ((uint32_t)(FP_ROWS >> 4) << 24);
    a.idesc_pv = (1u << 4) | ((uint32_t)(FP_HD >> 3) << 17) | ((uint32_t)(FP_ROWS >> 4) << 24) | (1u << 16);
    const long long rows = (long long)n_pages * n_kv * page_size;
    a.kv_rows = rows;
    CUtensorMap mk, mv;
    int rc = kv_tensor_map(&mk, k_cache, rows);
    if (rc) return rc;
    rc = kv_tensor_map(&mv, v_cache, rows);
    if (rc) return rc;
    static thread_local int configured_dev = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (configured_dev != dev) {
        cudaError_t e = cudaFuncSetAttribute(vsl_prefill_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)FP_SMEM);
        if (e != cudaSuccess) return launch_status(e, "flash_prefill smem attribute");
        configured_dev = dev;
    }
    const dim3 grid((unsigned)n_heads, (unsigned)((P + FP_ROWS - 1) / FP_ROWS));
    return launch_status(launch_k(vsl_prefill_attention_kernel, grid, dim3(FP_THREADS), FP_SMEM, st, mk, mv, a),
                         "flash_prefill launch");
}

}  // namespace vsl

using namespace vsl;

extern "C" int vsl_flash_prefill(const float* q, const void* k_cache, const void* v_cache, int n_pages,
                                 const int32_t* page_row, int max_pages, int page_size, const int32_t* pos, int n_rows,
                                 int n_heads, int n_kv, int head_dim, int max_len, float* out,
                                 const vsl_sparse_mask* mask, int* status, void* stream) {
    if (head_dim != FP_HD) return set_error(VSL_ERR_UNSUPPORTED, "flash_prefill: head_dim %d (128 only)", head_dim);
    SparseMask m = {};
    if (mask && mask->min_len > 0) m = SparseMask{mask->min_len, mask->window, mask->global_tokens, mask->block};
    return flash_prefill_impl(q, k_cache, v_cache, n_pages, page_row, max_pages, page_size, pos, n_rows, n_heads, n_kv,
                              max_len, out, status, (cudaStream_t)stream, &m, nullptr, 0, 0);
}
