// Decode projections: y = x W^T for a handful of activation rows, HBM-bound weight streaming.
//
// Replaces the projection math of the reference's attention.comp:63-99 (QKV), :191-199 (O),
// feed_forward.comp:36-61 (gate/up/down) and final_linear.comp:38-86 (lm_head), which the
// engine dispatches from attention_with_weights / feed_forward_with_weights /
// final_projection_with_weights (vk_symbiote/src/VulkanSymbioteEngine.cpp:2440-2584,
// 2726-2807, 3028-3130).
//
// Design (B200): weights are read exactly once per decode step, so the kernel is a pure
// HBM stream. Each CTA owns a contiguous, balanced range of row pairs; a warp streams two
// rows at a time with 16-byte L1-bypassing loads, U vectors per row in flight per lane,
// and reduces with warp shuffles. The (optionally RMS-normalised) activations are staged
// once per CTA in shared memory as fp32. Launched with programmatic dependent launch: the
// first weight vectors are requested before griddepcontrol.wait, so the weight stream of
// projection n+1 overlaps the tail of kernel n. Epilogues fuse the residual add, SwiGLU,
// RoPE + paged KV append, and the lm_head argmax / Gumbel sampler.
#include <cstdio>
#include <cuda_runtime.h>

#include "common.cuh"
#include "epilogue.cuh"
#include "quant_layout.h"
#include "tc_gemm.h"
#include "launch.cuh"
#include "trace.cuh"

VSL_TRACE_UNIT(gemv)

namespace vsl {

constexpr int GEMV_THREADS = 256;

static GemvParams traced(GemvParams p) {
    p.trace_id = VSL_TRACE_ID();
    return p;
}
constexpr int GEMV_U = 8;
constexpr int GEMV_L2_HEAD = 96 * 1024;

template <typename WT, int NB, int EK, bool NORM>
__global__ void __launch_bounds__(GEMV_THREADS, 2) vsl_gemv_kernel(const GemvParams p) {
    VSL_TRACE_ENTRY();
    extern __shared__ __align__(16) float xs[];  // [NB][K] fp32 activations
    __shared__ float red[NB][GEMV_THREADS / 32];
    constexpr int VEC = WTraits<WT>::VEC;
    const int K = p.K, N = p.N;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int NW = GEMV_THREADS / 32;
    const int nvec = K / VEC;
    const int n_units = (N + 1) >> 1;
    // balanced contiguous range of row pairs for this CTA
    const int u_begin = (int)(((long long)n_units * blockIdx.x) / gridDim.x);
    const int u_end = (int)(((long long)n_units * (blockIdx.x + 1)) / gridDim.x);
    const WT* W = reinterpret_cast<const WT*>(p.W);

    int unit = u_begin + warp;

    // L2 window: the CTA's rows are one contiguous byte range; request its head now
    {
        const size_t row_bytes = (size_t)K * sizeof(WT);
        const size_t r_lo = 2 * (size_t)u_begin, r_hi = min((size_t)N, 2 * (size_t)u_end);
        const char* base = reinterpret_cast<const char*>(W) + r_lo * row_bytes;
        const size_t total = (r_hi - r_lo) * row_bytes;
        const size_t head = min(total, (size_t)GEMV_L2_HEAD);
        for (size_t off = (size_t)threadIdx.x * 16384; off < head; off += (size_t)GEMV_THREADS * 16384)
            prefetch_l2(base + off, (uint32_t)min((size_t)16384, head - off));
    }

    pdl_wait();
    VSL_TRACE_RELEASED();
    pdl_launch_dependents();

    // ---- stage activations (RMS-normalised if requested) ----
    const int B = p.B;
    if (NORM) {
        float ss[NB];
#pragma unroll
        for (int b = 0; b < NB; b++) ss[b] = 0.0f;
        for (int k = threadIdx.x; k < K; k += GEMV_THREADS) {
#pragma unroll
            for (int b = 0; b < NB; b++) {
                float v = b < B ? p.x[(size_t)b * K + k] : 0.0f;
                ss[b] += v * v;
            }
        }
#pragma unroll
        for (int b = 0; b < NB; b++) {
            float s = warp_sum(ss[b]);
            if (lane == 0) red[b][warp] = s;
        }
        __syncthreads();
#pragma unroll
        for (int b = 0; b < NB; b++) {
            float s = 0.0f;
#pragma unroll
            for (int w = 0; w < NW; w++) s += red[b][w];
            ss[b] = sqrtf(s / (float)K + p.eps);  // rms_norm.comp:32-34: x / sqrt(var) * w
        }
        for (int k = threadIdx.x; k < K; k += GEMV_THREADS) {
            float w = p.norm_w[k];
#pragma unroll
            for (int b = 0; b < NB; b++)
                xs[b * K + k] = b < B ? p.x[(size_t)b * K + k] / ss[b] * w : 0.0f;
        }
    } else {
        for (int k = threadIdx.x; k < K; k += GEMV_THREADS) {
#pragma unroll
            for (int b = 0; b < NB; b++) xs[b * K + k] = b < B ? p.x[(size_t)b * K + k] : 0.0f;
        }
    }
    __syncthreads();

    unsigned long long best[NB];
#pragma unroll
    for (int b = 0; b < NB; b++) best[b] = 0ull;
    int step = 0;
    if (EK == EK_LMHEAD && p.inv_temp > 0.0f) step = *p.step_counter;

    for (; unit < u_end; unit += NW) {
        const int r0 = 2 * unit;
        const bool has1 = r0 + 1 < N;
        const int r1 = has1 ? r0 + 1 : r0;
        const WT* w0 = W + (size_t)r0 * K;
        const WT* w1 = W + (size_t)r1 * K;
        // keep the L2 window moving: this warp's next pair
        if (lane == 0 && unit + NW < u_end) {
            const int rn = 2 * (unit + NW);
            const int rows = min(2, N - rn);
            prefetch_l2(W + (size_t)rn * K, (uint32_t)((size_t)rows * K * sizeof(WT)));
        }
        float acc0[NB], acc1[NB];
#pragma unroll
        for (int b = 0; b < NB; b++) { acc0[b] = 0.0f; acc1[b] = 0.0f; }
        int v = lane;
        for (; v + 32 * (GEMV_U - 1) < nvec; v += 32 * GEMV_U) {
            uint4 a[GEMV_U], c[GEMV_U];
#pragma unroll
            for (int u = 0; u < GEMV_U; u++) {
                a[u] = ldg_stream(w0 + (size_t)(v + 32 * u) * VEC);
                c[u] = ldg_stream(w1 + (size_t)(v + 32 * u) * VEC);
            }
#pragma unroll
            for (int u = 0; u < GEMV_U; u++) {
                float fa[VEC], fc[VEC];
                WTraits<WT>::widen(a[u], fa);
                WTraits<WT>::widen(c[u], fc);
                const int k = (v + 32 * u) * VEC;
#pragma unroll
                for (int b = 0; b < NB; b++) {
                    const float4* xv = reinterpret_cast<const float4*>(xs + b * K + k);
#pragma unroll
                    for (int i = 0; i < VEC / 4; i++) {
                        float4 xx = xv[i];
                        acc0[b] = fmaf(fa[4 * i + 0], xx.x, acc0[b]);
                        acc0[b] = fmaf(fa[4 * i + 1], xx.y, acc0[b]);
                        acc0[b] = fmaf(fa[4 * i + 2], xx.z, acc0[b]);
                        acc0[b] = fmaf(fa[4 * i + 3], xx.w, acc0[b]);
                        acc1[b] = fmaf(fc[4 * i + 0], xx.x, acc1[b]);
                        acc1[b] = fmaf(fc[4 * i + 1], xx.y, acc1[b]);
                        acc1[b] = fmaf(fc[4 * i + 2], xx.z, acc1[b]);
                        acc1[b] = fmaf(fc[4 * i + 3], xx.w, acc1[b]);
                    }
                }
            }
        }
        for (; v < nvec; v += 32) {
            uint4 a = ldg_stream(w0 + (size_t)v * VEC);
            uint4 c = ldg_stream(w1 + (size_t)v * VEC);
            float fa[VEC], fc[VEC];
            WTraits<WT>::widen(a, fa);
            WTraits<WT>::widen(c, fc);
            const int k = v * VEC;
#pragma unroll
            for (int b = 0; b < NB; b++) {
#pragma unroll
                for (int i = 0; i < VEC; i++) {
                    acc0[b] = fmaf(fa[i], xs[b * K + k + i], acc0[b]);
                    acc1[b] = fmaf(fc[i], xs[b * K + k + i], acc1[b]);
                }
            }
        }
#pragma unroll
        for (int b = 0; b < NB; b++) {
            acc0[b] = warp_sum(acc0[b]);
            acc1[b] = warp_sum(acc1[b]);
        }
        // epilogue: lane b handles activation row b
#pragma unroll
        for (int b = 0; b < NB; b++) {
            if (lane != b || b >= B) continue;
            gemv_pair_epilogue<EK>(p, b, r0, unit, has1, acc0[b], acc1[b], best[b], step);
        }
    }
    if (EK == EK_LMHEAD) {
#pragma unroll
        for (int b = 0; b < NB; b++)
            if (lane == b && b < B && best[b] != 0ull) atomicMax(p.slots + b, best[b]);
    }
    if (p.pf_ptr && lane == 0) prefetch_share(p.pf_ptr, p.pf_bytes, blockIdx.x, gridDim.x, warp, NW);
    VSL_TRACE_EXIT(p.trace_id, (unsigned)(EK * 100 + (NORM ? 10 : 0) + NB));
}

// ---------------------------------------------------------------------------------------
// Block-quantized weights (Q8_0 / Q4_0 / Q4_1 in the repacked row layout of quant_layout.h)
// ---------------------------------------------------------------------------------------
// One 16-byte vector of quants is 16 (Q8_0, half a block) or 32 (Q4_0, one block) weights.
// Quants become floats without conversion instructions: a 32-bit pattern u < 2^23 read as an
// fp32 value is exactly u * 2^-149 (a subnormal, or the first normal binade), so one byte
// permute that drops the biased quant (q + 128 for Q8_0, the stored nibble for Q4_0) into the
// low byte of a zero word gives the exact float u * 2^-149. The activations are staged
// multiplied by 2^64, so each product u * x * 2^-85 stays a normal fp32 number, and the
// products are accumulated two at a time with the packed fp32 FMA (fma.rn.f32x2) of sm_100.
// Per vector the zero point comes out once: sum(q * x) = 2^85 * sum(u * x') - z * sum(x), with
// z = 128 (Q8_0) or 8 (Q4_0) and the per-vector activation sums staged beside the activations;
// the row accumulates d * that (one fp32 FMA per vector and row).
template <int QT> struct QTraits;
template <> struct QTraits<VSL_Q8_0> {
    static constexpr int VEC = 16;     // weights per 16-byte vector
    static constexpr float ZP = 128.0f;  // bias of the stored byte
    // u[i] = biased quant of element i (as fp32 bit pattern)
    __device__ __forceinline__ static void unpack(const uint4& v, uint32_t* u) {
        const uint32_t w[4] = {v.x ^ 0x80808080u, v.y ^ 0x80808080u, v.z ^ 0x80808080u, v.w ^ 0x80808080u};
#pragma unroll
        for (int j = 0; j < 4; j++)
#pragma unroll
            for (int i = 0; i < 4; i++) u[4 * j + i] = __byte_perm(w[j], 0u, 0x4440u + i);
    }
};
template <> struct QTraits<VSL_Q4_0> {
    static constexpr int VEC = 32;
    static constexpr float ZP = 8.0f;
    __device__ __forceinline__ static void unpack(const uint4& v, uint32_t* u) {
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const uint32_t lo = w[j] & 0x0F0F0F0Fu, hi = (w[j] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                u[4 * j + i] = __byte_perm(lo, 0u, 0x4440u + i);       // element 4j + i
                u[16 + 4 * j + i] = __byte_perm(hi, 0u, 0x4440u + i);  // element 16 + 4j + i
            }
        }
    }
};

// Q4_1: the same nibbles, unsigned; value = nibble * d + m, so a vector contributes
// d * sum(u * x) + m * sum(x), and the staged per-vector sums are the plain sums (ZP = 1).
template <> struct QTraits<VSL_Q4_1> {
    static constexpr int VEC = 32;
    static constexpr float ZP = 1.0f;
    __device__ __forceinline__ static void unpack(const uint4& v, uint32_t* u) { QTraits<VSL_Q4_0>::unpack(v, u); }
};

__device__ __forceinline__ unsigned long long pack2(uint32_t lo, uint32_t hi) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
    return r;
}
__device__ __forceinline__ unsigned long long pack2f(float lo, float hi) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
// acc.{x,y} += a.{x,y} * b.{x,y}, each lane one fp32 FMA (round to nearest, subnormals kept)
__device__ __forceinline__ void ffma2(unsigned long long& acc, unsigned long long a, unsigned long long b) {
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(a), "l"(b));
}
__device__ __forceinline__ float sum2(unsigned long long v) {
    float lo, hi;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
    return lo + hi;
}

constexpr float Q_XSCALE = 18446744073709551616.0f;  // 2^64, activation pre-scale
constexpr float Q_UNSCALE = 38685626227668133590597632.0f;  // 2^85 = 2^149 / 2^64

// Activations are staged as fp32 (times 2^64) with 4 floats of padding after every VEC
// values, so the 16-byte shared-memory reads of a warp (lane l reads chunk l) fall in
// distinct banks; the per-vector sums (times the zero point) follow the activations.
template <int QT>
__host__ __device__ constexpr int q_xpitch(int K) {
    return K + (K / QTraits<QT>::VEC) * 4;
}
// per activation row: the padded activations, then the vector sums, rounded up to 4 floats so
// that every row starts 16-byte aligned (the float4 reads)
template <int QT>
__host__ __device__ constexpr int q_stage_floats(int K) {
    return q_xpitch<QT>(K) + (K / QTraits<QT>::VEC + 3) / 4 * 4;
}

template <int QT, int NB, int EK, bool NORM>
__global__ void __launch_bounds__(GEMV_THREADS, 2) vsl_gemv_q_kernel(const GemvParams p) {
    VSL_TRACE_ENTRY();
    extern __shared__ __align__(16) float xs[];  // [NB][q_stage_floats(K)]
    __shared__ float red[NB][GEMV_THREADS / 32];
    constexpr int VEC = QTraits<QT>::VEC;
    constexpr int CH = VEC + 4;  // padded chunk
    const int K = p.K, N = p.N;
    const int XP = q_xpitch<QT>(K), SP = q_stage_floats<QT>(K);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int NW = GEMV_THREADS / 32;
    const int nvec = K / VEC;
    const size_t RB = weight_row_bytes(QT, K), QB = quant_bytes(QT, K);
    const int MO = (int)(scale_bytes(K) / 2);  // Q4_1: minimums follow the scales (fp16 elements)
    const int n_units = (N + 1) >> 1;
    const int u_begin = (int)(((long long)n_units * blockIdx.x) / gridDim.x);
    const int u_end = (int)(((long long)n_units * (blockIdx.x + 1)) / gridDim.x);
    const char* W = reinterpret_cast<const char*>(p.W);

    int unit = u_begin + warp;
    {
        const size_t r_lo = 2 * (size_t)u_begin, r_hi = min((size_t)N, 2 * (size_t)u_end);
        const char* base = W + r_lo * RB;
        const size_t total = (r_hi - r_lo) * RB;
        const size_t head = min(total, (size_t)GEMV_L2_HEAD);
        for (size_t off = (size_t)threadIdx.x * 16384; off < head; off += (size_t)GEMV_THREADS * 16384)
            prefetch_l2(base + off, (uint32_t)min((size_t)16384, head - off));
    }

    pdl_wait();
    VSL_TRACE_RELEASED();
    pdl_launch_dependents();

    const int B = p.B;
    float den[NB];
#pragma unroll
    for (int b = 0; b < NB; b++) den[b] = 1.0f;
    if (NORM) {
#pragma unroll
        for (int b = 0; b < NB; b++) den[b] = 0.0f;
        for (int k = threadIdx.x; k < K; k += GEMV_THREADS) {
#pragma unroll
            for (int b = 0; b < NB; b++) {
                float v = b < B ? p.x[(size_t)b * K + k] : 0.0f;
                den[b] += v * v;
            }
        }
#pragma unroll
        for (int b = 0; b < NB; b++) {
            float s = warp_sum(den[b]);
            if (lane == 0) red[b][warp] = s;
        }
        __syncthreads();
#pragma unroll
        for (int b = 0; b < NB; b++) {
            float s = 0.0f;
#pragma unroll
            for (int w = 0; w < NW; w++) s += red[b][w];
            den[b] = sqrtf(s / (float)K + p.eps);  // rms_norm.comp:32-34: x / sqrt(var) * w
        }
    }
    for (int k = threadIdx.x; k < K; k += GEMV_THREADS) {
        const float w = NORM ? p.norm_w[k] : 1.0f;
        const int xi = k + (k / VEC) * 4;
#pragma unroll
        for (int b = 0; b < NB; b++) {
            const float v = b < B ? p.x[(size_t)b * K + k] : 0.0f;
            xs[b * SP + xi] = (NORM ? v / den[b] * w : v) * Q_XSCALE;
        }
    }
    __syncthreads();
    // zero-point term of every vector: z * sum of its activations (fixed order)
    for (int i = threadIdx.x; i < NB * nvec; i += GEMV_THREADS) {
        const int b = i / nvec, v = i - b * nvec;
        const float* c = xs + b * SP + v * CH;
        float s = 0.0f;
#pragma unroll
        for (int j = 0; j < VEC; j++) s += c[j];
        xs[b * SP + XP + v] = s * (QTraits<QT>::ZP / Q_XSCALE);
    }
    __syncthreads();

    unsigned long long best[NB];
#pragma unroll
    for (int b = 0; b < NB; b++) best[b] = 0ull;
    int step = 0;
    if (EK == EK_LMHEAD && p.inv_temp > 0.0f) step = *p.step_counter;

    constexpr int U = (QT != VSL_Q8_0 && NB >= 4) ? 2 : 4;  // vectors in flight per row and lane
    constexpr bool MIN = QT == VSL_Q4_1;
    for (; unit < u_end; unit += NW) {
        const int r0 = 2 * unit;
        const bool has1 = r0 + 1 < N;
        const int r1 = has1 ? r0 + 1 : r0;
        const char* row0 = W + (size_t)r0 * RB;
        const char* row1 = W + (size_t)r1 * RB;
        const unsigned short* sc0 = reinterpret_cast<const unsigned short*>(row0 + QB);
        const unsigned short* sc1 = reinterpret_cast<const unsigned short*>(row1 + QB);
        if (lane == 0 && unit + NW < u_end) {  // keep the L2 window moving: this warp's next pair
            const int rn = 2 * (unit + NW);
            prefetch_l2(W + (size_t)rn * RB, (uint32_t)(min(2, N - rn) * RB));
        }
        float acc0[NB], acc1[NB];
#pragma unroll
        for (int b = 0; b < NB; b++) { acc0[b] = 0.0f; acc1[b] = 0.0f; }
        auto consume = [&](const uint4& a, const uint4& c, float d0, float d1, float m0, float m1, int v) {
            uint32_t ua[VEC], uc[VEC];
            QTraits<QT>::unpack(a, ua);
            QTraits<QT>::unpack(c, uc);
#pragma unroll
            for (int b = 0; b < NB; b++) {
                unsigned long long t0 = 0ull, t1 = 0ull;
                const float4* xv = reinterpret_cast<const float4*>(xs + b * SP + v * CH);
#pragma unroll
                for (int i = 0; i < VEC / 4; i++) {
                    const float4 xx = xv[i];
                    const unsigned long long x01 = pack2f(xx.x, xx.y), x23 = pack2f(xx.z, xx.w);
                    ffma2(t0, pack2(ua[4 * i + 0], ua[4 * i + 1]), x01);
                    ffma2(t0, pack2(ua[4 * i + 2], ua[4 * i + 3]), x23);
                    ffma2(t1, pack2(uc[4 * i + 0], uc[4 * i + 1]), x01);
                    ffma2(t1, pack2(uc[4 * i + 2], uc[4 * i + 3]), x23);
                }
                const float zx = xs[b * SP + XP + v];
                if (MIN) {  // d * sum(u x) + m * sum(x)
                    acc0[b] = fmaf(d0, Q_UNSCALE * sum2(t0), fmaf(m0, zx, acc0[b]));
                    acc1[b] = fmaf(d1, Q_UNSCALE * sum2(t1), fmaf(m1, zx, acc1[b]));
                } else {    // d * (sum(u x) - z sum(x))
                    acc0[b] = fmaf(d0, fmaf(Q_UNSCALE, sum2(t0), -zx), acc0[b]);
                    acc1[b] = fmaf(d1, fmaf(Q_UNSCALE, sum2(t1), -zx), acc1[b]);
                }
            }
        };
        int v = lane;
        for (; v + 32 * (U - 1) < nvec; v += 32 * U) {
            uint4 a[U], c[U];
            unsigned short s0[U], s1[U], n0[U], n1[U];
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int vv = v + 32 * u;
                a[u] = ldg_stream(row0 + (size_t)vv * 16);
                c[u] = ldg_stream(row1 + (size_t)vv * 16);
                s0[u] = __ldcs(sc0 + (vv * VEC) / QBLK);
                s1[u] = __ldcs(sc1 + (vv * VEC) / QBLK);
                if (MIN) {
                    n0[u] = __ldcs(sc0 + MO + (vv * VEC) / QBLK);
                    n1[u] = __ldcs(sc1 + MO + (vv * VEC) / QBLK);
                }
            }
#pragma unroll
            for (int u = 0; u < U; u++)
                consume(a[u], c[u], __half2float(__ushort_as_half(s0[u])), __half2float(__ushort_as_half(s1[u])),
                        MIN ? __half2float(__ushort_as_half(n0[u])) : 0.0f,
                        MIN ? __half2float(__ushort_as_half(n1[u])) : 0.0f, v + 32 * u);
        }
        for (; v < nvec; v += 32) {
            const uint4 a = ldg_stream(row0 + (size_t)v * 16);
            const uint4 c = ldg_stream(row1 + (size_t)v * 16);
            const float d0 = __half2float(__ushort_as_half(__ldcs(sc0 + (v * VEC) / QBLK)));
            const float d1 = __half2float(__ushort_as_half(__ldcs(sc1 + (v * VEC) / QBLK)));
            const float m0 = MIN ? __half2float(__ushort_as_half(__ldcs(sc0 + MO + (v * VEC) / QBLK))) : 0.0f;
            const float m1 = MIN ? __half2float(__ushort_as_half(__ldcs(sc1 + MO + (v * VEC) / QBLK))) : 0.0f;
            consume(a, c, d0, d1, m0, m1, v);
        }
#pragma unroll
        for (int b = 0; b < NB; b++) {
            acc0[b] = warp_sum(acc0[b]);
            acc1[b] = warp_sum(acc1[b]);
        }
#pragma unroll
        for (int b = 0; b < NB; b++) {
            if (lane != b || b >= B) continue;
            gemv_pair_epilogue<EK>(p, b, r0, unit, has1, acc0[b], acc1[b], best[b], step);
        }
    }
    if (EK == EK_LMHEAD) {
#pragma unroll
        for (int b = 0; b < NB; b++)
            if (lane == b && b < B && best[b] != 0ull) atomicMax(p.slots + b, best[b]);
    }
    if (p.pf_ptr && lane == 0) prefetch_share(p.pf_ptr, p.pf_bytes, blockIdx.x, gridDim.x, warp, NW);
    VSL_TRACE_EXIT(p.trace_id, (unsigned)(EK * 100 + (NORM ? 10 : 0) + NB));
}

// ---------------------------------------------------------------------------------------
// host dispatch
// ---------------------------------------------------------------------------------------

// activation rows one launch stages in shared memory (fp32 [rows][K]); the compiled row
// counts are 1, 2 and 4
static int max_rows_per_launch(int wdtype, int K) {
    const size_t room = 200 * 1024;
    const size_t pitch = wdtype == VSL_Q8_0   ? (size_t)q_stage_floats<VSL_Q8_0>(K)
                         : wdtype == VSL_Q4_0 ? (size_t)q_stage_floats<VSL_Q4_0>(K)
                         : wdtype == VSL_Q4_1 ? (size_t)q_stage_floats<VSL_Q4_1>(K)
                                              : (size_t)K;
    const int c = (int)(room / (pitch * sizeof(float)));
    return c >= 4 ? 4 : c >= 2 ? 2 : c;
}

template <typename WT, int NB, int EK, bool NORM>
static int launch_gemv_t(const GemvParams& p, cudaStream_t st) {
    auto kern = vsl_gemv_kernel<WT, NB, EK, NORM>;
    const size_t smem = (size_t)NB * p.K * sizeof(float);
    static thread_local int configured_dev = -1;
    static thread_local size_t configured_smem = 0;
    static thread_local int occ = 1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (configured_dev != dev || configured_smem != smem) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return launch_status(e, "gemv smem attribute");
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, GEMV_THREADS, smem);
        if (e != cudaSuccess) return launch_status(e, "gemv occupancy");
        if (occ < 1) return set_error(VSL_ERR_UNSUPPORTED, "gemv: K=%d does not fit in shared memory", p.K);
        if (occ > 2) occ = 2;
        configured_dev = dev;
        configured_smem = smem;
    }
    // grid = whole waves of resident CTAs; each CTA owns a contiguous, balanced range of row pairs
    const int n_units = (p.N + 1) / 2;
    const int nw = GEMV_THREADS / 32;
    int grid = sm_count() * occ;
    const int max_grid = (n_units + nw - 1) / nw;
    if (grid > max_grid) grid = max_grid;
    if (grid < 1) grid = 1;
    return launch_status(launch_k(kern, dim3(grid), dim3(GEMV_THREADS), smem, st, traced(p)), "gemv launch");
}

template <int QT, int NB, int EK, bool NORM>
static int launch_gemv_q_t(const GemvParams& p, cudaStream_t st) {
    auto kern = vsl_gemv_q_kernel<QT, NB, EK, NORM>;
    const size_t smem = (size_t)NB * q_stage_floats<QT>(p.K) * sizeof(float);
    static thread_local int configured_dev = -1;
    static thread_local size_t configured_smem = 0;
    static thread_local int occ = 1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (configured_dev != dev || configured_smem != smem) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return launch_status(e, "gemv smem attribute");
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, GEMV_THREADS, smem);
        if (e != cudaSuccess) return launch_status(e, "gemv occupancy");
        if (occ < 1) return set_error(VSL_ERR_UNSUPPORTED, "gemv: K=%d does not fit in shared memory", p.K);
        if (occ > 2) occ = 2;
        configured_dev = dev;
        configured_smem = smem;
    }
    const int n_units = (p.N + 1) / 2;
    const int nw = GEMV_THREADS / 32;
    int grid = sm_count() * occ;
    const int max_grid = (n_units + nw - 1) / nw;
    if (grid > max_grid) grid = max_grid;
    if (grid < 1) grid = 1;
    return launch_status(launch_k(kern, dim3(grid), dim3(GEMV_THREADS), smem, st, traced(p)), "gemv launch");
}

template <int QT, int EK, bool NORM>
static int launch_gemv_q_nb(const GemvParams& p, cudaStream_t st) {
    if (p.B <= 1) return launch_gemv_q_t<QT, 1, EK, NORM>(p, st);
    if (p.B <= 2) return launch_gemv_q_t<QT, 2, EK, NORM>(p, st);
    return launch_gemv_q_t<QT, 4, EK, NORM>(p, st);
}

template <typename WT, int EK, bool NORM>
static int launch_gemv_nb(const GemvParams& p, cudaStream_t st) {
    if (p.B <= 1) return launch_gemv_t<WT, 1, EK, NORM>(p, st);
    if (p.B <= 2) return launch_gemv_t<WT, 2, EK, NORM>(p, st);
    return launch_gemv_t<WT, 4, EK, NORM>(p, st);
}

template <int EK, bool NORM>
static int launch_gemv_w(int wdtype, const GemvParams& p, cudaStream_t st) {
    switch (wdtype) {
        case VSL_F32: return launch_gemv_nb<float, EK, NORM>(p, st);
        case VSL_F16: return launch_gemv_nb<__half, EK, NORM>(p, st);
        case VSL_BF16: return launch_gemv_nb<__nv_bfloat16, EK, NORM>(p, st);
        case VSL_Q8_0: return launch_gemv_q_nb<VSL_Q8_0, EK, NORM>(p, st);
        case VSL_Q4_0: return launch_gemv_q_nb<VSL_Q4_0, EK, NORM>(p, st);
        case VSL_Q4_1: return launch_gemv_q_nb<VSL_Q4_1, EK, NORM>(p, st);
        default: return set_error(VSL_ERR_UNSUPPORTED, "gemv: weight dtype %d", wdtype);
    }
}

template <int EK>
static int launch_gemv_norm(int wdtype, const GemvParams& p, cudaStream_t st) {
    return p.norm_w ? launch_gemv_w<EK, true>(wdtype, p, st) : launch_gemv_w<EK, false>(wdtype, p, st);
}

static int check_common(int wdtype, const void* W, int N, int K, const float* x, int B) {
    if (wdtype != VSL_F32 && wdtype != VSL_F16 && wdtype != VSL_BF16 && !is_quant(wdtype))
        return set_error(VSL_ERR_UNSUPPORTED, "weight dtype %d", wdtype);
    if (!W || !x || N <= 0 || K <= 0 || B <= 0)
        return set_error(VSL_ERR_INVALID, "gemv: null pointer or empty shape (N=%d K=%d B=%d)", N, K, B);
    if (is_quant(wdtype) && K % QBLK)
        return set_error(VSL_ERR_INVALID, "gemv: quantized rows need K a multiple of %d (K=%d)", QBLK, K);
    if (((uintptr_t)W & 15) || weight_row_bytes(wdtype, (size_t)K) % 16)
        return set_error(VSL_ERR_INVALID, "gemv: weight rows must be 16-byte aligned (K=%d)", K);
    if ((uintptr_t)x & 15) return set_error(VSL_ERR_INVALID, "gemv: activations must be 16-byte aligned");
    return VSL_OK;
}

// Large batches go to the tensor cores when the caller provides a route (every weight tile
// read once for all rows); otherwise they are processed in chunks of 4 activation rows, each
// chunk re-streaming W.
static int run_chunks(int wdtype, int kind, GemvParams p, cudaStream_t st, int y_cols,
                      const TcRoute* tc = nullptr) {
    const int B = p.B;
    if (tc && tc->ws && B >= tc->min_batch && tc_supported(wdtype, p.N, p.K, B))
        return tc_project(wdtype, kind, p, tc->ws, tc->bytes, tc->status ? tc->status : p.status, st);
    // activation rows per launch: at most 4, and at most what fits beside the weight ring
    const int cmax = max_rows_per_launch(wdtype, p.K);
    if (cmax < 1) return set_error(VSL_ERR_UNSUPPORTED, "gemv: K=%d exceeds the shared-memory staging limit", p.K);
    for (int b0 = 0; b0 < B; b0 += cmax) {
        GemvParams q = p;
        q.B = B - b0 < cmax ? B - b0 : cmax;
        q.x = p.x + (size_t)b0 * p.K;
        if (p.y) q.y = p.y + (size_t)b0 * y_cols;
        if (p.pos) q.pos = p.pos + b0;
        if (p.q_out) q.q_out = p.q_out + (size_t)b0 * p.n_heads * p.head_dim;
        if (p.page_table) q.page_table = p.page_table + (size_t)b0 * p.max_pages;
        if (p.slots) q.slots = p.slots + b0;
        int rc;
        switch (kind) {
            case EK_STORE: rc = launch_gemv_norm<EK_STORE>(wdtype, q, st); break;
            case EK_ADD: rc = launch_gemv_norm<EK_ADD>(wdtype, q, st); break;
            case EK_SWIGLU: rc = launch_gemv_norm<EK_SWIGLU>(wdtype, q, st); break;
            case EK_QKV: rc = launch_gemv_norm<EK_QKV>(wdtype, q, st); break;
            default: rc = launch_gemv_norm<EK_LMHEAD>(wdtype, q, st); break;
        }
        if (rc) return rc;
    }
    return VSL_OK;
}

}  // namespace vsl

using namespace vsl;

extern "C" int vsl_gemv(int wdtype, const void* W, int N, int K, const float* x, int B, float* y, int epilogue,
                        const float* norm_w, float eps, void* stream) {
    int rc = check_common(wdtype, W, N, K, x, B);
    if (rc) return rc;
    if (!y) return set_error(VSL_ERR_INVALID, "gemv: null output");
    if (epilogue == VSL_EPI_SWIGLU && (N & 1))
        return set_error(VSL_ERR_INVALID, "gemv: SwiGLU needs interleaved gate/up rows (N even), N=%d", N);
    GemvParams p = {};
    p.W = W; p.N = N; p.K = K; p.x = x; p.B = B; p.y = y; p.norm_w = norm_w; p.eps = eps;
    int kind = epilogue == VSL_EPI_ADD ? EK_ADD : epilogue == VSL_EPI_SWIGLU ? EK_SWIGLU : EK_STORE;
    if (epilogue != VSL_EPI_STORE && epilogue != VSL_EPI_ADD && epilogue != VSL_EPI_SWIGLU)
        return set_error(VSL_ERR_INVALID, "gemv: unknown epilogue %d", epilogue);
    return run_chunks(wdtype, kind, p, (cudaStream_t)stream, epilogue == VSL_EPI_SWIGLU ? N / 2 : N);
}

extern "C" int vsl_qkv_rope_append(int wdtype, const void* Wqkv, int n_heads, int n_kv, int head_dim, int K,
                                   const float* x, const float* norm_w, float eps, int B, const int32_t* pos,
                                   const float* rope_cos, const float* rope_sin, float* q_out, void* k_cache,
                                   void* v_cache, int kvdtype, const int32_t* page_table, int max_pages,
                                   int page_size, void* stream) {
    if (n_heads <= 0 || n_kv <= 0 || head_dim <= 0 || (head_dim & 1) || n_heads % n_kv)
        return set_error(VSL_ERR_INVALID, "qkv: bad head geometry (%d/%d x %d)", n_heads, n_kv, head_dim);
    const int N = (n_heads + 2 * n_kv) * head_dim;
    int rc = check_common(wdtype, Wqkv, N, K, x, B);
    if (rc) return rc;
    if (!pos || !rope_cos || !rope_sin || !q_out || !k_cache || !v_cache || !page_table || max_pages <= 0 ||
        page_size <= 0)
        return set_error(VSL_ERR_INVALID, "qkv: null pointer or empty cache geometry");
    if (kvdtype != VSL_F32 && kvdtype != VSL_F16 && kvdtype != VSL_BF16)
        return set_error(VSL_ERR_UNSUPPORTED, "qkv: kv dtype %d", kvdtype);
    GemvParams p = {};
    p.W = Wqkv; p.N = N; p.K = K; p.x = x; p.B = B; p.norm_w = norm_w; p.eps = eps;
    p.n_heads = n_heads; p.n_kv = n_kv; p.head_dim = head_dim; p.pos = pos;
    p.rope_cos = rope_cos; p.rope_sin = rope_sin; p.q_out = q_out; p.k_cache = k_cache; p.v_cache = v_cache;
    p.kvdtype = kvdtype; p.page_table = page_table; p.max_pages = max_pages; p.page_size = page_size;
    return run_chunks(wdtype, EK_QKV, p, (cudaStream_t)stream, 0);
}

// Engine-internal entry points: a device status word for out-of-range positions and the
// L2 prefetch hint for the weights of the next kernel in the decode step.
namespace vsl {
bool tc_route_taken(const TcRoute* tc, int wdtype, int N, int K, int B) {
    return tc && tc->ws && B >= tc->min_batch && tc_supported(wdtype, N, K, B) && tc->bytes >= tc_workspace_bytes(N, K, B);
}

int gemv_hint(int wdtype, const void* W, int N, int K, const float* x, int B, float* y, int epilogue,
              const float* norm_w, float eps, const void* pf_ptr, size_t pf_bytes, cudaStream_t stream,
              const TcRoute* tc, bool x_presplit, const void* x2_in, void* x2_out) {
    int rc = check_common(wdtype, W, N, K, x, B);
    if (rc) return rc;
    if (x_presplit && (norm_w || !tc_route_taken(tc, wdtype, N, K, B)))
        return set_error(VSL_ERR_INVALID, "gemv: pre-split activations need the tensor-core route and no norm");
    if (x2_out && (epilogue != VSL_EPI_SWIGLU || !tc_route_taken(tc, wdtype, N, K, B)))
        return set_error(VSL_ERR_INVALID, "gemv: a split output needs the SwiGLU epilogue on the tensor-core route");
    GemvParams p = {};
    p.W = W; p.N = N; p.K = K; p.x = x; p.B = B; p.y = y; p.norm_w = norm_w; p.eps = eps;
    p.pf_ptr = pf_ptr; p.pf_bytes = pf_bytes;
    p.x_presplit = x_presplit ? 1 : 0;
    p.x2_in = x2_in;
    p.x2_out = x2_out;
    p.x2_out_rows = x2_out ? (int)tc_split_rows(B) : 0;
    p.x2_out_bf16 = wdtype == VSL_BF16 ? 1 : 0;
    int kind = epilogue == VSL_EPI_ADD ? EK_ADD : epilogue == VSL_EPI_SWIGLU ? EK_SWIGLU : EK_STORE;
    return run_chunks(wdtype, kind, p, stream, epilogue == VSL_EPI_SWIGLU ? N / 2 : N, tc);
}

int lm_head_hint(int wdtype, const void* W, int V_local, int K, const float* x, const float* norm_w, float eps, int B,
                 float* logits, unsigned long long* slots, int vocab_offset, float temperature, uint64_t seed,
                 const int32_t* step_counter, const void* pf_ptr, size_t pf_bytes, cudaStream_t stream,
                 const TcRoute* tc) {
    GemvParams p = {};
    p.W = W; p.N = V_local; p.K = K; p.x = x; p.B = B; p.y = logits; p.norm_w = norm_w; p.eps = eps;
    p.slots = slots; p.vocab_offset = vocab_offset;
    p.inv_temp = temperature > 0.0f ? 1.0f / temperature : 0.0f;
    p.seed = seed; p.step_counter = step_counter;
    p.pf_ptr = pf_ptr; p.pf_bytes = pf_bytes;
    return run_chunks(wdtype, EK_LMHEAD, p, stream, V_local, tc);
}

int qkv_rope_append_status(int wdtype, const void* Wqkv, int n_heads, int n_kv, int head_dim, int K,
                           const float* x, const float* norm_w, float eps, int B, const int32_t* pos,
                           const float* rope_cos, const float* rope_sin, float* q_out, void* k_cache,
                           void* v_cache, int kvdtype, const int32_t* page_table, int max_pages, int page_size,
                           int* status, cudaStream_t stream, const void* pf_ptr, size_t pf_bytes,
                           const TcRoute* tc) {
    GemvParams p = {};
    p.W = Wqkv; p.N = (n_heads + 2 * n_kv) * head_dim; p.K = K; p.x = x; p.B = B; p.norm_w = norm_w; p.eps = eps;
    p.n_heads = n_heads; p.n_kv = n_kv; p.head_dim = head_dim; p.pos = pos;
    p.rope_cos = rope_cos; p.rope_sin = rope_sin; p.q_out = q_out; p.k_cache = k_cache; p.v_cache = v_cache;
    p.kvdtype = kvdtype; p.page_table = page_table; p.max_pages = max_pages; p.page_size = page_size;
    p.status = status;
    p.pf_ptr = pf_ptr; p.pf_bytes = pf_bytes;
    return run_chunks(wdtype, EK_QKV, p, stream, 0, tc);
}
}  // namespace vsl

extern "C" int vsl_lm_head_sample(int wdtype, const void* W, int V_local, int K, const float* x,
                                  const float* norm_w, float eps, int B, float* logits,
                                  unsigned long long* argmax_slots, int vocab_offset, float temperature,
                                  uint64_t seed, const int32_t* step_counter, void* stream) {
    int rc = check_common(wdtype, W, V_local, K, x, B);
    if (rc) return rc;
    if (!logits || !argmax_slots) return set_error(VSL_ERR_INVALID, "lm_head: null logits or slots");
    if (temperature > 0.0f && !step_counter)
        return set_error(VSL_ERR_INVALID, "lm_head: sampling needs a device step counter");
    GemvParams p = {};
    p.W = W; p.N = V_local; p.K = K; p.x = x; p.B = B; p.y = logits; p.norm_w = norm_w; p.eps = eps;
    p.slots = argmax_slots; p.vocab_offset = vocab_offset;
    p.inv_temp = temperature > 0.0f ? 1.0f / temperature : 0.0f;
    p.seed = seed; p.step_counter = step_counter;
    return run_chunks(wdtype, EK_LMHEAD, p, (cudaStream_t)stream, V_local);
}
