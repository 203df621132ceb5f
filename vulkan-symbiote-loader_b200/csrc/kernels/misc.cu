// Small decode kernels: embedding gather, standalone RMSNorm, argmax, the seeded synthetic
// initialiser, and the end-of-step token bookkeeping.
#include <atomic>
#include <type_traits>
#include <cuda_runtime.h>
#include <math_constants.h>

#include "common.cuh"
#include "quant_layout.h"
#include "launch.cuh"

namespace vsl {

// ---------------------------------------------------------------------------------------
// launch helpers
// ---------------------------------------------------------------------------------------
static std::atomic<bool> g_pdl{true};
bool pdl_enabled() { return g_pdl.load(std::memory_order_relaxed); }
void set_pdl_enabled(bool on) { g_pdl.store(on, std::memory_order_relaxed); }

int sm_count() {
    static thread_local int cached_dev = -1, cached = 148;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev != cached_dev) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && n > 0) cached = n;
        cached_dev = dev;
    }
    return cached;
}

// ---------------------------------------------------------------------------------------
// embedding gather: x[b][j] = E[min(id, V-1)][j] (embedding_lookup.comp:29-40)
// ---------------------------------------------------------------------------------------
template <typename WT>
__global__ void vsl_embed_kernel(const WT* __restrict__ table, int V, int d, const int32_t* __restrict__ ids,
                             float* __restrict__ x, unsigned long long* slots) {
    pdl_wait();
    pdl_launch_dependents();
    const int b = blockIdx.x;
    int id = ids[b];
    if (id < 0) id = 0;
    if (id > V - 1) id = V - 1;
    const WT* row = table + (size_t)id * d;
    for (int j = threadIdx.x; j < d; j += blockDim.x) x[(size_t)b * d + j] = WTraits<WT>::load(row, j);
    if (slots && threadIdx.x == 0) slots[b] = 0ull;  // argmax slot of this step's sampler
}

// Block-quantized table (device row layout of quant_layout.h): element j of the row is
// quant(j) * d(j / 32) in fp32 (Q4_1: then + m(j / 32) in fp32), the reference's
// dequantisation (GGUFLoader.cpp:1150-1207).
template <int QT>
__global__ void vsl_embed_q_kernel(const unsigned char* __restrict__ table, int V, int d, const int32_t* __restrict__ ids,
                               float* __restrict__ x, unsigned long long* slots) {
    pdl_wait();
    pdl_launch_dependents();
    const int b = blockIdx.x;
    int id = ids[b];
    if (id < 0) id = 0;
    if (id > V - 1) id = V - 1;
    const unsigned char* row = table + (size_t)id * weight_row_bytes(QT, d);
    const __half* sc = reinterpret_cast<const __half*>(row + quant_bytes(QT, d));
    const __half* mn = sc + scale_bytes(d) / 2;  // Q4_1 minimums follow the scales
    for (int j = threadIdx.x; j < d; j += blockDim.x) {
        const float s = __half2float(sc[j / QBLK]);
        int q;
        if (QT == VSL_Q8_0) {
            q = (int)(signed char)row[j];
        } else {
            const int blk = j / QBLK, i = j % QBLK;
            const unsigned char byte = row[blk * 16 + (i & 15)];
            q = (int)(i < 16 ? (byte & 15) : (byte >> 4)) - (QT == VSL_Q4_1 ? 0 : 8);
        }
        x[(size_t)b * d + j] = QT == VSL_Q4_1 ? __fadd_rn(__fmul_rn((float)q, s), __half2float(mn[j / QBLK]))
                                              : (float)q * s;
    }
    if (slots && threadIdx.x == 0) slots[b] = 0ull;
}

int embed_impl(int dtype, const void* table, int V, int d, const int32_t* ids, int B, float* x,
               unsigned long long* slots, cudaStream_t st) {
    if (!table || !ids || !x || V <= 0 || d <= 0 || B <= 0) return set_error(VSL_ERR_INVALID, "embed: bad arguments");
    dim3 grid(B), block(256);
    if (is_quant(dtype) && d % QBLK) return set_error(VSL_ERR_INVALID, "embed: quantized rows need d %% 32 == 0");
    switch (dtype) {
        case VSL_Q8_0:
            return launch_status(launch_k(vsl_embed_q_kernel<VSL_Q8_0>, grid, block, 0, st, (const unsigned char*)table, V,
                                          d, ids, x, slots),
                                 "embed");
        case VSL_Q4_0:
            return launch_status(launch_k(vsl_embed_q_kernel<VSL_Q4_0>, grid, block, 0, st, (const unsigned char*)table, V,
                                          d, ids, x, slots),
                                 "embed");
        case VSL_Q4_1:
            return launch_status(launch_k(vsl_embed_q_kernel<VSL_Q4_1>, grid, block, 0, st, (const unsigned char*)table, V,
                                          d, ids, x, slots),
                                 "embed");
        case VSL_F32:
            return launch_status(launch_k(vsl_embed_kernel<float>, grid, block, 0, st, (const float*)table, V, d, ids, x, slots),
                                 "embed");
        case VSL_F16:
            return launch_status(
                launch_k(vsl_embed_kernel<__half>, grid, block, 0, st, (const __half*)table, V, d, ids, x, slots), "embed");
        case VSL_BF16:
            return launch_status(launch_k(vsl_embed_kernel<__nv_bfloat16>, grid, block, 0, st,
                                          (const __nv_bfloat16*)table, V, d, ids, x, slots),
                                 "embed");
        default: return set_error(VSL_ERR_UNSUPPORTED, "embed: dtype %d", dtype);
    }
}

// ---------------------------------------------------------------------------------------
// RMSNorm (rms_norm.comp:24-34): one CTA per row
// ---------------------------------------------------------------------------------------
__global__ void vsl_rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w, int d, float eps,
                               float* __restrict__ y) {
    __shared__ float red[32];
    pdl_wait();
    pdl_launch_dependents();
    const int b = blockIdx.x;
    const float* xb = x + (size_t)b * d;
    float ss = 0.0f;
    for (int j = threadIdx.x; j < d; j += blockDim.x) ss += xb[j] * xb[j];
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.0f;
    for (int i = 0; i < (int)(blockDim.x >> 5); i++) tot += red[i];
    const float den = sqrtf(tot / (float)d + eps);
    for (int j = threadIdx.x; j < d; j += blockDim.x) y[(size_t)b * d + j] = xb[j] / den * w[j];
}

// ---------------------------------------------------------------------------------------
// argmax over fp32 rows (first maximum), one CTA per row
// ---------------------------------------------------------------------------------------
__global__ void vsl_argmax_kernel(const float* __restrict__ logits, int V, int32_t* __restrict__ out) {
    __shared__ unsigned long long red[32];
    pdl_wait();
    pdl_launch_dependents();
    const int b = blockIdx.x;
    unsigned long long best = 0ull;
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
        float v = logits[(size_t)b * V + i];
        if (v == v) best = max(best, pack_argmax(v, (uint32_t)i));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int i = 1; i < (int)(blockDim.x >> 5); i++) best = max(best, red[i]);
        best = max(best, red[0]);
        out[b] = best ? (int32_t)unpack_argmax_idx(best) : 0;
    }
}

// ---------------------------------------------------------------------------------------
// seeded synthetic initialiser (same definition as vsl/synth.py)
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ unsigned long long smix(unsigned long long z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

template <typename T>
__global__ void vsl_synth_kernel(T* __restrict__ out, unsigned long long base, unsigned long long start,
                             unsigned long long n, float c) {
    for (unsigned long long j = (unsigned long long)blockIdx.x * blockDim.x + threadIdx.x; j < n;
         j += (unsigned long long)gridDim.x * blockDim.x) {
        const unsigned long long h = smix(base + start + j);
        const int s = (int)(h & 0xffffu) + (int)((h >> 16) & 0xffffu) + (int)((h >> 32) & 0xffffu) + (int)(h >> 48) -
                      131070;
        const float v = __fmul_rn((float)s, c);
        if constexpr (std::is_same<T, __half>::value) out[j] = __float2half_rn(v);
        else if constexpr (std::is_same<T, __nv_bfloat16>::value) out[j] = __float2bfloat16_rn(v);
        else out[j] = v;
    }
}

static unsigned long long host_smix(unsigned long long z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

int synth_impl(void* dst, int dtype, uint64_t seed, uint64_t tid, uint64_t start, uint64_t n, double sigma,
               cudaStream_t st) {
    if (!dst) return set_error(VSL_ERR_INVALID, "synth_fill: null destination");
    if (n == 0) return VSL_OK;
    const unsigned long long base = host_smix(seed ^ (tid * 0xD1B54A32D192ED03ull));
    const float c = (float)(1.7320508075688772 * sigma / 65536.0);
    unsigned long long blocks = (n + 255) / 256;
    if (blocks > (unsigned long long)sm_count() * 16) blocks = (unsigned long long)sm_count() * 16;
    dim3 grid((unsigned)blocks), block(256);
    cudaError_t e;
    switch (dtype) {
        case VSL_F32: e = launch_k(vsl_synth_kernel<float>, grid, block, 0, st, (float*)dst, base, start, n, c); break;
        case VSL_F16: e = launch_k(vsl_synth_kernel<__half>, grid, block, 0, st, (__half*)dst, base, start, n, c); break;
        case VSL_BF16:
            e = launch_k(vsl_synth_kernel<__nv_bfloat16>, grid, block, 0, st, (__nv_bfloat16*)dst, base, start, n, c);
            break;
        default: return set_error(VSL_ERR_UNSUPPORTED, "synth_fill: dtype %d", dtype);
    }
    return launch_status(e, "synth_fill");
}

// 2-D slice of a seeded tensor: element (i, j) of the slice is global element
// (row0 + i) * src_cols + col0 + j, written to dst[i * dst_ld + j] (tensor-parallel shards
// and the interleaved gate/up layout are generated in place).
template <typename T>
__global__ void vsl_synth2d_kernel(T* __restrict__ dst, size_t dst_ld, unsigned long long base, size_t row0,
                               size_t nrows, size_t src_cols, size_t col0, size_t ncols, float c) {
    const size_t total = nrows * ncols;
    for (size_t j = (size_t)blockIdx.x * blockDim.x + threadIdx.x; j < total; j += (size_t)gridDim.x * blockDim.x) {
        const size_t r = j / ncols, cc = j - r * ncols;
        const unsigned long long gi = (unsigned long long)((row0 + r) * src_cols + col0 + cc);
        const unsigned long long h = smix(base + gi);
        const int s = (int)(h & 0xffffu) + (int)((h >> 16) & 0xffffu) + (int)((h >> 32) & 0xffffu) + (int)(h >> 48) -
                      131070;
        const float v = __fmul_rn((float)s, c);
        T* o = dst + r * dst_ld + cc;
        if constexpr (std::is_same<T, __half>::value) *o = __float2half_rn(v);
        else if constexpr (std::is_same<T, __nv_bfloat16>::value) *o = __float2bfloat16_rn(v);
        else *o = v;
    }
}

// Seeded block-quantized tensor, written in the device row layout (row pitch dst_ld bytes):
// global element gi = row * src_cols + col has quant h(gi) (Q8_0: h % 255 - 127; Q4_0: nibble
// 1 + h % 15, value nibble - 8, symmetric like Q8_0; Q4_1: nibble h % 16) and global block
// gb = row * (src_cols / 32) + col / 32 the scale d = fp16(m * c), m = 49152 + (h'(gb) & 0x7fff),
// h' from a second stream of the same tensor; a Q4_1 block's minimum is fp16(-7.5 * d).
template <int QT>
__global__ void vsl_synthq_kernel(unsigned char* __restrict__ dst, size_t dst_ld, unsigned long long base,
                              unsigned long long sbase, size_t row0, size_t nrows, size_t src_cols, size_t col0,
                              size_t ncols, float c) {
    const size_t qb = quant_bytes(QT, ncols), nblk = ncols / QBLK;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    const size_t t0 = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    for (size_t j = t0; j < nrows * qb; j += stride) {  // one quant byte per iteration
        const size_t r = j / qb, cb = j - r * qb;
        const size_t grow = (row0 + r) * src_cols + col0;
        unsigned char out;
        if (QT == VSL_Q8_0) {
            const unsigned long long h = smix(base + grow + cb);
            out = (unsigned char)(signed char)((int)(h % 255ull) - 127);
        } else {
            const size_t blk = cb / 16, i = cb % 16;  // byte i holds elements i and i + 16 of the block
            const unsigned long long h0 = smix(base + grow + blk * QBLK + i);
            const unsigned long long h1 = smix(base + grow + blk * QBLK + i + 16);
            out = QT == VSL_Q4_1 ? (unsigned char)((h0 % 16ull) | ((h1 % 16ull) << 4))
                                 : (unsigned char)((1ull + h0 % 15ull) | ((1ull + h1 % 15ull) << 4));
        }
        dst[r * dst_ld + cb] = out;
    }
    const size_t sb = scale_bytes(ncols) / 2;  // scale slots, padding included
    for (size_t j = t0; j < nrows * sb; j += stride) {
        const size_t r = j / sb, k = j - r * sb;
        __half v = __float2half_rn(0.0f);
        if (k < nblk) {
            const unsigned long long gb = (row0 + r) * (src_cols / QBLK) + col0 / QBLK + k;
            const unsigned long long h = smix(sbase + gb);
            v = __float2half_rn(__fmul_rn((float)(49152u + (unsigned)(h & 0x7fffull)), c));
        }
        reinterpret_cast<__half*>(dst + r * dst_ld + qb)[k] = v;
        if (QT == VSL_Q4_1)  // minimum: fp16(-7.5 * d), +0 in the padding
            reinterpret_cast<__half*>(dst + r * dst_ld + qb + 2 * sb)[k] =
                k < nblk ? __float2half_rn(__fmul_rn(-7.5f, __half2float(v))) : __float2half_rn(0.0f);
    }
}

// scale-stream seed of a quantized synthetic tensor
static unsigned long long synthq_scale_base(uint64_t seed, uint64_t tid) {
    return host_smix(seed ^ ((tid ^ 0x5CA1E5ull) * 0xD1B54A32D192ED03ull));
}
// fp32 factor of the block scales: d = m * c has mean ~ sigma / std(quant)
static float synthq_scale_c(int dtype, double sigma) {
    // std of U{-127..127}, U{-7..7}, U{0..15}
    const double sq = dtype == VSL_Q8_0 ? 73.6115932 : dtype == VSL_Q4_1 ? 4.6097722 : 4.3204938;
    return (float)(sigma / sq / 65536.0);
}

int synthq2d_impl(void* dst, int dtype, size_t dst_ld, uint64_t seed, uint64_t tid, size_t row0, size_t nrows,
                  size_t src_cols, size_t col0, size_t ncols, double sigma, cudaStream_t st) {
    if (!dst || !is_quant(dtype) || col0 % QBLK || ncols % QBLK || src_cols % QBLK || col0 + ncols > src_cols ||
        dst_ld < weight_row_bytes(dtype, ncols))
        return set_error(VSL_ERR_INVALID, "synthq2d: bad slice");
    if (nrows == 0 || ncols == 0) return VSL_OK;
    const unsigned long long base = host_smix(seed ^ (tid * 0xD1B54A32D192ED03ull));
    const unsigned long long sbase = synthq_scale_base(seed, tid);
    const float c = synthq_scale_c(dtype, sigma);
    dim3 grid((unsigned)(sm_count() * 16)), block(256);
    cudaError_t e = dtype == VSL_Q8_0
                        ? launch_k(vsl_synthq_kernel<VSL_Q8_0>, grid, block, 0, st, (unsigned char*)dst, dst_ld, base, sbase,
                                   row0, nrows, src_cols, col0, ncols, c)
                    : dtype == VSL_Q4_1
                        ? launch_k(vsl_synthq_kernel<VSL_Q4_1>, grid, block, 0, st, (unsigned char*)dst, dst_ld, base, sbase,
                                   row0, nrows, src_cols, col0, ncols, c)
                        : launch_k(vsl_synthq_kernel<VSL_Q4_0>, grid, block, 0, st, (unsigned char*)dst, dst_ld, base, sbase,
                                   row0, nrows, src_cols, col0, ncols, c);
    return launch_status(e, "synthq2d");
}

int synth2d_impl(void* dst, int dtype, size_t dst_ld, uint64_t seed, uint64_t tid, size_t row0, size_t nrows,
                 size_t src_cols, size_t col0, size_t ncols, double sigma, cudaStream_t st) {
    if (!dst || ncols > dst_ld || col0 + ncols > src_cols)
        return set_error(VSL_ERR_INVALID, "synth2d: bad slice");
    if (nrows == 0 || ncols == 0) return VSL_OK;
    const unsigned long long base = host_smix(seed ^ (tid * 0xD1B54A32D192ED03ull));
    const float c = (float)(1.7320508075688772 * sigma / 65536.0);
    dim3 grid((unsigned)(sm_count() * 16)), block(256);
    cudaError_t e;
    switch (dtype) {
        case VSL_F32:
            e = launch_k(vsl_synth2d_kernel<float>, grid, block, 0, st, (float*)dst, dst_ld, base, row0, nrows, src_cols,
                         col0, ncols, c);
            break;
        case VSL_F16:
            e = launch_k(vsl_synth2d_kernel<__half>, grid, block, 0, st, (__half*)dst, dst_ld, base, row0, nrows, src_cols,
                         col0, ncols, c);
            break;
        case VSL_BF16:
            e = launch_k(vsl_synth2d_kernel<__nv_bfloat16>, grid, block, 0, st, (__nv_bfloat16*)dst, dst_ld, base, row0,
                         nrows, src_cols, col0, ncols, c);
            break;
        default: return set_error(VSL_ERR_UNSUPPORTED, "synth2d: dtype %d", dtype);
    }
    return launch_status(e, "synth2d");
}

// ---------------------------------------------------------------------------------------
// end of a decode step: sampled id from the argmax slot, next input id (forced or
// sampled), token log, position advance and step counter
// ---------------------------------------------------------------------------------------
__global__ void vsl_finalize_kernel(const unsigned long long* __restrict__ slots, int B, int32_t* ids, int32_t* pos,
                                int32_t* step_counter, const int32_t* __restrict__ forced, const int32_t* n_forced,
                                int32_t* log, int log_cap, int32_t* sampled_out, int max_pos, int* status) {
    pdl_wait();
    pdl_launch_dependents();
    const int b = threadIdx.x;
    const int step = *step_counter;
    if (b < B) {
        const unsigned long long s = slots[b];
        const int32_t sampled = s ? (int32_t)unpack_argmax_idx(s) : 0;
        if (step < log_cap) log[(size_t)step * B + b] = sampled;
        sampled_out[b] = sampled;
        const int nf = *n_forced;
        ids[b] = (step + 1 < nf) ? forced[(size_t)(step + 1) * B + b] : sampled;
        // a full cache (pos == max_pos) is legal; a step that ran past it is not
        const int np = pos[b] + 1;
        if (np > max_pos && status) atomicCAS(status, 0, VSL_ERR_BOUNDS);
        pos[b] = np < max_pos ? np : max_pos;
    }
    __syncthreads();
    if (threadIdx.x == 0) *step_counter = step + 1;
}

int finalize_impl(const unsigned long long* slots, int B, int32_t* ids, int32_t* pos, int32_t* step_counter,
                  const int32_t* forced, const int32_t* n_forced, int32_t* log, int log_cap, int32_t* sampled_out,
                  int max_pos, int* status, cudaStream_t st) {
    if (B > 1024) return set_error(VSL_ERR_UNSUPPORTED, "finalize: batch %d > 1024", B);
    return launch_status(launch_k(vsl_finalize_kernel, dim3(1), dim3(B < 32 ? 32 : ((B + 31) / 32) * 32), 0, st, slots, B,
                                  ids, pos, step_counter, forced, n_forced, log, log_cap, sampled_out, max_pos, status),
                         "finalize");
}

// End of a prefill: sequence `seq` continues from position new_pos with the token sampled from
// the prompt's last logits (the argmax key in `slot`).
__global__ void vsl_prefill_finish_kernel(const unsigned long long* __restrict__ slot, int32_t* ids, int32_t* pos, int seq,
                                      int new_pos, int32_t* next_out) {
    pdl_wait();
    pdl_launch_dependents();
    if (threadIdx.x == 0) {
        const unsigned long long s = *slot;
        const int32_t id = s ? (int32_t)unpack_argmax_idx(s) : 0;
        ids[seq] = id;
        pos[seq] = new_pos;
        *next_out = id;
    }
}

int prefill_finish_impl(const unsigned long long* slot, int32_t* ids, int32_t* pos, int seq, int new_pos,
                        int32_t* next_out, cudaStream_t st) {
    return launch_status(launch_k(vsl_prefill_finish_kernel, dim3(1), dim3(32), 0, st, slot, ids, pos, seq, new_pos, next_out),
                         "prefill finish");
}

}  // namespace vsl

using namespace vsl;

extern "C" int vsl_embed_gather(int dtype, const void* table, int V, int d, const int32_t* ids, int B, float* x,
                                void* stream) {
    return embed_impl(dtype, table, V, d, ids, B, x, nullptr, (cudaStream_t)stream);
}

extern "C" int vsl_rmsnorm(const float* x, const float* w, int B, int d, float eps, float* y, void* stream) {
    if (!x || !w || !y || B <= 0 || d <= 0) return set_error(VSL_ERR_INVALID, "rmsnorm: bad arguments");
    return launch_status(launch_k(vsl_rmsnorm_kernel, dim3(B), dim3(256), 0, (cudaStream_t)stream, x, w, d, eps, y),
                         "rmsnorm");
}

extern "C" int vsl_argmax(const float* logits, int B, int V, int32_t* out_ids, void* stream) {
    if (!logits || !out_ids || B <= 0 || V <= 0) return set_error(VSL_ERR_INVALID, "argmax: bad arguments");
    return launch_status(launch_k(vsl_argmax_kernel, dim3(B), dim3(512), 0, (cudaStream_t)stream, logits, V, out_ids),
                         "argmax");
}

extern "C" int vsl_synth_fill_q(void* dst, int dtype, size_t row_pitch, uint64_t seed, uint64_t tensor_id,
                                size_t rows, size_t cols, double sigma, void* stream) {
    return vsl::synthq2d_impl(dst, dtype, row_pitch, seed, tensor_id, 0, rows, cols, 0, cols, sigma,
                              (cudaStream_t)stream);
}

extern "C" int vsl_synth_fill(void* dst, int dtype, uint64_t seed, uint64_t tensor_id, uint64_t start, uint64_t n,
                              double sigma, void* stream) {
    return synth_impl(dst, dtype, seed, tensor_id, start, n, sigma, (cudaStream_t)stream);
}
