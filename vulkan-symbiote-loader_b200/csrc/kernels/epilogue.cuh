// Projection epilogues shared by the per-op GEMV kernels and the fused decode step:
// residual add, SwiGLU, RoPE + paged KV append, lm_head logits + argmax/Gumbel folding.
#pragma once
#include "common.cuh"
#include "p2p_allreduce.h"

namespace vsl {

enum EpiKind { EK_STORE = 0, EK_ADD = 1, EK_SWIGLU = 2, EK_QKV = 3, EK_LMHEAD = 4 };

struct GemvParams {
    const void* W;
    int N, K;
    const float* x;
    int B;
    float* y;
    const float* norm_w;
    float eps;
    // QKV + RoPE + KV append
    int n_heads, n_kv, head_dim;
    const int32_t* pos;
    const float* rope_cos;
    const float* rope_sin;
    float* q_out;
    void* k_cache;
    void* v_cache;
    int kvdtype;
    const int32_t* page_table;
    int max_pages, page_size;
    // lm_head sampler
    unsigned long long* slots;
    int vocab_offset;
    float inv_temp;
    unsigned long long seed;
    const int32_t* step_counter;
    int* status;
    // L2 prefetch hint: weights of the kernel that follows; each CTA requests its share
    // once its own rows are done, filling the tail of this launch
    const void* pf_ptr;
    size_t pf_bytes;
    unsigned trace_id;  // launch id of the trace build (unused otherwise)
    // tensor-core route only: the split activations are already there (written by the producing
    // kernel: at x2_in, or at the workspace start when x2_in is null), so no activation-split
    // launch precedes the GEMM
    int x_presplit;
    const void* x2_in;
    // EK_SWIGLU on the tensor-core route: write the output as the next projection's split
    // activations instead of y (hi rows from 0, lo rows from x2_out_rows; N / 2 columns)
    void* x2_out;
    int x2_out_rows, x2_out_bf16;
};

__device__ __forceinline__ float silu_f(float z) { return z / (1.0f + expf(-z)); }

__device__ __forceinline__ unsigned long long smix64(unsigned long long z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// Gumbel(0,1) noise for (seed, step, b, index): -log(-log(u)), u in (0,1).
__device__ __forceinline__ float gumbel(unsigned long long seed, int step, int b, uint32_t idx) {
    unsigned long long h = smix64(smix64(seed ^ ((unsigned long long)step * 0x9E3779B97F4A7C15ull)) +
                                  (((unsigned long long)b << 32) | idx));
    float u = ((float)(h >> 40) + 0.5f) * (1.0f / 16777216.0f);
    return -logf(-logf(u));
}

// Values an epilogue reads from global memory, fetched ahead of the dot products so that their
// latency overlaps the weight stream: the residual pair (EK_ADD) or the RoPE cos/sin of the
// pair (EK_QKV), plus the sequence's position and its KV page.
struct EpiPre {
    float a0, a1;
    int pos, page;
};

// Position of sequence b and the page that holds it (page -1 when the position is outside the
// cache; the epilogue then records VSL_ERR_BOUNDS).
__device__ __forceinline__ void epi_pos_page(const GemvParams& p, int b, int& pos, int& page) {
    pos = p.pos[b];
    page = (pos < 0 || pos >= p.max_pages * p.page_size) ? -1
                                                         : p.page_table[(size_t)b * p.max_pages + pos / p.page_size];
}

template <int EK>
__device__ __forceinline__ EpiPre epi_fetch(const GemvParams& p, int b, int r0, bool has1, int pos, int page) {
    EpiPre e = {0.0f, 0.0f, pos, page};
    if (EK == EK_ADD) {  // the residual may have been written by another SM: read it from L2
        const float* y0 = p.y + (size_t)b * p.N + r0;
        e.a0 = __ldcg(y0);
        if (has1) e.a1 = __ldcg(y0 + 1);
    } else if (EK == EK_QKV) {
        const int hd = p.head_dim;
        if (page >= 0 && r0 < (p.n_heads + p.n_kv) * hd) {
            const int half = hd >> 1;
            const size_t t = (size_t)pos * half + ((r0 % hd) >> 1);
            e.a0 = p.rope_cos[t];
            e.a1 = p.rope_sin[t];
        }
    }
    return e;
}

// Epilogue of one row pair (r0 even, r0 + 1 present when has1) for activation row b, given
// its fetched inputs; `unit` is the pair index r0 / 2. `best` accumulates the lm_head argmax key.
template <int EK>
__device__ __forceinline__ void epi_apply(const GemvParams& p, const EpiPre& e, int b, int r0, int unit, bool has1,
                                          float s0, float s1, unsigned long long& best, int step) {
    const int N = p.N;
    if (EK == EK_STORE) {
        p.y[(size_t)b * N + r0] = s0;
        if (has1) p.y[(size_t)b * N + r0 + 1] = s1;
    } else if (EK == EK_ADD) {
        float* y0 = p.y + (size_t)b * N + r0;
        *y0 = e.a0 + s0;
        if (has1) y0[1] = e.a1 + s1;
    } else if (EK == EK_SWIGLU) {
        const float v = silu_f(s0) * s1;
        if (p.x2_out) {  // as hi / lo 16-bit halves of the next projection's split tile
            const size_t K2 = (size_t)(N >> 1);
            const size_t ih = (size_t)b * K2 + unit, il = ((size_t)p.x2_out_rows + b) * K2 + unit;
            if (p.x2_out_bf16) {
                const __nv_bfloat16 h = __float2bfloat16_rn(v);
                static_cast<__nv_bfloat16*>(p.x2_out)[ih] = h;
                static_cast<__nv_bfloat16*>(p.x2_out)[il] = __float2bfloat16_rn(v - __bfloat162float(h));
            } else {
                const __half h = __float2half_rn(v);
                static_cast<__half*>(p.x2_out)[ih] = h;
                static_cast<__half*>(p.x2_out)[il] = __float2half_rn(v - __half2float(h));
            }
        } else {
            p.y[(size_t)b * (N >> 1) + unit] = v;
        }
    } else if (EK == EK_QKV) {
        const int hd = p.head_dim;
        const int qd = p.n_heads * hd, kvd = p.n_kv * hd;
        if (e.page < 0) {
            if (p.status) atomicCAS(p.status, 0, VSL_ERR_BOUNDS);
            return;
        }
        const int el = r0 % hd;  // even
        float o0 = s0, o1 = s1;
        if (r0 < qd + kvd) {  // rotate q and k: adjacent pair (el, el+1)
            o0 = __fsub_rn(__fmul_rn(s0, e.a0), __fmul_rn(s1, e.a1));
            o1 = __fadd_rn(__fmul_rn(s0, e.a1), __fmul_rn(s1, e.a0));
        }
        if (r0 < qd) {
            p.q_out[(size_t)b * qd + r0] = o0;
            p.q_out[(size_t)b * qd + r0 + 1] = o1;
        } else {
            const bool is_v = r0 >= qd + kvd;
            const int rr = is_v ? r0 - qd - kvd : r0 - qd;
            const int g = rr / hd;
            const size_t idx = (((size_t)e.page * p.n_kv + g) * p.page_size + (e.pos % p.page_size)) * hd + el;
            void* cache = is_v ? p.v_cache : p.k_cache;
            kv_put(cache, idx, o0, p.kvdtype);
            kv_put(cache, idx + 1, o1, p.kvdtype);
        }
    } else if (EK == EK_LMHEAD) {
        p.y[(size_t)b * N + r0] = s0;
        if (has1) p.y[(size_t)b * N + r0 + 1] = s1;
        float c0 = s0, c1 = s1;
        const uint32_t g0 = (uint32_t)(p.vocab_offset + r0);
        if (p.inv_temp > 0.0f) {
            c0 = s0 * p.inv_temp + gumbel(p.seed, step, b, g0);
            c1 = s1 * p.inv_temp + gumbel(p.seed, step, b, g0 + 1);
        }
        if (c0 == c0) best = max(best, pack_argmax(c0, g0));
        if (has1 && c1 == c1) best = max(best, pack_argmax(c1, g0 + 1));
    }
}

// Fetch + apply in one go (the per-operation GEMV kernels, whose epilogue follows the sums).
template <int EK>
__device__ __forceinline__ void gemv_pair_epilogue(const GemvParams& p, int b, int r0, int unit, bool has1, float s0,
                                                   float s1, unsigned long long& best, int step) {
    int pos = 0, page = 0;
    if (EK == EK_QKV) epi_pos_page(p, b, pos, page);
    const EpiPre e = epi_fetch<EK>(p, b, r0, has1, pos, page);
    epi_apply<EK>(p, e, b, r0, unit, has1, s0, s1, best, step);
}

}  // namespace vsl
