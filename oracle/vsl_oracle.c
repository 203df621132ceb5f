/*
 * vsl_oracle.c -- CPU restatement of the Vulkan-Symbiote-Loader decode token loop.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the parity oracle and the timed CPU baseline.
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference legs
 * load it; the product library (libvsl.so) never links, calls or falls back to it.
 *
 * Parity status: the reference ships no golden vectors, known-answer tests or fixtures
 * for this path (vk_symbiote/tests/validation_tests.cpp only checks VkResult helpers) and
 * its own path cannot be built here (every translation unit includes <vulkan/vulkan.h>
 * through vk_symbiote/include/vk_symbiote/Common.h:21). Parity against the reference is
 * therefore UNPINNED by reference outputs; each function below follows the reference
 * source line it cites, and the whole oracle is cross-checked against an independent
 * float64 NumPy restatement (tests/golden/make_golden.py) and known-answer vectors
 * derived from the cited reference code.
 *
 * Decode math (one step, per sequence b at absolute position pos[b]):
 *   x   = E[min(id, V-1)]                          embedding_lookup.comp:29-40
 *   per layer l:
 *     n = x / sqrt(mean(x^2) + eps) * w_attn       rms_norm.comp:24-34
 *     q,k,v = n Wq^T, n Wk^T, n Wv^T               attention.comp:63-99 (GGUF [out][in] rows)
 *     RoPE adjacent pairs, f = theta^(-2i/hd)      Utils.cpp:101-110, fused_matmul_rope.comp:48-82
 *     append k,v at pos                            VulkanSymbioteEngine.cpp:41-54, attention.comp:101-108
 *     o_h = softmax(q_h K^T / sqrt(hd)) V,         attention.comp:116-189, kv = h*nkv/nh (:92)
 *     x  += o Wo^T                                 architecture_design.md:334-347 (residual)
 *     m  = rmsnorm(x, w_ffn)
 *     x  += (silu(m Wg^T) * (m Wu^T)) Wd^T         feed_forward.comp:21,38-61
 *   x = rmsnorm(x, w_out); logits = x Wout^T       final_linear.comp:38-86 (bias 0)
 *   id = first argmax (strict >)                   VulkanSymbioteEngine.cpp:1794-1804, Utils.cpp:174-184
 *
 * All arithmetic is fp32 with fp32 accumulation; fp16/bf16 weights are upcast exactly
 * (GGUFLoader.cpp:1225-1262 does the exact IEEE half->float). When the KV cache dtype is
 * fp16, K and V are rounded to fp16 (round-to-nearest-even) on append, exactly as the
 * device cache stores them.
 */
#define _GNU_SOURCE
#include <stdint.h>
#include <stdlib.h>
#include <stdio.h>
#include <string.h>
#include <math.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>
#ifdef _OPENMP
#include <omp.h>
#endif
#if defined(__F16C__) && defined(__AVX2__)
#include <immintrin.h>
#define ORC_HAVE_F16C 1
#endif

/* ggml tensor type ids (standard GGUF), used for weights and the KV cache */
enum { ORC_F32 = 0, ORC_F16 = 1, ORC_Q4_0 = 2, ORC_Q4_1 = 3, ORC_Q8_0 = 8, ORC_BF16 = 30 };
static inline int orc_is_quant(int dt) { return dt == ORC_Q4_0 || dt == ORC_Q4_1 || dt == ORC_Q8_0; }

/* ------------------------------------------------------------------------- */
/* number formats                                                            */
/* ------------------------------------------------------------------------- */

/* exact IEEE binary16 -> binary32 (GGUFLoader.cpp:1225-1262 restated) */
float orc_h2f(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu;
    uint32_t m = h & 0x3ffu;
    uint32_t bits;
    if (e == 0) {
        if (m == 0) {
            bits = sign;
        } else {
            int ee = 113; /* 127 - 15 + 1 */
            while (!(m & 0x400u)) { m <<= 1; ee--; }
            m &= 0x3ffu;
            bits = sign | ((uint32_t)ee << 23) | (m << 13);
        }
    } else if (e == 31) {
        bits = sign | 0x7f800000u | (m << 13);
    } else {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* binary32 -> binary16, round to nearest even */
uint16_t orc_f2h(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7fffffffu;
    if (ax > 0x7f800000u) return (uint16_t)(sign | 0x7e00u);       /* NaN */
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);      /* rounds to inf */
    if (ax < 0x38800000u) {                                         /* half subnormal / zero */
        float a;
        memcpy(&a, &ax, 4);
        float q = nearbyintf(a * 16777216.0f);                      /* units of 2^-24, RNE */
        return (uint16_t)(sign | (uint32_t)q);
    }
    uint32_t e = (ax >> 23) - 112u;
    uint32_t m = ax & 0x7fffffu;
    uint32_t hm = m >> 13, rem = m & 0x1fffu;
    uint32_t h = (e << 10) | hm;
    if (rem > 0x1000u || (rem == 0x1000u && (hm & 1u))) h++;
    return (uint16_t)(sign | h);
}

float orc_bf2f(uint16_t b) {
    uint32_t bits = (uint32_t)b << 16;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

uint16_t orc_f2bf(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    if ((x & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((x >> 16) | 0x40u);
    x += 0x7fffu + ((x >> 16) & 1u);
    return (uint16_t)(x >> 16);
}

static inline float load_elem(const void* p, int dtype, size_t i) {
    switch (dtype) {
        case ORC_F16: return orc_h2f(((const uint16_t*)p)[i]);
        case ORC_BF16: return orc_bf2f(((const uint16_t*)p)[i]);
        default: return ((const float*)p)[i];
    }
}

/* ------------------------------------------------------------------------- */
/* seeded synthetic tensors (same definition as vsl/synth.py and the device  */
/* initialiser): Irwin-Hall(4) of 16-bit lanes of splitmix64, scaled exactly */
/* ------------------------------------------------------------------------- */

static inline uint64_t smix(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

uint64_t orc_synth_u64(uint64_t seed, uint64_t tensor_id, uint64_t i) {
    uint64_t base = smix(seed ^ (tensor_id * 0xD1B54A32D192ED03ull));
    return smix(base + i);
}

float orc_synth_scale(double sigma) { return (float)(1.7320508075688772 * sigma / 65536.0); }

static inline float synth_val(uint64_t base, uint64_t i, float c) {
    uint64_t h = smix(base + i);
    int s = (int)(h & 0xffffu) + (int)((h >> 16) & 0xffffu) + (int)((h >> 32) & 0xffffu) +
            (int)(h >> 48) - 131070;
    return (float)s * c;
}

/* fill n elements [start, start+n) of tensor `tensor_id` into out (dtype) */
void orc_synth_fill(uint64_t seed, uint64_t tensor_id, uint64_t start, uint64_t n, double sigma,
                    int dtype, void* out) {
    uint64_t base = smix(seed ^ (tensor_id * 0xD1B54A32D192ED03ull));
    float c = orc_synth_scale(sigma);
#pragma omp parallel for schedule(static)
    for (int64_t j = 0; j < (int64_t)n; j++) {
        float v = synth_val(base, start + (uint64_t)j, c);
        if (dtype == ORC_F16) ((uint16_t*)out)[j] = orc_f2h(v);
        else if (dtype == ORC_BF16) ((uint16_t*)out)[j] = orc_f2bf(v);
        else ((float*)out)[j] = v;
    }
}

/* ------------------------------------------------------------------------- */
/* block-quantized weights (GGUF Q8_0 / Q4_0 / Q4_1, 32 elements per block)  */
/* ------------------------------------------------------------------------- */

/* GGUFLoader.cpp dequantize_tensor: per block, d = fp16_to_fp32(first two bytes) (:1131-1147,
 * exact IEEE half), then value = q * d in fp32: Q8_0 q = int8 qs[i] (:1185-1200); Q4_0
 * q = nibble - 8 (:1150-1162); Q4_1 (:1173-1196) blocks carry a second fp16, the minimum m,
 * after d, and value = (float)nibble * d + m (an fp32 multiply, then an fp32 add). The reference
 * reads the nibbles of byte i as elements 2i (low) and 2i + 1 (high) (:1154-1159, :1187-1191);
 * ggml's format defines them as elements i and i + 16. Both orders are restated: legacy_q4 = 1
 * follows the reference loader, 0 the format. */
void orc_dequant_blocks(int dtype, const void* blocks, size_t n_elems, int legacy_q4, float* out) {
    const uint8_t* p = (const uint8_t*)blocks;
    const size_t bb = dtype == ORC_Q8_0 ? 34 : dtype == ORC_Q4_1 ? 20 : 18;
    for (size_t b = 0; b * 32 < n_elems; b++, p += bb) {
        const float d = orc_h2f((uint16_t)(p[0] | (p[1] << 8)));
        float* o = out + b * 32;
        if (dtype == ORC_Q8_0) {
            for (int i = 0; i < 32; i++) o[i] = (float)(int8_t)p[2 + i] * d;
        } else if (dtype == ORC_Q4_1) {
            const float m = orc_h2f((uint16_t)(p[2] | (p[3] << 8)));
            for (int i = 0; i < 16; i++) {
                const int lo = p[4 + i] & 0x0F, hi = (p[4 + i] >> 4) & 0x0F;
                const float vlo = (float)lo * d, vhi = (float)hi * d;
                if (legacy_q4) { o[2 * i] = vlo + m; o[2 * i + 1] = vhi + m; }
                else { o[i] = vlo + m; o[i + 16] = vhi + m; }
            }
        } else {
            for (int i = 0; i < 16; i++) {
                const int lo = (p[2 + i] & 0x0F) - 8, hi = ((p[2 + i] >> 4) & 0x0F) - 8;
                if (legacy_q4) { o[2 * i] = (float)lo * d; o[2 * i + 1] = (float)hi * d; }
                else { o[i] = (float)lo * d; o[i + 16] = (float)hi * d; }
            }
        }
    }
}

/* Seeded block-quantized tensor [rows][cols], dequantized (the device initialiser writes the
 * same quants and scales in its packed layout): element gi = r * cols + c has quant
 * h(gi) % 255 - 127 (Q8_0), (1 + h(gi) % 15) - 8 (Q4_0) or h(gi) % 16 (Q4_1); block
 * gb = r * (cols / 32) + c / 32 has scale d = fp16(m * k), m = 49152 + (h'(gb) & 0x7fff), h' the
 * tensor's second stream and k = sigma / std(quant) / 65536 in fp32; a Q4_1 block's minimum is
 * fp16(-7.5 * d) (so its values are centred), value = quant * d + minimum. */
void orc_synthq_dequant(uint64_t seed, uint64_t tensor_id, size_t rows, size_t cols, double sigma, int dtype,
                        float* out) {
    const uint64_t base = smix(seed ^ (tensor_id * 0xD1B54A32D192ED03ull));
    const uint64_t sbase = smix(seed ^ ((tensor_id ^ 0x5CA1E5ull) * 0xD1B54A32D192ED03ull));
    const double sq = dtype == ORC_Q8_0 ? 73.6115932 : dtype == ORC_Q4_1 ? 4.6097722 : 4.3204938;
    const float k = (float)(sigma / sq / 65536.0);
    const size_t nb = cols / 32;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < (int64_t)rows; r++)
        for (size_t b = 0; b < nb; b++) {
            const uint64_t hs = smix(sbase + (uint64_t)r * nb + b);
            const float m = (float)(49152u + (unsigned)(hs & 0x7fffull));
            const float d = orc_h2f(orc_f2h(m * k));
            const float mn = orc_h2f(orc_f2h(-7.5f * d));
            for (int i = 0; i < 32; i++) {
                const size_t gi = (size_t)r * cols + b * 32 + (size_t)i;
                const uint64_t h = smix(base + gi);
                if (dtype == ORC_Q4_1) {
                    const float v = (float)(int)(h % 16ull) * d;
                    out[gi] = v + mn;
                    continue;
                }
                const int q = dtype == ORC_Q8_0 ? (int)(h % 255ull) - 127 : (int)(1ull + h % 15ull) - 8;
                out[gi] = (float)q * d;
            }
        }
}

/* prompt ids: uniform in [0, V) (modulo mapping of a 64-bit draw) */
void orc_synth_ids(uint64_t seed, uint64_t stream, int n, int vocab, int32_t* out) {
    for (int i = 0; i < n; i++)
        out[i] = (int32_t)(orc_synth_u64(seed, 0xFFFF0000ull + stream, (uint64_t)i) % (uint64_t)vocab);
}

/* synthetic tensor ids shared with the device initialiser */
enum { TID_TOK_EMBD = 1, TID_OUTPUT = 2, TID_OUTPUT_NORM = 3 };
enum { K_ATTN_NORM = 0, K_Q = 1, K_K = 2, K_V = 3, K_O = 4, K_FFN_NORM = 5, K_GATE = 6, K_UP = 7, K_DOWN = 8 };
static inline uint64_t tid_layer(int l, int k) { return 256ull + (uint64_t)l * 16ull + (uint64_t)k; }
static inline uint64_t tid_kv(int l, int isv) { return 0x40000000ull + (uint64_t)l * 2ull + (uint64_t)isv; }

/* ------------------------------------------------------------------------- */
/* primitive ops (exported for per-kernel parity tests)                      */
/* ------------------------------------------------------------------------- */

/* fp32 dot with 16 interleaved accumulators (fixed order, vectorisable without -ffast-math) */
static float dot_row(const void* w, int dtype, const float* x, int K) {
    float acc[16] = {0};
    int k = 0;
    if (dtype == ORC_F32) {
        const float* wf = (const float*)w;
        for (; k + 16 <= K; k += 16)
            for (int j = 0; j < 16; j++) acc[j] += wf[k + j] * x[k + j];
        for (; k < K; k++) acc[k & 15] += wf[k] * x[k];
    } else if (dtype == ORC_F16) {
        const uint16_t* wh = (const uint16_t*)w;
#ifdef ORC_HAVE_F16C
        for (; k + 16 <= K; k += 16) {
            __m256 a = _mm256_cvtph_ps(_mm_loadu_si128((const __m128i*)(wh + k)));
            __m256 b = _mm256_cvtph_ps(_mm_loadu_si128((const __m128i*)(wh + k + 8)));
            float t[16];
            _mm256_storeu_ps(t, a);
            _mm256_storeu_ps(t + 8, b);
            for (int j = 0; j < 16; j++) acc[j] += t[j] * x[k + j];
        }
#endif
        for (; k < K; k++) acc[k & 15] += orc_h2f(wh[k]) * x[k];
    } else {
        const uint16_t* wb = (const uint16_t*)w;
        for (; k + 16 <= K; k += 16)
            for (int j = 0; j < 16; j++) acc[j] += orc_bf2f(wb[k + j]) * x[k + j];
        for (; k < K; k++) acc[k & 15] += orc_bf2f(wb[k]) * x[k];
    }
    for (int s = 8; s >= 1; s >>= 1)
        for (int j = 0; j < s; j++) acc[j] += acc[j + s];
    return acc[0];
}

static size_t dtype_size(int dtype) { return dtype == ORC_F32 ? 4 : 2; }

/* y[b][n] = sum_k W[n][k] x[b][k]; W row-major [N][K] (GGUF ne = [K, N]) */
void orc_gemv(int dtype, const void* W, int N, int K, const float* x, int B, float* y) {
    size_t es = dtype_size(dtype);
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; n++) {
        const void* row = (const char*)W + (size_t)n * (size_t)K * es;
        for (int b = 0; b < B; b++) y[(size_t)b * N + n] = dot_row(row, dtype, x + (size_t)b * K, K);
    }
}

/* rms_norm.comp:24-34: y = x / sqrt(sum(x^2)/d + eps) * w, sequential fp32 sum */
void orc_rmsnorm(const float* x, const void* w, int wdtype, int B, int d, float eps, float* y) {
    for (int b = 0; b < B; b++) {
        const float* xb = x + (size_t)b * d;
        float ss = 0.0f;
        for (int j = 0; j < d; j++) ss += xb[j] * xb[j];
        float var = ss / (float)d + eps;
        float den = sqrtf(var);
        for (int j = 0; j < d; j++) y[(size_t)b * d + j] = xb[j] / den * load_elem(w, wdtype, (size_t)j);
    }
}

/* RoPE tables: cos/sin of pos * theta^(-2i/hd), evaluated in double and rounded once
 * (Utils.cpp:101-110 evaluates pow/cos/sin in float; the double evaluation makes the
 * table reproducible bit-for-bit by the device, which uploads the same table). */
void orc_rope_table(int n_pos, int head_dim, float theta, float* cos_out, float* sin_out) {
    int half = head_dim / 2;
    for (int p = 0; p < n_pos; p++)
        for (int i = 0; i < half; i++) {
            double f = pow((double)theta, -(double)(2 * i) / (double)head_dim);
            double a = (double)p * f;
            cos_out[(size_t)p * half + i] = (float)cos(a);
            sin_out[(size_t)p * half + i] = (float)sin(a);
        }
}

/* rotate adjacent pairs (2i, 2i+1) of each head in place (fused_matmul_rope.comp:48-82) */
void orc_rope_apply(float* v, int n_heads, int head_dim, const float* cos_row, const float* sin_row) {
    int half = head_dim / 2;
    for (int h = 0; h < n_heads; h++) {
        float* p = v + (size_t)h * head_dim;
        for (int i = 0; i < half; i++) {
            float c = cos_row[i], s = sin_row[i];
            float a = p[2 * i], b = p[2 * i + 1];
            p[2 * i] = a * c - b * s;
            p[2 * i + 1] = a * s + b * c;
        }
    }
}

/* silu(z) = z / (1 + exp(-z))  (feed_forward.comp:21) */
static inline float silu(float z) { return z / (1.0f + expf(-z)); }

void orc_swiglu(const float* g, const float* u, int n, float* a) {
    for (int i = 0; i < n; i++) a[i] = silu(g[i]) * u[i];
}

/* first argmax with strict '>' (VulkanSymbioteEngine.cpp:1794-1804) */
int32_t orc_argmax(const float* v, int n) {
    int32_t best = 0;
    float bv = v[0];
    for (int i = 1; i < n; i++)
        if (v[i] > bv) { bv = v[i]; best = i; }
    return best;
}

/* Long-context sparse mask of the reference (sparse_attention.comp:77-131), selected when the
 * sequence is longer than min_len (VulkanSymbioteEngine.cpp:788: use_sparse_attention &&
 * seq_len > 8192; window 512, 16 global tokens, blocks of 1024, Common.h:71-74). For a query at
 * position pos of a sequence of pos + 1 tokens the shader's index arithmetic gives one
 * contiguous range [first, pos]:
 *   get_attention_window (:77-101): window_start = pos > W ? pos - W : 0; a query among the
 *     first G tokens starts at 0, any other at min(G, window_start); the range ends at pos + 1;
 *   compute_ring_attention (:105-131): block_start = (pos / BLK) * BLK; the start is raised to
 *     block_start - W when block_start > W; the end is cut at the block's end (>= pos + 1).
 * The shader keeps 512 scores in shared memory and reads 0 for later ones (:143-158); that
 * buffer limit is not part of the mask and is not restated. min_len <= 0: dense (first 0). */
int orc_sparse_first(int min_len, int window, int global, int block, int pos) {
    if (min_len <= 0 || pos + 1 <= min_len) return 0;
    int ws = pos > window ? pos - window : 0;
    int start = pos < global ? 0 : (global < ws ? global : ws);
    int bs = (pos / block) * block;
    int clamp = bs > window ? bs - window : 0;
    return start > clamp ? start : clamp;
}

/* One query head against its KV group: Kg,Vg point at [max_seq][hd] of group g, positions
 * [first, len). attention.comp:116-189: scores scaled by 1/sqrt(hd), max-subtracted softmax,
 * then normalised probabilities times V. */
static void attn_head(const float* qh, const void* Kc, const void* Vc, int kvdtype, size_t gbase,
                      int head_dim, int first, int len, float* oh, float* scratch) {
    float scale = 1.0f / sqrtf((float)head_dim);
    float mx = -INFINITY;
    for (int t = first; t < len; t++) {
        size_t base = gbase + (size_t)t * head_dim;
        float s = 0.0f;
        for (int e = 0; e < head_dim; e++) s += qh[e] * load_elem(Kc, kvdtype, base + e);
        s *= scale;
        scratch[t] = s;
        if (s > mx) mx = s;
    }
    float sum = 0.0f;
    for (int t = first; t < len; t++) {
        scratch[t] = expf(scratch[t] - mx);
        sum += scratch[t];
    }
    for (int e = 0; e < head_dim; e++) oh[e] = 0.0f;
    for (int t = first; t < len; t++) {
        float p = scratch[t] / sum;
        size_t base = gbase + (size_t)t * head_dim;
        for (int e = 0; e < head_dim; e++) oh[e] += p * load_elem(Vc, kvdtype, base + e);
    }
}

/* Single-query attention for one sequence over a contiguous cache
 * K,V: [n_kv][max_seq][hd] (dtype kvdtype), attend to t in [first, len) (first = 0: dense).
 * Query head h reads KV group g = h*n_kv/n_heads (attention.comp:92). */
void orc_attention_from(const float* q, const void* Kc, const void* Vc, int kvdtype, int n_heads, int n_kv,
                        int head_dim, int max_seq, int first, int len, float* o, float* scratch) {
    for (int h = 0; h < n_heads; h++) {
        int g = (int)((long)h * n_kv / n_heads);
        attn_head(q + (size_t)h * head_dim, Kc, Vc, kvdtype, (size_t)g * max_seq * head_dim, head_dim,
                  first, len, o + (size_t)h * head_dim, scratch);
    }
}
void orc_attention(const float* q, const void* Kc, const void* Vc, int kvdtype, int n_heads,
                   int n_kv, int head_dim, int max_seq, int len, float* o, float* scratch) {
    orc_attention_from(q, Kc, Vc, kvdtype, n_heads, n_kv, head_dim, max_seq, 0, len, o, scratch);
}

/* ------------------------------------------------------------------------- */
/* minimal standard GGUF v2/v3 reader (independent of the product loader)    */
/* ------------------------------------------------------------------------- */

typedef struct {
    char name[96];
    int dtype;
    int n_dims;
    uint64_t ne[4];
    uint64_t offset;
} orc_tensor;

typedef struct {
    int n_layers, d, n_heads, n_kv, head_dim, ffn, vocab;
    float rope_theta, eps;
    int wdtype, kvdtype, max_seq, max_batch;
} orc_config;

typedef struct {
    const void* p;
    int dtype;
} orc_w;

typedef struct {
    orc_w attn_norm, wq, wk, wv, wo, ffn_norm, wg, wu, wd;
} orc_layer;

typedef struct {
    orc_config c;
    orc_w tok_embd, output, out_norm;
    orc_layer* layers;
    /* storage */
    void* map;
    size_t map_len;
    void* owned; /* synthetic weights */
    float** qbufs; /* dequantized copies of block-quantized GGUF tensors */
    int n_qbufs;
    /* KV cache [l][b][kv][max_seq][hd] in kvdtype */
    void* kcache;
    void* vcache;
    float* rope_cos;
    float* rope_sin;
    int rope_len;
    int sp_min_len, sp_window, sp_global, sp_block; /* sparse mask (sp_min_len 0: dense) */
} orc_model;

typedef struct {
    const uint8_t* p;
    const uint8_t* end;
    int err;
} rd_t;

static uint64_t rd_u(rd_t* r, int n) {
    if (r->p + n > r->end) { r->err = 1; return 0; }
    uint64_t v = 0;
    memcpy(&v, r->p, (size_t)n);
    r->p += n;
    return v;
}

static void rd_str(rd_t* r, char* out, size_t cap) {
    uint64_t len = rd_u(r, 8);
    if (r->err || r->p + len > r->end) { r->err = 1; return; }
    size_t c = len < cap - 1 ? (size_t)len : cap - 1;
    if (out) { memcpy(out, r->p, c); out[c] = 0; }
    r->p += len;
}

static const int gguf_scalar_size[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};

static void rd_skip_value(rd_t* r, uint32_t t) {
    if (t == 8) { rd_str(r, NULL, 1); return; }
    if (t == 9) {
        uint32_t et = (uint32_t)rd_u(r, 4);
        uint64_t cnt = rd_u(r, 8);
        if (et == 8) { for (uint64_t i = 0; i < cnt && !r->err; i++) rd_str(r, NULL, 1); }
        else if (et < 13 && gguf_scalar_size[et]) {
            uint64_t bytes = cnt * (uint64_t)gguf_scalar_size[et];
            if (r->p + bytes > r->end) r->err = 1; else r->p += bytes;
        } else r->err = 1;
        return;
    }
    if (t < 13 && gguf_scalar_size[t]) { rd_u(r, gguf_scalar_size[t]); return; }
    r->err = 1;
}

static double rd_num(rd_t* r, uint32_t t) {
    switch (t) {
        case 0: return (double)(uint8_t)rd_u(r, 1);
        case 1: return (double)(int8_t)rd_u(r, 1);
        case 2: return (double)(uint16_t)rd_u(r, 2);
        case 3: return (double)(int16_t)rd_u(r, 2);
        case 4: return (double)(uint32_t)rd_u(r, 4);
        case 5: return (double)(int32_t)rd_u(r, 4);
        case 6: { uint32_t b = (uint32_t)rd_u(r, 4); float f; memcpy(&f, &b, 4); return f; }
        case 7: return (double)(uint8_t)rd_u(r, 1);
        case 10: return (double)rd_u(r, 8);
        case 11: return (double)(int64_t)rd_u(r, 8);
        case 12: { uint64_t b = rd_u(r, 8); double f; memcpy(&f, &b, 8); return f; }
        default: rd_skip_value(r, t); return NAN;
    }
}

static void model_free_storage(orc_model* m) {
    if (m->map) munmap(m->map, m->map_len);
    free(m->owned);
    for (int i = 0; i < m->n_qbufs; i++) free(m->qbufs[i]);
    free(m->qbufs);
    free(m->layers);
    free(m->kcache);
    free(m->vcache);
    free(m->rope_cos);
    free(m->rope_sin);
}

static int model_alloc_runtime(orc_model* m) {
    orc_config* c = &m->c;
    size_t kvn = (size_t)c->n_layers * c->max_batch * c->n_kv * c->max_seq * c->head_dim;
    size_t es = dtype_size(c->kvdtype);
    m->kcache = calloc(kvn, es);
    m->vcache = calloc(kvn, es);
    m->rope_len = c->max_seq;
    m->rope_cos = (float*)malloc(sizeof(float) * (size_t)c->max_seq * (c->head_dim / 2));
    m->rope_sin = (float*)malloc(sizeof(float) * (size_t)c->max_seq * (c->head_dim / 2));
    if (!m->kcache || !m->vcache || !m->rope_cos || !m->rope_sin) return -8;
    orc_rope_table(c->max_seq, c->head_dim, c->rope_theta, m->rope_cos, m->rope_sin);
    return 0;
}

static const char* layer_suffix[9] = {"attn_norm", "attn_q", "attn_k", "attn_v", "attn_output",
                                      "ffn_norm", "ffn_gate", "ffn_up", "ffn_down"};

/* Load a standard GGUF (ggml tensor type ids, general.alignment respected).
 * Metadata keys follow GGUFLoader.cpp:673-728; head_dim = d / heads (:725). */
int orc_model_load_gguf_ex(const char* path, int kvdtype, int max_seq, int max_batch, int legacy_q4,
                           orc_model** out) {
    int fd = open(path, O_RDONLY);
    if (fd < 0) return -6;
    struct stat st;
    if (fstat(fd, &st) != 0) { close(fd); return -6; }
    void* map = mmap(NULL, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (map == MAP_FAILED) return -6;
    orc_model* m = (orc_model*)calloc(1, sizeof(orc_model));
    m->map = map;
    m->map_len = (size_t)st.st_size;
    rd_t r = {(const uint8_t*)map, (const uint8_t*)map + st.st_size, 0};
    uint32_t magic = (uint32_t)rd_u(&r, 4);
    uint32_t version = (uint32_t)rd_u(&r, 4);
    if (magic != 0x46554747u || version < 2 || version > 3) { model_free_storage(m); free(m); return -7; }
    uint64_t n_tensors = rd_u(&r, 8), n_kv = rd_u(&r, 8);
    orc_config* c = &m->c;
    memset(c, 0, sizeof(*c));
    c->rope_theta = 10000.0f; /* Common.h:63 */
    c->eps = 1e-5f;           /* Common.h:68 */
    uint64_t alignment = 32;
    int has_kv_heads = 0;
    for (uint64_t i = 0; i < n_kv && !r.err; i++) {
        char key[256];
        rd_str(&r, key, sizeof key);
        uint32_t t = (uint32_t)rd_u(&r, 4);
        if (t == 8 || t == 9) { rd_skip_value(&r, t); continue; }
        double v = rd_num(&r, t);
        if (!strcmp(key, "llama.embedding_length")) c->d = (int)v;
        else if (!strcmp(key, "llama.block_count")) c->n_layers = (int)v;
        else if (!strcmp(key, "llama.attention.head_count")) c->n_heads = (int)v;
        else if (!strcmp(key, "llama.attention.head_count_kv")) { c->n_kv = (int)v; has_kv_heads = 1; }
        else if (!strcmp(key, "llama.feed_forward_length")) c->ffn = (int)v;
        else if (!strcmp(key, "llama.vocab_size")) c->vocab = (int)v;
        else if (!strcmp(key, "llama.rope.freq_base")) c->rope_theta = (float)v;
        else if (!strcmp(key, "llama.attention.layer_norm_rms_epsilon")) c->eps = (float)v;
        else if (!strcmp(key, "general.alignment")) alignment = (uint64_t)v;
    }
    if (!has_kv_heads) c->n_kv = c->n_heads;
    orc_tensor* ts = (orc_tensor*)calloc(n_tensors ? n_tensors : 1, sizeof(orc_tensor));
    for (uint64_t i = 0; i < n_tensors && !r.err; i++) {
        rd_str(&r, ts[i].name, sizeof ts[i].name);
        ts[i].n_dims = (int)rd_u(&r, 4);
        for (int j = 0; j < ts[i].n_dims && j < 4; j++) ts[i].ne[j] = rd_u(&r, 8);
        ts[i].dtype = (int)rd_u(&r, 4);
        ts[i].offset = rd_u(&r, 8);
    }
    if (r.err || c->d <= 0 || c->n_heads <= 0 || c->n_layers <= 0) {
        free(ts); model_free_storage(m); free(m); return -7;
    }
    size_t hdr = (size_t)(r.p - (const uint8_t*)map);
    size_t data0 = (hdr + alignment - 1) / alignment * alignment;
    c->head_dim = c->d / c->n_heads;
    c->kvdtype = kvdtype;
    c->max_seq = max_seq;
    c->max_batch = max_batch;
    m->layers = (orc_layer*)calloc((size_t)c->n_layers, sizeof(orc_layer));
    int found = 0;
    for (uint64_t i = 0; i < n_tensors; i++) {
        orc_w w = {(const uint8_t*)map + data0 + ts[i].offset, ts[i].dtype};
        if (ts[i].dtype != ORC_F32 && ts[i].dtype != ORC_F16 && ts[i].dtype != ORC_BF16 && !orc_is_quant(ts[i].dtype))
            continue;
        if (orc_is_quant(ts[i].dtype)) {
            /* the reference dequantises quantized tensors to fp32 when it reads them
             * (read_tensor_data -> dequantize_tensor, GGUFLoader.cpp:776-778) */
            size_t n = 1;
            for (int j = 0; j < ts[i].n_dims && j < 4; j++) n *= (size_t)ts[i].ne[j];
            float* f = (float*)malloc(n * sizeof(float));
            if (!f) { free(ts); model_free_storage(m); free(m); return -8; }
            orc_dequant_blocks(ts[i].dtype, w.p, n, legacy_q4, f);
            m->qbufs = (float**)realloc(m->qbufs, sizeof(float*) * (size_t)(m->n_qbufs + 1));
            m->qbufs[m->n_qbufs++] = f;
            w.p = f;
            w.dtype = ORC_F32;
        }
        const char* nm = ts[i].name;
        if (!strcmp(nm, "token_embd.weight")) {
            m->tok_embd = w; found++;
            if (c->vocab == 0) c->vocab = (int)ts[i].ne[1];
            c->wdtype = ts[i].dtype; /* the file's type (quantized tensors are held as fp32) */
        } else if (!strcmp(nm, "output.weight")) { m->output = w; found++; }
        else if (!strcmp(nm, "output_norm.weight")) { m->out_norm = w; found++; }
        else if (!strncmp(nm, "blk.", 4)) {
            int l = atoi(nm + 4);
            const char* dot = strchr(nm + 4, '.');
            if (!dot || l < 0 || l >= c->n_layers) continue;
            char suf[64];
            snprintf(suf, sizeof suf, "%s", dot + 1);
            char* w2 = strstr(suf, ".weight");
            if (!w2) continue;
            *w2 = 0;
            orc_w* slots = (orc_w*)&m->layers[l];
            for (int k = 0; k < 9; k++)
                if (!strcmp(suf, layer_suffix[k]) || (k == K_O && !strcmp(suf, "attn_o"))) {
                    slots[k] = w; found++;
                }
            if (!strcmp(nm + 4 + (dot - (nm + 4)) + 1, "ffn_gate.weight") && c->ffn == 0)
                c->ffn = (int)ts[i].ne[1];
        }
    }
    free(ts);
    if (found != 3 + 9 * c->n_layers) { model_free_storage(m); free(m); return -7; }
    int rc = model_alloc_runtime(m);
    if (rc) { model_free_storage(m); free(m); return rc; }
    *out = m;
    return 0;
}

int orc_model_load_gguf(const char* path, int kvdtype, int max_seq, int max_batch, orc_model** out) {
    return orc_model_load_gguf_ex(path, kvdtype, max_seq, max_batch, 0, out);
}

/* Build a model whose weights come from the seeded generator (norms = 1.0),
 * exactly the tensors vsl/synth.py writes into a GGUF and the device initialiser fills. */
int orc_model_synthetic(const orc_config* cfg, uint64_t seed, double sigma, orc_model** out) {
    orc_model* m = (orc_model*)calloc(1, sizeof(orc_model));
    m->c = *cfg;
    orc_config* c = &m->c;
    const int quant = orc_is_quant(c->wdtype);
    size_t es = quant ? 4 : dtype_size(c->wdtype); /* quantized weights are held dequantized */
    size_t qd = (size_t)c->n_heads * c->head_dim, kvd = (size_t)c->n_kv * c->head_dim;
    size_t per_layer = qd * c->d + 2 * kvd * c->d + c->d * qd + 3 * (size_t)c->ffn * c->d;
    size_t mats = per_layer * c->n_layers + 2 * (size_t)c->vocab * c->d;
    size_t norms = (size_t)(2 * c->n_layers + 1) * c->d;
    m->owned = malloc(mats * es + norms * 4 + 64);
    if (!m->owned) { free(m); return -8; }
    m->layers = (orc_layer*)calloc((size_t)c->n_layers, sizeof(orc_layer));
    uint8_t* p = (uint8_t*)m->owned;
    float* nrm = (float*)(p + mats * es);
    for (size_t i = 0; i < norms; i++) nrm[i] = 1.0f;
#define TAKE(dst, tid, rows, cols)                                                   \
    do {                                                                             \
        if (quant) orc_synthq_dequant(seed, (tid), (rows), (cols), sigma, c->wdtype, (float*)p); \
        else orc_synth_fill(seed, (tid), 0, (uint64_t)(rows) * (cols), sigma, c->wdtype, p); \
        (dst).p = p; (dst).dtype = quant ? ORC_F32 : c->wdtype; p += (size_t)(rows) * (cols) * es; \
    } while (0)
    TAKE(m->tok_embd, TID_TOK_EMBD, c->vocab, c->d);
    TAKE(m->output, TID_OUTPUT, c->vocab, c->d);
    m->out_norm.p = nrm; m->out_norm.dtype = ORC_F32; nrm += c->d;
    for (int l = 0; l < c->n_layers; l++) {
        orc_layer* L = &m->layers[l];
        L->attn_norm.p = nrm; L->attn_norm.dtype = ORC_F32; nrm += c->d;
        L->ffn_norm.p = nrm; L->ffn_norm.dtype = ORC_F32; nrm += c->d;
        TAKE(L->wq, tid_layer(l, K_Q), qd, c->d);
        TAKE(L->wk, tid_layer(l, K_K), kvd, c->d);
        TAKE(L->wv, tid_layer(l, K_V), kvd, c->d);
        TAKE(L->wo, tid_layer(l, K_O), c->d, qd);
        TAKE(L->wg, tid_layer(l, K_GATE), c->ffn, c->d);
        TAKE(L->wu, tid_layer(l, K_UP), c->ffn, c->d);
        TAKE(L->wd, tid_layer(l, K_DOWN), c->d, c->ffn);
    }
#undef TAKE
    int rc = model_alloc_runtime(m);
    if (rc) { model_free_storage(m); free(m); return rc; }
    *out = m;
    return 0;
}

void orc_model_free(orc_model* m) {
    if (!m) return;
    model_free_storage(m);
    free(m);
}

void orc_model_get_config(const orc_model* m, orc_config* out) { *out = m->c; }

static size_t kv_index(const orc_config* c, int l, int b, int g, int t) {
    return ((((size_t)l * c->max_batch + b) * c->n_kv + g) * c->max_seq + t) * c->head_dim;
}

static void kv_store(const orc_model* m, void* cache, size_t idx, const float* v, int n) {
    if (m->c.kvdtype == ORC_F16) for (int i = 0; i < n; i++) ((uint16_t*)cache)[idx + i] = orc_f2h(v[i]);
    else if (m->c.kvdtype == ORC_BF16) for (int i = 0; i < n; i++) ((uint16_t*)cache)[idx + i] = orc_f2bf(v[i]);
    else memcpy((float*)cache + idx, v, sizeof(float) * (size_t)n);
}

/* Sparse long-context attention (orc_sparse_first) for every later step; min_len 0 = dense. */
int orc_model_set_sparse(orc_model* m, int min_len, int window, int global, int block) {
    if (!m || min_len < 0 || window < 0 || global < 0 || (min_len > 0 && block <= 0)) return -1;
    m->sp_min_len = min_len;
    m->sp_window = window;
    m->sp_global = global;
    m->sp_block = block;
    return 0;
}

void orc_model_clear_kv(orc_model* m) {
    orc_config* c = &m->c;
    size_t kvn = (size_t)c->n_layers * c->max_batch * c->n_kv * c->max_seq * c->head_dim;
    memset(m->kcache, 0, kvn * dtype_size(c->kvdtype));
    memset(m->vcache, 0, kvn * dtype_size(c->kvdtype));
}

/* Fill KV positions [0, n_pos) of every layer/sequence with seeded values
 * (tensor ids tid_kv(l, 0|1), element index ((b*n_kv + g)*n_pos + t)*hd + e). */
int orc_model_fill_kv_synthetic(orc_model* m, uint64_t seed, double sigma, int n_pos, int B) {
    orc_config* c = &m->c;
    if (n_pos > c->max_seq || B > c->max_batch) return -1;
    size_t es = dtype_size(c->kvdtype);
    size_t span = (size_t)n_pos * c->head_dim;
    for (int l = 0; l < c->n_layers; l++)
        for (int isv = 0; isv < 2; isv++)
            for (int b = 0; b < B; b++)
                for (int g = 0; g < c->n_kv; g++) {
                    void* cache = isv ? m->vcache : m->kcache;
                    size_t idx = kv_index(c, l, b, g, 0);
                    uint64_t start = ((uint64_t)b * c->n_kv + g) * span;
                    orc_synth_fill(seed, tid_kv(l, isv), start, span, sigma, c->kvdtype,
                                   (uint8_t*)cache + idx * es);
                }
    return 0;
}

/* One decode step for B sequences. ids[b] is the input token at absolute position pos[b].
 * Writes logits[B][V] (may be NULL) and the greedy ids out_ids[B] (may be NULL). */
int orc_model_step(orc_model* m, int B, const int32_t* ids, const int32_t* pos, float* logits,
                   int32_t* out_ids) {
    orc_config* c = &m->c;
    if (B <= 0 || B > c->max_batch) return -1;
    for (int b = 0; b < B; b++)
        if (pos[b] < 0 || pos[b] >= c->max_seq) return -5;
    int d = c->d, hd = c->head_dim;
    int qd = c->n_heads * hd, kvd = c->n_kv * hd, F = c->ffn, V = c->vocab;
    size_t eb = dtype_size(m->tok_embd.dtype);
    float* x = (float*)malloc(sizeof(float) * (size_t)B * d);
    float* n = (float*)malloc(sizeof(float) * (size_t)B * (d > F ? d : F));
    float* q = (float*)malloc(sizeof(float) * (size_t)B * qd);
    float* k = (float*)malloc(sizeof(float) * (size_t)B * kvd);
    float* v = (float*)malloc(sizeof(float) * (size_t)B * kvd);
    float* o = (float*)malloc(sizeof(float) * (size_t)B * qd);
    float* t = (float*)malloc(sizeof(float) * (size_t)B * (d > F ? d : F));
    float* g = (float*)malloc(sizeof(float) * (size_t)B * F);
    float* u = (float*)malloc(sizeof(float) * (size_t)B * F);
    float* lg = logits ? logits : (float*)malloc(sizeof(float) * (size_t)B * V);
    int max_len = 0;
    for (int b = 0; b < B; b++) if (pos[b] + 1 > max_len) max_len = pos[b] + 1;
    /* embedding_lookup.comp:29-32: clamp id to V-1 */
    for (int b = 0; b < B; b++) {
        int id = ids[b] < 0 ? 0 : ids[b];
        if (id > V - 1) id = V - 1;
        for (int j = 0; j < d; j++)
            x[(size_t)b * d + j] = load_elem((const uint8_t*)m->tok_embd.p + (size_t)id * d * eb,
                                             m->tok_embd.dtype, (size_t)j);
    }
    int half = hd / 2;
    for (int l = 0; l < c->n_layers; l++) {
        orc_layer* L = &m->layers[l];
        orc_rmsnorm(x, L->attn_norm.p, L->attn_norm.dtype, B, d, c->eps, n);
        orc_gemv(L->wq.dtype, L->wq.p, qd, d, n, B, q);
        orc_gemv(L->wk.dtype, L->wk.p, kvd, d, n, B, k);
        orc_gemv(L->wv.dtype, L->wv.p, kvd, d, n, B, v);
        for (int b = 0; b < B; b++) {
            const float* cr = m->rope_cos + (size_t)pos[b] * half;
            const float* sr = m->rope_sin + (size_t)pos[b] * half;
            orc_rope_apply(q + (size_t)b * qd, c->n_heads, hd, cr, sr);
            orc_rope_apply(k + (size_t)b * kvd, c->n_kv, hd, cr, sr);
            for (int gi = 0; gi < c->n_kv; gi++) {
                size_t idx = kv_index(c, l, b, gi, pos[b]);
                kv_store(m, m->kcache, idx, k + (size_t)b * kvd + (size_t)gi * hd, hd);
                kv_store(m, m->vcache, idx, v + (size_t)b * kvd + (size_t)gi * hd, hd);
            }
        }
#pragma omp parallel
        {
            float* scratch = (float*)malloc(sizeof(float) * (size_t)max_len);
#pragma omp for schedule(static) collapse(2)
            for (int b = 0; b < B; b++)
                for (int h = 0; h < c->n_heads; h++) {
                    int gi = (int)((long)h * c->n_kv / c->n_heads); /* attention.comp:92 */
                    attn_head(q + (size_t)b * qd + (size_t)h * hd, m->kcache, m->vcache, c->kvdtype,
                              kv_index(c, l, b, gi, 0), hd,
                              orc_sparse_first(m->sp_min_len, m->sp_window, m->sp_global, m->sp_block, pos[b]),
                              pos[b] + 1, o + (size_t)b * qd + (size_t)h * hd, scratch);
                }
            free(scratch);
        }
        orc_gemv(L->wo.dtype, L->wo.p, d, qd, o, B, t);
        for (size_t i = 0; i < (size_t)B * d; i++) x[i] += t[i];
        orc_rmsnorm(x, L->ffn_norm.p, L->ffn_norm.dtype, B, d, c->eps, n);
        orc_gemv(L->wg.dtype, L->wg.p, F, d, n, B, g);
        orc_gemv(L->wu.dtype, L->wu.p, F, d, n, B, u);
        orc_swiglu(g, u, B * F, g);
        orc_gemv(L->wd.dtype, L->wd.p, d, F, g, B, t);
        for (size_t i = 0; i < (size_t)B * d; i++) x[i] += t[i];
    }
    orc_rmsnorm(x, m->out_norm.p, m->out_norm.dtype, B, d, c->eps, n);
    orc_gemv(m->output.dtype, m->output.p, V, d, n, B, lg);
    if (out_ids)
        for (int b = 0; b < B; b++) out_ids[b] = orc_argmax(lg + (size_t)b * V, V);
    free(x); free(n); free(q); free(k); free(v); free(o); free(t); free(g); free(u);
    if (!logits) free(lg);
    return 0;
}

int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void orc_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}
