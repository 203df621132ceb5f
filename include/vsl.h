/*
 * vsl.h -- C ABI of the B200-native Vulkan-Symbiote decode engine (libvsl.so).
 *
 * The reference exposes its decode path only as C++ classes; its "kernel runtime"
 * (vk_symbiote/src/ShaderRuntime.cpp) binds GLSL pipelines and dispatches them with
 * ShaderRuntime::dispatch_compute (ShaderRuntime.cpp:1484-1542). This header replaces that
 * role with plain C entry points: device pointers are caller-owned, every call takes an
 * explicit cudaStream_t (passed as void*), never synchronises, and returns a status code
 * (VSL_OK or a negative VSL_ERR_*); vsl_last_error_string() describes the last failure
 * on the calling thread. No C++ exception crosses this boundary.
 *
 * Layout conventions
 *   - Weights are GGUF row-major [N][K] (GGUF ne = [K, N]); a projection computes
 *     y[b][n] = sum_k W[n][k] * x[b][k] with fp32 accumulation. Rows are 16-byte aligned
 *     (K * sizeof(elem) % 16 == 0).
 *   - Activations and the residual stream are fp32 [B][dim].
 *   - Paged KV cache: k_cache / v_cache are [n_pages][n_kv][page_size][head_dim] in the
 *     KV dtype; page_table is int32 [B][max_pages] mapping a sequence's logical page to a
 *     physical page. Position p of sequence b lives in page page_table[b][p / page_size],
 *     slot p % page_size.
 *   - pos[b] is the absolute position of the token being decoded; the attention length
 *     is pos[b] + 1.
 *   - RoPE tables rope_cos / rope_sin are fp32 [max_pos][head_dim/2]: cos/sin of
 *     pos * theta^(-2i/head_dim), adjacent-pair rotation (vk_symbiote/src/Utils.cpp:101-110).
 */
#ifndef VSL_H
#define VSL_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define VSL_API __attribute__((visibility("default")))
#else
#define VSL_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes (the reference returns negative ints through Expected<T>,
 *      vk_symbiote/include/vk_symbiote/Common.h:88-193) ---- */
#define VSL_OK 0
#define VSL_ERR_INVALID (-1)
#define VSL_ERR_CUDA (-2)
#define VSL_ERR_NCCL (-3)
#define VSL_ERR_TIMEOUT (-4)
#define VSL_ERR_BOUNDS (-5)
#define VSL_ERR_IO (-6)
#define VSL_ERR_FORMAT (-7)
#define VSL_ERR_OOM (-8)
#define VSL_ERR_UNSUPPORTED (-9)
#define VSL_ERR_STATE (-10)

/* ---- element types: ggml / GGUF tensor type ids ---- */
#define VSL_F32 0
#define VSL_F16 1
#define VSL_BF16 30
#define VSL_Q4_0 2  /* weights only, device layout: see vsl_weight_row_bytes / vsl_repack_gguf_rows */
#define VSL_Q4_1 3  /* weights only, same device layout plus a per-block fp16 minimum */
#define VSL_Q8_0 8

/* ---- projection epilogues ---- */
#define VSL_EPI_STORE 0  /* y[b][n]  = acc                                             */
#define VSL_EPI_ADD 1    /* y[b][n] += acc  (residual add)                             */
#define VSL_EPI_SWIGLU 2 /* rows interleaved (gate_i, up_i): y[b][i] = silu(g) * up    */

VSL_API const char* vsl_last_error_string(void);
VSL_API int vsl_version(void);

/* ======================================================================================
 * Kernels
 * ====================================================================================== */

/* Embedding gather with id clamp to V-1 (replaces embed_tokens_with_weights,
 * vk_symbiote/src/VulkanSymbioteEngine.cpp:2886-3026, and embedding_lookup.comp:21-41).
 * table [V][d] in dtype; ids int32 [B]; x fp32 [B][d]. */
VSL_API int vsl_embed_gather(int dtype, const void* table, int V, int d, const int32_t* ids, int B, float* x,
                     void* stream);

/* RMSNorm y = x / sqrt(mean(x^2) + eps) * w (replaces rms_norm_with_weights,
 * VulkanSymbioteEngine.cpp:2809-2884, and rms_norm.comp:17-35). x, y fp32 [B][d]; w fp32 [d]. */
VSL_API int vsl_rmsnorm(const float* x, const float* w, int B, int d, float eps, float* y, void* stream);

/* Decode projection y = x W^T for B <= 16 rows of activations (replaces the projection
 * parts of attention_with_weights :2440-2584, feed_forward_with_weights :2726-2807 and
 * final_projection_with_weights :3028-3130). If norm_w is non-NULL the activations are
 * RMS-normalised with norm_w (fp32 [K], epsilon eps) first, fusing rms_norm_with_weights.
 * epilogue: VSL_EPI_STORE / VSL_EPI_ADD (y is the fp32 residual) / VSL_EPI_SWIGLU (N even,
 * y has N/2 columns; feed_forward.comp:21,49-61). */
VSL_API int vsl_gemv(int wdtype, const void* W, int N, int K, const float* x, int B, float* y, int epilogue,
             const float* norm_w, float eps, void* stream);

/* Batched projection on the tcgen05 tensor cores for 1 <= B <= 128 activation rows (the
 * skinny-GEMM form of vsl_gemv for batched decode: every weight tile is read from HBM once
 * for all B rows; same projection sites as vsl_gemv). W is fp16 or bf16 with N >= 128,
 * K >= 64 and K % 8 == 0; x, y, norm_w, eps and epilogue mean what they mean for vsl_gemv.
 * The fp32 activations enter the tensor cores as a hi + lo pair of 16-bit values, so results
 * match the fp32-activation GEMV to ~1e-6 relative (fp16) / ~2e-5 (bf16).
 * workspace: caller-owned device memory of vsl_skinny_gemm_tc_workspace_size bytes, 1 KB
 * aligned, zero-filled before its first use (the kernel leaves its arrival counters, kept at
 * the tail of the workspace, zero again). Calls of different shapes may share a workspace
 * sized with the largest N, K and B together; calls that share one must be ordered on one
 * stream. Two launches on `stream`. */
VSL_API int vsl_skinny_gemm_tc_workspace_size(int N, int K, int B, size_t* bytes);
VSL_API int vsl_skinny_gemm_tc(int wdtype, const void* W, int N, int K, const float* x, int B, float* y,
                               int epilogue, const float* norm_w, float eps, void* workspace,
                               size_t workspace_bytes, void* stream);

/* Fused QKV projection + RoPE + KV-cache append (replaces attention.comp:63-108 and the CPU
 * append KVCacheEntry::append_kv, VulkanSymbioteEngine.cpp:41-54). Wqkv rows are
 * [Wq (n_heads*hd); Wk (n_kv*hd); Wv (n_kv*hd)] over K = d_model inputs. x is the fp32
 * residual, normalised with norm_w. Writes q_out fp32 [B][n_heads*hd] (rotated) and the
 * rotated K and plain V of position pos[b] into the paged caches. */
VSL_API int vsl_qkv_rope_append(int wdtype, const void* Wqkv, int n_heads, int n_kv, int head_dim, int K,
                        const float* x, const float* norm_w, float eps, int B, const int32_t* pos,
                        const float* rope_cos, const float* rope_sin, float* q_out, void* k_cache,
                        void* v_cache, int kvdtype, const int32_t* page_table, int max_pages, int page_size,
                        void* stream);

/* Bytes of scratch vsl_flash_decode needs for B sequences of up to max_len positions. */
VSL_API int vsl_flash_decode_workspace_size(int B, int n_heads, int n_kv, int head_dim, int max_len, int split_len,
                                    size_t* bytes);

/* Split-K flash-decode attention over the paged cache, GQA-aware (query head h reads KV
 * group h*n_kv/n_heads, attention.comp:92; softmax of q.K/sqrt(hd), attention.comp:116-189).
 * q fp32 [B][n_heads*hd]; out fp32 [B][n_heads*hd]. split_len (a multiple of page_size)
 * is the number of positions one CTA covers; the grid covers max_len. workspace must hold
 * vsl_flash_decode_workspace_size() bytes and be zero-filled before its first use (the
 * kernel leaves its split counters at zero when it returns). */
VSL_API int vsl_flash_decode(const float* q, const void* k_cache, const void* v_cache, int kvdtype,
                     const int32_t* page_table, int max_pages, int page_size, const int32_t* pos, int B,
                     int n_heads, int n_kv, int head_dim, int max_len, int split_len, float* out, void* workspace,
                     size_t workspace_bytes, void* stream);

/* Long-context sparse mask (the reference's sparse_attention.comp:77-131, switched on when
 * use_sparse_attention && seq_len > 8192, VulkanSymbioteEngine.cpp:788; defaults window 512,
 * 16 global tokens, 1024-position blocks, Common.h:71-74). A query at position pos of a
 * sequence of pos + 1 > min_len tokens attends to positions [first, pos] with, following the
 * shader's index arithmetic,
 *     ws = pos > window ? pos - window : 0
 *     start = pos < global_tokens ? 0 : min(global_tokens, ws)
 *     bs = (pos / block) * block;  clamp = bs > window ? bs - window : 0
 *     first = max(start, clamp)
 * (contiguous: in the shader the global tokens only enter through that min). Shorter sequences,
 * and min_len <= 0, attend densely. The shader's 512-entry score buffer, which reads 0 for the
 * scores beyond it, is a storage limit and not part of the mask. */
typedef struct {
    int min_len;
    int window;
    int global_tokens;
    int block;
} vsl_sparse_mask;

/* Long-context decode attention with the score product on the tcgen05 tensor cores (same
 * semantics and cache layout as vsl_flash_decode; fp16 KV, head_dim 128, up to 8 query heads
 * per KV group, B <= 64, page_size a multiple of 64). n_pages is the size of the physical page
 * pool the page table indexes. Work is split evenly over persistent CTAs whatever the
 * per-sequence lengths; sequences shared by several CTAs are merged deterministically.
 * workspace: vsl_flash_decode_tc_workspace_size bytes, zero-filled before first use (its
 * counters are left zero by every call). */
VSL_API int vsl_flash_decode_tc_workspace_size(int B, int n_kv, size_t* bytes);
VSL_API int vsl_flash_decode_tc(const float* q, const void* k_cache, const void* v_cache, int n_pages,
                                const int32_t* page_table, int max_pages, int page_size, const int32_t* pos, int B,
                                int n_heads, int n_kv, int head_dim, int max_len, float* out, void* workspace,
                                size_t workspace_bytes, void* stream);

/* vsl_flash_decode / vsl_flash_decode_tc with the sparse mask applied per query row (mask NULL
 * or min_len <= 0: dense, the same as the plain entry points). Same workspaces. */
VSL_API int vsl_flash_decode_sparse(const float* q, const void* k_cache, const void* v_cache, int kvdtype,
                                    const int32_t* page_table, int max_pages, int page_size, const int32_t* pos, int B,
                                    int n_heads, int n_kv, int head_dim, int max_len, int split_len, float* out,
                                    void* workspace, size_t workspace_bytes, const vsl_sparse_mask* mask,
                                    void* stream);
VSL_API int vsl_flash_decode_tc_sparse(const float* q, const void* k_cache, const void* v_cache, int n_pages,
                                       const int32_t* page_table, int max_pages, int page_size, const int32_t* pos,
                                       int B, int n_heads, int n_kv, int head_dim, int max_len, float* out,
                                       void* workspace, size_t workspace_bytes, const vsl_sparse_mask* mask,
                                       void* stream);

/* Decode attention for short caches (same semantics and cache layout as vsl_flash_decode_sparse;
 * fp16 or fp32 KV, head_dim 64 or 128, up to 8 query heads per KV group, page_size a multiple of
 * 64): one CTA per (sequence, KV group) processes 256 positions (128 with fp32 KV) at a time and
 * needs no workspace. status (nullable device int) receives VSL_ERR_TIMEOUT if a bounded wait
 * expires. Meant for caches of up to about a thousand positions. */
VSL_API int vsl_flash_decode_short(const float* q, const void* k_cache, const void* v_cache, int kvdtype,
                                   const int32_t* page_table, int max_pages, int page_size, const int32_t* pos, int B,
                                   int n_heads, int n_kv, int head_dim, int max_len, float* out,
                                   const vsl_sparse_mask* mask, int* status, void* stream);

/* Prompt attention (the reference runs attention.comp once per prompt token during its prompt
 * pass, VulkanSymbioteEngine.cpp:678-765): n_rows query rows of ONE sequence, row r at position
 * pos[r] and attending to positions [first, pos[r]] of the cache (first from the sparse mask,
 * 0 when mask is NULL or dense), with the rows' own K and V already in the cache. page_row is
 * that sequence's page-table row (max_pages entries); q and out are [n_rows][n_heads][128]
 * fp32. fp16 KV, head_dim 128, page_size a multiple of 64; query blocks of 128 rows on the
 * tcgen05 tensor cores, one CTA per (head, block). status (nullable device int) receives
 * VSL_ERR_TIMEOUT if a bounded wait expires. No workspace. */
VSL_API int vsl_flash_prefill(const float* q, const void* k_cache, const void* v_cache, int n_pages,
                              const int32_t* page_row, int max_pages, int page_size, const int32_t* pos, int n_rows,
                              int n_heads, int n_kv, int head_dim, int max_len, float* out,
                              const vsl_sparse_mask* mask, int* status, void* stream);

/* Allocation-free form of vsl_flash_decode (no counterpart in the reference). For callers
 * that must not have the library allocate device memory -- hosts that own every device
 * byte through their own pool or budget, or loops that cannot take an allocation's implicit
 * synchronisation -- the split-K scratch comes from a fixed 4 MiB device array inside
 * libvsl.so (one per GPU that loads the library, held until the process exits). Shapes
 * whose scratch (vsl_flash_decode_workspace_size) exceeds 4 MiB are rejected with
 * VSL_ERR_UNSUPPORTED. The first call on a device looks up the array's device address
 * with that device current, so make that first call before any stream capture. Every
 * call shares the one array: calls that can overlap on the GPU (different streams, or
 * different host threads on the same device) race and must be serialised by the caller.
 * Each call clears the split counters it needs before launching. The looked-up address is kept
 * per device for the rest of the process: a cudaDeviceReset on that device ends the context the
 * address belongs to, so after one this entry point must not be called again in that process. */
VSL_API int vsl_flash_decode_noalloc(const float* q, const void* k_cache, const void* v_cache, int kvdtype,
                                     const int32_t* page_table, int max_pages, int page_size, const int32_t* pos,
                                     int B, int n_heads, int n_kv, int head_dim, int max_len, int split_len,
                                     float* out, void* stream);

/* lm_head projection fused with the sampler (replaces final_projection_with_weights
 * :3028-3130 and sample_token :1540-1553). Computes logits[b][n] for the local vocab slice
 * (global index = vocab_offset + n) and folds each row into argmax_slots[b] (uint64,
 * must be zero before the call) with a 64-bit max of (value key, ~index): the largest
 * value wins and ties go to the lowest index, like greedy_sampling's strict '>' scan
 * (:1794-1804). With temperature > 0 the folded value is logit/temperature + Gumbel noise
 * drawn from (seed, *step_counter, b, index), which samples the softmax distribution. */
VSL_API int vsl_lm_head_sample(int wdtype, const void* W, int V_local, int K, const float* x, const float* norm_w,
                       float eps, int B, float* logits, unsigned long long* argmax_slots, int vocab_offset,
                       float temperature, uint64_t seed, const int32_t* step_counter, void* stream);

/* Greedy argmax of fp32 logits [B][V] (first maximum). */
VSL_API int vsl_argmax(const float* logits, int B, int V, int32_t* out_ids, void* stream);

/* Fill n elements [start, start+n) of seeded synthetic tensor `tensor_id` on the device
 * (Irwin-Hall(4) of splitmix64 lanes scaled to standard deviation sigma, rounded to dtype).
 * Bit-identical to the host generator used to write GGUF fixtures. */
VSL_API int vsl_synth_fill(void* dst, int dtype, uint64_t seed, uint64_t tensor_id, uint64_t start, uint64_t n,
                   double sigma, void* stream);

/* One-shot peer-memory all-reduce of the tensor-parallel engine (it stands where an NCCL
 * all-reduce would follow each row-parallel projection; the reference has no multi-GPU path).
 * Each rank owns a receive buffer of vsl_p2p_buffer_size(n_ranks, cap_bytes) bytes (cap_bytes a
 * multiple of 4), 256-byte aligned and zero-filled once; bases[r] is rank r's buffer as this rank
 * addresses it (its own buffer, or a CUDA IPC / peer mapping of another GPU's). op 0 sums n fp32
 * values, op 1 takes the maximum of n uint64 keys, in place on `data` (16-byte aligned, n * element
 * size <= cap_bytes). The message travels as 8-byte words of a 32-bit piece and the call's epoch,
 * so arrival needs no separate flag or fence. It is cut into chunks of at least 1 KB, one CTA
 * each: a CTA stores its chunk into every rank's buffer, then waits up to wait_ns nanoseconds for
 * every rank's words in its own buffer and sums them in rank order, so all ranks get identical
 * bits. epochs is a zero-filled device array of 64 uint64 call counters (one per chunk) that every
 * call advances, also one that timed out; status (device int, may be NULL) receives
 * VSL_ERR_TIMEOUT when a peer's words never arrived, and the data are then left partly unreduced
 * (a call that finds VSL_ERR_TIMEOUT already in status only advances its epochs). Every rank makes
 * the same sequence of calls with the same n; one launch on `stream`. */
VSL_API int vsl_p2p_buffer_size(int n_ranks, size_t cap_bytes, size_t* bytes);
VSL_API int vsl_p2p_allreduce(void* const* bases, int n_ranks, int rank, size_t cap_bytes, void* data, int n, int op,
                              uint64_t* epochs, int* status, uint64_t wait_ns, void* stream);

/* ======================================================================================
 * Engine (replaces VulkanSymbioteEngine's decode loop, VulkanSymbioteEngine.cpp:678-765)
 * ====================================================================================== */

typedef struct vsl_engine vsl_engine;

typedef struct {
    int n_layers;
    int d_model;
    int n_heads;
    int n_kv_heads;
    int head_dim;
    int ffn;
    int vocab;
    float rope_theta;
    float rms_eps;
    int wdtype; /* VSL_F32 / VSL_F16 / VSL_BF16 / VSL_Q8_0 / VSL_Q4_0 / VSL_Q4_1 (every projection,
                   the embedding table and lm_head share it)                    */
} vsl_model_config;

typedef struct {
    int device;        /* CUDA device ordinal                                          */
    int max_batch;     /* sequences decoded together (B)                               */
    int max_seq;       /* KV positions per sequence                                    */
    int kv_dtype;      /* VSL_F32 / VSL_F16; -1 = F32 for F32 models, else F16         */
    int page_size;     /* KV page size in positions (0 = 64)                           */
    int split_len;     /* flash-decode positions per CTA (0 = automatic)               */
    int tp_rank;       /* tensor-parallel rank                                         */
    int tp_size;       /* tensor-parallel world size (1 = no NCCL)                     */
    const void* nccl_id; /* 128-byte ncclUniqueId from vsl_nccl_unique_id (tp_size > 1)  */
    double vram_budget_gb; /* 0 = no cap; above the cap layers stream from pinned host */
    int use_graph;     /* capture the decode step in a CUDA graph (default 1)          */
    int use_pdl;       /* programmatic dependent launch between kernels (default 1)    */
    int use_fused;     /* must be 0 (the default): decode steps run one kernel per operation,
                          replayed as a CUDA graph with programmatic dependent launch; the
                          persistent single-kernel step this field selected measured slower
                          and was removed (1 is refused with VSL_ERR_UNSUPPORTED)          */
    int use_p2p;       /* tensor parallel: 1 (default) = one-shot NVLink peer-memory all-reduces
                          (CUDA IPC buffers, one kernel per reduction); 0 = NCCL            */
    int legacy_q4;     /* 1 = read GGUF Q4_0 / Q4_1 nibbles in the reference loader's order
                          (GGUFLoader.cpp:1146-1160: element 2i low, 2i+1 high nibble of
                          byte i); 0 (default) = ggml's order (element i low, i+16 high)  */
    int sparse_min_len; /* long-context sparse attention, the reference's use_sparse_attention
                          (VulkanSymbioteEngine.cpp:788; sparse_attention.comp:77-131): a query at
                          position pos of a sequence longer than sparse_min_len attends to the
                          window vsl_sparse_mask describes. 0 (default) = dense attention at every
                          length; the reference switches at 8192                           */
    int sparse_window;   /* window W (0 = 512)                                               */
    int sparse_global;   /* global tokens G (0 = 16)                                         */
    int sparse_block;    /* block BLK (0 = 1024)                                             */
    int attn_route;      /* decode attention: 0 (default) = tcgen05-score attention when max_seq >= 2048
                          and max_batch >= 8, the short-cache kernel (one CTA per sequence and KV
                          group, 256-position rounds) when max_seq <= 1024, the split-K kernel
                          otherwise; 1 = split-K always; 2 = tcgen05 attention always (fp16 KV,
                          head_dim 128); 3 = the short-cache kernel always                  */
    int attn_prefetch;   /* 1 = the split-K attention kernel requests the output projection's weights
                          into L2 while it runs; 0 (default) = it does not (measured faster)  */
    int p2p_chunk_bytes; /* tensor parallel with use_p2p: bytes of the residual all-reduce's message
                          one CTA moves (0 = automatic: 1 KB chunks, at most 64 per message);
                          larger values mean fewer, longer CTAs. Same value on every rank.   */
    int nccl_timeout_ms; /* tensor parallel: the longest the host waits for work that involves the
                          other ranks (one call's stream work); past it, or when NCCL reports an
                          asynchronous error, the communicator is aborted, the call returns
                          VSL_ERR_TIMEOUT / VSL_ERR_NCCL and the engine refuses further work with
                          VSL_ERR_STATE (recreate it). 0 = 120000 (two minutes)               */
} vsl_engine_options;

VSL_API void vsl_engine_default_options(vsl_engine_options* opt);

/* Block-quantized weights (VSL_Q8_0 / VSL_Q4_0 / VSL_Q4_1) on the device: each row of K elements
 * (K a multiple of 32) is [quants: K bytes (Q8_0) or K/2 bytes (Q4_x)][K/32 fp16 scales, padded
 * to 16 bytes] and, for Q4_1 only, [K/32 fp16 minimums, padded to 16 bytes]; Q4_x byte i of a
 * block holds element i (low nibble) and i+16 (high nibble), value (nibble - 8) * d (Q4_0) or
 * nibble * d + m (Q4_1); Q8_0 value int8 * d. vsl_weight_row_bytes gives the row pitch (any dtype);
 * vsl_repack_gguf_rows converts rows [row0, row0+nrows) x columns [col0, col0+ncols) of a GGUF
 * tensor's block data (host) into that layout (host, row pitch out_ld bytes). The projection
 * kernels (vsl_gemv, vsl_qkv_rope_append, vsl_lm_head_sample) accept these dtypes. */
VSL_API int vsl_weight_row_bytes(int dtype, int K, size_t* bytes);
/* Seeded block-quantized tensor [rows][cols] (the engine's synthetic weights) written in the
 * device layout with row pitch row_pitch bytes (>= vsl_weight_row_bytes). */
VSL_API int vsl_synth_fill_q(void* dst, int dtype, size_t row_pitch, uint64_t seed, uint64_t tensor_id, size_t rows,
                             size_t cols, double sigma, void* stream);
VSL_API int vsl_repack_gguf_rows(int dtype, const void* blocks, size_t cols, size_t row0, size_t nrows, size_t col0,
                                 size_t ncols, void* out, size_t out_ld, int legacy_q4);

/* ======================================================================================
 * GGUF inspection (host only, no GPU needed)
 * ====================================================================================== */

/* Model configuration of a GGUF file as the engine would load it (GGUFLoader::load +
 * get_model_config, vk_symbiote/src/GGUFLoader.cpp:625-663, 673-728). */
VSL_API int vsl_gguf_model_config(const char* path, vsl_model_config* out);

/* Tensor lookup: ggml type id, dimensions (ne[0] innermost; unused entries 0) and absolute
 * file offset of the data (GGUFLoader::get_tensor, GGUFLoader.h:280). */
VSL_API int vsl_gguf_tensor_info(const char* path, const char* name, int* ggml_type, uint64_t ne[4], uint64_t* file_offset);


/* ncclUniqueId bytes for tensor-parallel engines (call on rank 0, broadcast to the rest).
 * An id forms exactly one communicator: every tensor-parallel engine group needs a fresh id. */
VSL_API int vsl_nccl_unique_id(void* out128);

/* Load a GGUF model (GGUFLoader::load + load_all_weights, VulkanSymbioteEngine.cpp:1114-1175,
 * 2189-2213): pinned-host staging and cudaMemcpyAsync into one HBM arena, native dtype. */
VSL_API int vsl_engine_create_gguf(const char* path, const vsl_engine_options* opt, vsl_engine** out);

/* Create an engine whose weights are filled on the device by the seeded generator
 * (identical tensors to a GGUF written by vsl/synth.py with the same seed). */
VSL_API int vsl_engine_create_synthetic(const vsl_model_config* cfg, uint64_t seed, double sigma,
                                const vsl_engine_options* opt, vsl_engine** out);

VSL_API int vsl_engine_destroy(vsl_engine* e);
VSL_API int vsl_engine_get_config(const vsl_engine* e, vsl_model_config* out);

/* Clear all sequences (clear_kv_cache, VulkanSymbioteEngine.h:116). */
VSL_API int vsl_engine_reset(vsl_engine* e);

/* Fill KV positions [0, n_pos) of the first B sequences with seeded values and set their
 * next position to n_pos (the 8B long-context workload's prefilled cache). */
VSL_API int vsl_engine_fill_kv_synthetic(vsl_engine* e, uint64_t seed, double sigma, int n_pos, int B);

/* Queue token ids to feed: ids [n_steps][B] (host). Step s consumes forced[s][b] when s is
 * below the forced count, otherwise the id sampled at step s-1. */
VSL_API int vsl_engine_set_forced(vsl_engine* e, const int32_t* ids, int n_steps, int B);

/* Run n_steps decode steps for B active sequences entirely on the device (graph replays);
 * sampled ids accumulate in the engine's token log. temperature <= 0 is greedy. */
VSL_API int vsl_engine_run(vsl_engine* e, int n_steps, int B, float temperature, uint64_t seed);

/* One host-driven step: copy ids (host, [B]) in, decode, copy sampled ids (host, [B]) out,
 * and optionally the logits (host, [B][vocab], gathered across TP ranks on every rank). */
VSL_API int vsl_engine_step_host(vsl_engine* e, const int32_t* ids, int B, int32_t* out_ids, float* out_logits);

/* Copy the token log (ids sampled at steps [0, n)) to host memory [n][B]. */
VSL_API int vsl_engine_read_tokens(vsl_engine* e, int n, int B, int32_t* out);

/* Positions of the B sequences (host copy). */
VSL_API int vsl_engine_positions(vsl_engine* e, int B, int32_t* out);

/* Greedy / temperature generation from a host prompt: prompt (n_prompt ids) for sequence 0,
 * up to max_new tokens into out_ids; stops early at any id in stop_ids (the reference stops
 * on 0 or 2, VulkanSymbioteEngine.cpp:747-749). *n_out receives the count. */
VSL_API int vsl_engine_generate(vsl_engine* e, const int32_t* prompt, int n_prompt, int max_new, float temperature,
                        uint64_t seed, const int32_t* stop_ids, int n_stop, int32_t* out_ids, int* n_out);

/* The stream the engine launches its work on (cudaStream_t as void*). */
VSL_API void* vsl_engine_stream(vsl_engine* e);

/* Kernels launched per decode step and bytes of weights + KV read per step at the
 * current positions (algorithmic bytes for the roofline). */
VSL_API int vsl_engine_step_stats(vsl_engine* e, int B, int* kernels_per_step, double* bytes_per_step);

/* Device bytes held by the engine: weights (HBM arena), paged KV cache, and everything
 * else (activations, token log, attention workspace). Feeds get_vram_stats(). */
VSL_API int vsl_engine_memory_stats(vsl_engine* e, size_t* weight_bytes, size_t* kv_bytes, size_t* other_bytes);

/* Prompt pass (the batched prompt processing the reference's generate lacks: it re-runs the whole
 * sequence per token, VulkanSymbioteEngine.cpp:678-765): ids[0..n) are positions pos..pos+n-1 of
 * sequence `seq`, processed up to 64 at a time as rows of one batch (tensor-core projections; each
 * row attends causally through its own position over the sequence's pages). Their KV is written,
 * pos advances by n, and the sequence's next input becomes the greedy argmax of the last prompt
 * token's logits, returned in *next_id (logits: optional [vocab] of that token). Decoding then
 * continues with vsl_engine_run / vsl_engine_step_host. */
VSL_API int vsl_engine_prefill(vsl_engine* e, const int32_t* ids, int n, int seq, int32_t* next_id, float* logits);

/* Batched serving (the reference's generate_text_batch, VulkanSymbioteEngine.cpp:850-935, loops
 * over its prompts one at a time): prompts = n_seq prompts concatenated, lens[b] ids each
 * (n_seq <= max_batch). Each sequence gets its own prompt pass, then all decode together, one
 * graph-launched step per token for the whole batch. out_ids[b * max_new + k] receives sequence
 * b's ids, n_out[b] how many (a sequence ends after emitting one of stop_ids). */
VSL_API int vsl_engine_generate_batch(vsl_engine* e, const int32_t* prompts, const int* lens, int n_seq, int max_new,
                                      float temperature, uint64_t seed, const int32_t* stop_ids, int n_stop,
                                      int32_t* out_ids, int* n_out);

/* Continuous batching: free sequence slot `seq` (position 0; the other slots keep their state),
 * then vsl_engine_prefill(e, new_prompt, n, seq, ...) admits a new request into it while the
 * others continue to decode through vsl_engine_run. */
VSL_API int vsl_engine_reset_seq(vsl_engine* e, int seq);

/* ======================================================================================
 * Tokenizer (host only): SentencePiece BPE from a GGUF vocabulary (tokenizer.ggml.model
 * "llama"), else the reference's byte-level behaviour (Tokenizer.cpp:113-198).
 * vsl_tokenize writes the ids (BOS first when the vocabulary asks for it) and their count
 * in *n (VSL_ERR_BOUNDS if cap is smaller); vsl_detokenize the UTF-8 text and its length.
 * ====================================================================================== */
typedef struct vsl_tokenizer vsl_tokenizer;
VSL_API int vsl_tokenizer_create_gguf(const char* path, vsl_tokenizer** out);
VSL_API void vsl_tokenizer_destroy(vsl_tokenizer* t);
VSL_API int vsl_tokenizer_info(vsl_tokenizer* t, int* vocab_size, int* is_subword, int32_t* bos_id, int32_t* eos_id);
VSL_API int vsl_tokenize(vsl_tokenizer* t, const char* text, size_t len, int32_t* out, int cap, int* n);
VSL_API int vsl_detokenize(vsl_tokenizer* t, const int32_t* ids, int n, char* out, size_t cap, size_t* len);

/* Weight residency under vram_budget_gb (replaces PackManager::get_vram_stats and the pack
 * scheduler's state, NomadPack.cpp:1190-1249, 1323-1326; VulkanSymbioteEngine.cpp:1555-1599):
 * layers 0..resident_layers-1 stay in HBM, the other streamed_layers live in pinned host memory
 * and are copied into two rotating HBM slots every step (streamed_bytes_per_step over the host
 * link). Without a budget, or when the model fits, streamed_layers is 0. */
VSL_API int vsl_engine_residency(vsl_engine* e, uint32_t* resident_layers, uint32_t* streamed_layers,
                                 uint64_t* streamed_bytes_per_step, uint64_t* host_bytes);

/* The residency plan itself (pure host arithmetic, what the engine applies at creation):
 * layer_bytes per decoder layer, n_layers, fixed_bytes that must stay in HBM (KV cache,
 * activations, workspaces, embeddings, lm_head), budget_gb (0 = no cap). Returns
 * VSL_ERR_OOM when the budget cannot hold the fixed part plus two layer slots. */
VSL_API int vsl_pack_plan(uint64_t layer_bytes, uint32_t n_layers, uint64_t fixed_bytes, double budget_gb,
                          uint32_t* resident_layers, uint32_t* streamed_layers);

/* Sticky device status word of the engine (0 = OK; VSL_ERR_TIMEOUT / VSL_ERR_BOUNDS set by
 * kernels that gave up on a bounded wait or rejected an index). */
VSL_API int vsl_engine_device_status(vsl_engine* e, int* status);

/* Failure injection for tests (failures are made on the host, never by faulting a GPU): set
 * the sticky device status word to `code` (VSL_OK or a VSL_ERR_*) as a kernel that gave up on a
 * bounded wait or rejected an index would. The next host-facing call that reads the word
 * (vsl_engine_step_host, vsl_engine_prefill, vsl_engine_generate, vsl_engine_generate_batch after
 * their decode steps) returns it as its error; vsl_engine_reset clears it. */
VSL_API int vsl_engine_inject_status(vsl_engine* e, int code);

#ifdef __cplusplus
}
#endif

#endif /* VSL_H */
