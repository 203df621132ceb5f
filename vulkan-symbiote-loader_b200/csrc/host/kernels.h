// Host-side declarations of the engine-internal kernel launchers (defined in csrc/kernels).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "../kernels/p2p_allreduce.h"
#include "../kernels/quant_layout.h"
#include "../kernels/sparse_mask.h"

namespace vsl {

int synthq2d_impl(void* dst, int dtype, size_t dst_ld, uint64_t seed, uint64_t tid, size_t row0, size_t nrows,
                  size_t src_cols, size_t col0, size_t ncols, double sigma, cudaStream_t st);
// GGUF Q8_0 / Q4_0 rows -> device row layout (host memory on both sides). `blocks` is the
// tensor's data ([rows][cols / 32] GGUF blocks); rows [row0, row0 + nrows) x columns
// [col0, col0 + ncols) (multiples of 32) go to out (row pitch out_ld bytes). legacy_q4: read
// Q4_0 nibbles in the reference loader's order (element 2i low nibble, 2i + 1 high nibble of
// byte i, GGUFLoader.cpp:1146-1160) instead of ggml's.
int repack_gguf_rows(int dtype, const void* blocks, size_t cols, size_t row0, size_t nrows, size_t col0, size_t ncols,
                     void* out, size_t out_ld, int legacy_q4);

struct P2pPeers;
int p2p_setup(P2pPeers* out, void** local, void** opened, int rank, int n, int cap, int elem_bytes, void* comm,
              unsigned long long* epoch, int* status, cudaStream_t st);
void p2p_teardown(void* local, void** opened, int n);

// Engine-owned route of batched projections onto the tensor cores (kernels/tc_gemm.cu):
// a workspace of tc_workspace_bytes for the largest projection and batch, zero-filled once.
struct TcRoute {
    void* ws;
    size_t bytes;
    int min_batch;  // projections with at least this many activation rows use the tensor cores
    int* status;    // device status word for expired waits
    void* x2_next = nullptr;  // split activations of the down projection, written by gate/up
    size_t x2_next_bytes = 0;
};
size_t tc_workspace_bytes(int N, int K, int B);
constexpr int TC_MIN_BATCH = 5;  // below this the GEMV streams the weights once per launch anyway
constexpr int TC_MAX_BATCH = 128;  // activation rows per launch (MMA N = 2 x padded rows <= 256)

int embed_impl(int dtype, const void* table, int V, int d, const int32_t* ids, int B, float* x,
               unsigned long long* slots, cudaStream_t st);
int qkv_rope_append_status(int wdtype, const void* Wqkv, int n_heads, int n_kv, int head_dim, int K,
                           const float* x, const float* norm_w, float eps, int B, const int32_t* pos,
                           const float* rope_cos, const float* rope_sin, float* q_out, void* k_cache,
                           void* v_cache, int kvdtype, const int32_t* page_table, int max_pages, int page_size,
                           int* status, cudaStream_t stream, const void* pf_ptr, size_t pf_bytes,
                           const TcRoute* tc = nullptr);
// x_presplit: the tensor-core route reads split activations already in place (x2_in, or the
// workspace start when null); x2_out (SwiGLU on the tensor-core route): write the output as the
// next projection's split activations (hi rows, lo rows from tc_split_rows(B)) instead of y.
int gemv_hint(int wdtype, const void* W, int N, int K, const float* x, int B, float* y, int epilogue,
              const float* norm_w, float eps, const void* pf_ptr, size_t pf_bytes, cudaStream_t stream,
              const TcRoute* tc = nullptr, bool x_presplit = false, const void* x2_in = nullptr,
              void* x2_out = nullptr);
// Whether gemv_hint takes the tensor-core route for this projection (then x_presplit may be used).
bool tc_route_taken(const TcRoute* tc, int wdtype, int N, int K, int B);
size_t tc_split_rows(int B);  // padded activation rows of the split tile (hi rows, then lo rows)
int lm_head_hint(int wdtype, const void* W, int V_local, int K, const float* x, const float* norm_w, float eps, int B,
                 float* logits, unsigned long long* slots, int vocab_offset, float temperature, uint64_t seed,
                 const int32_t* step_counter, const void* pf_ptr, size_t pf_bytes, cudaStream_t stream,
                 const TcRoute* tc = nullptr);
int flash_decode_impl(const float* q, const void* k_cache, const void* v_cache, int kvdtype,
                      const int32_t* page_table, int max_pages, int page_size, const int32_t* pos, int B,
                      int n_heads, int n_kv, int head_dim, int max_len, int split_len, float* out, void* workspace,
                      size_t workspace_bytes, cudaStream_t stream, const void* pf_ptr, size_t pf_bytes,
                      bool shared_pages = false, const SparseMask* sparse = nullptr, int n_splits_max = 0,
                      int* status = nullptr);
// Short caches: one CTA per (sequence, KV group), 256-position rounds, no workspace (attention.cu).
constexpr int FS_MAX_LEN = 1024;  // the engine's automatic route takes it up to this max_seq
int flash_decode_short_impl(const float* q, const void* k_cache, const void* v_cache, int kvdtype,
                            const int32_t* page_table, int max_pages, int page_size, const int32_t* pos, int B,
                            int n_heads, int n_kv, int head_dim, int max_len, float* out, cudaStream_t stream,
                            const void* pf_ptr, size_t pf_bytes, const SparseMask* sparse, int* status);
// workspace of flash_decode_impl with n_splits splits per (sequence, group)
size_t flash_decode_workspace_bytes(int B, int n_heads, int n_kv, int head_dim, int n_splits);
size_t flash_decode_tc_workspace_bytes(int B, int n_kv);
bool flash_decode_tc_supported(int kvdtype, int head_dim, int n_heads, int n_kv, int B, int page_size);
int flash_decode_tc_impl(const float* q, const void* k_cache, const void* v_cache, int n_pages,
                         const int32_t* page_table, int max_pages, int page_size, const int32_t* pos, int B,
                         int n_heads, int n_kv, int max_len, float* out, void* workspace, size_t workspace_bytes,
                         int* status, cudaStream_t st, const SparseMask* sparse = nullptr);
// Prompt attention: up to 128 rows per query block of one sequence (one page-table row), fp16
// KV, head_dim 128; grid = heads x query blocks (attention_prefill.cu).
bool flash_prefill_supported(int kvdtype, int head_dim, int n_heads, int n_kv, int page_size);
// x2 (optional): instead of out, write the rows as the split activations of the following
// tensor-core projection: hi rows [0, P), lo rows [x2_rows, x2_rows + P), n_heads * 128 columns,
// bf16 when x2_bf16 else fp16.
int flash_prefill_impl(const float* q, const void* k_cache, const void* v_cache, int n_pages, const int32_t* page_row,
                       int max_pages, int page_size, const int32_t* pos, int P, int n_heads, int n_kv, int max_len,
                       float* out, int* status, cudaStream_t st, const SparseMask* sparse = nullptr,
                       void* x2 = nullptr, int x2_bf16 = 0, int x2_rows = 0);
constexpr int FDTC_MIN_SEQ = 2048;   // caches from this length on use the tensor-core attention ...
constexpr int FDTC_MIN_BATCH = 8;    // ... when the engine serves at least this many sequences
int synth_impl(void* dst, int dtype, uint64_t seed, uint64_t tid, uint64_t start, uint64_t n, double sigma,
               cudaStream_t st);
int finalize_impl(const unsigned long long* slots, int B, int32_t* ids, int32_t* pos, int32_t* step_counter,
                  const int32_t* forced, const int32_t* n_forced, int32_t* log, int log_cap, int32_t* sampled_out,
                  int max_pos, int* status, cudaStream_t st);
int prefill_finish_impl(const unsigned long long* slot, int32_t* ids, int32_t* pos, int seq, int new_pos,
                        int32_t* next_out, cudaStream_t st);
int sm_count();
bool pdl_enabled();
void set_pdl_enabled(bool on);

}  // namespace vsl
