// DecodeEngine: the B200 decode token loop behind vsl_engine_* and VulkanSymbioteEngine.
//
// One engine per GPU (tensor-parallel rank). All weights live in one HBM arena, laid out
// per layer as one contiguous block [Wqkv | Wo | Wgate/up interleaved | Wdown | norms], so
// a layer can also be streamed as a single copy when the model exceeds the HBM budget.
// A decode step is one CUDA graph (captured once per batch size / sampler mode): the ids,
// positions, step counter and token log are device-resident, so consecutive steps run
// with no host round trip.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <map>
#include <memory>
#include <string>
#include <vector>

#include "../../../include/vk_symbiote/GGUFLoader.h"
#include "../../../include/vk_symbiote/NomadPack.h"
#include "kernels.h"
#include "../kernels/p2p_allreduce.h"
#include "../../../include/vsl.h"

namespace vsl {

struct LayerPtrs {
    void* wqkv = nullptr;   // [(nh_l + 2 nkv_l) hd][d]
    void* wo = nullptr;     // [d][nh_l hd]
    void* wgu = nullptr;    // [2 F_l][d], rows (gate_i, up_i) interleaved
    void* wd = nullptr;     // [d][F_l]
    float* attn_norm = nullptr;
    float* ffn_norm = nullptr;
    void* k_cache = nullptr;  // [n_pages][nkv_l][page][hd]
    void* v_cache = nullptr;
    // streamed layers (over the HBM budget): weights live at `host` (pinned) and are copied
    // into HBM slot `slot` each step; the pointers above then address the slot
    char* host = nullptr;
    int slot = -1;
};

class DecodeEngine {
public:
    static int create(const vsl_model_config& cfg, const vsl_engine_options& opt, std::unique_ptr<DecodeEngine>& out);
    ~DecodeEngine();

    int load_gguf(vk_symbiote::GGUFLoader& loader);
    int init_synthetic(uint64_t seed, double sigma);

    int reset();
    int fill_kv_synthetic(uint64_t seed, double sigma, int n_pos, int B);
    int set_forced(const int32_t* ids, int n_steps, int B);
    int run(int n_steps, int B, float temperature, uint64_t seed);
    int step_host(const int32_t* ids, int B, int32_t* out_ids, float* out_logits);
    // Prompt pass: positions pos..pos+n-1 of sequence `seq` run as up to 128 rows at a time
    // (tensor-core projections, causal attention through per-row positions over the sequence's
    // pages); writes their KV and leaves `seq` ready to decode the token sampled greedily from
    // the last prompt token's logits.
    int prefill(const int32_t* ids, int n, int seq, int32_t* next_id, float* out_logits, float temperature = 0.0f,
                uint64_t seed = 0);
    // Free one sequence slot (position 0) while the others keep their state.
    int reset_seq(int seq);
    // n_seq prompts (concatenated, lens[b] ids each): one prompt pass per sequence, then batched
    // decode steps; out_ids[b * max_new + k], n_out[b] ids per sequence (stop ids end a sequence).
    int generate_batch(const int32_t* prompts, const int* lens, int n_seq, int max_new, float temperature,
                       uint64_t seed, const int32_t* stop_ids, int n_stop, int32_t* out_ids, int* n_out);
    int read_tokens(int n, int B, int32_t* out);
    int positions(int B, int32_t* out);
    int generate(const int32_t* prompt, int n_prompt, int max_new, float temperature, uint64_t seed,
                 const int32_t* stop_ids, int n_stop, int32_t* out_ids, int* n_out);
    int device_status(int* status);
    // Test hook: write `code` into the sticky status word on the engine's stream, as a kernel that
    // gave up on a bounded wait or rejected an index would (failures are made on the host).
    int inject_status(int code);
    int step_stats(int B, int* kernels, double* bytes);

    const vsl_model_config& config() const { return cfg_; }
    cudaStream_t stream() const { return stream_; }
    int max_batch() const { return opt_.max_batch; }
    int max_seq() const { return opt_.max_seq; }
    size_t arena_bytes() const { return arena_bytes_; }
    size_t kv_bytes() const { return kv_bytes_; }
    size_t other_bytes() const { return act_bytes_ + fd_ws_bytes_ + tc_ws_bytes_ + fdtc_ws_bytes_; }
    vk_symbiote::PackResidency residency() const { return residency_; }

private:
    DecodeEngine() = default;
    int init(const vsl_model_config& cfg, const vsl_engine_options& opt);
    int alloc_buffers();
    int enqueue_step(int B, float temperature, uint64_t seed);
    int get_graph(int B, float temperature, uint64_t seed, cudaGraphExec_t* exec);
    // buffers of one pass over the decoder layers (decode step or prefill chunk)
    struct StepBufs {
        float* x;
        float* q;
        float* attn;
        float* act;
        int32_t* pos;
        int32_t* pages;
        void* fd_ws;
        size_t fd_bytes;
        void* fdtc_ws;
        size_t fdtc_bytes;
        const TcRoute* tc;
        bool shared_pages;  // rows are consecutive positions of one sequence (prompt chunk)
    };
    int enqueue_layers(const StepBufs& sb, int B);
    static constexpr int PF_ROWS = 128;  // prompt rows per prefill chunk (one query block)
    int alloc_prefill();
    void* pf_mem_ = nullptr;
    int32_t* pf_ids_ = nullptr;   // [PF] ids, then [PF] positions, then [PF][max_pages] page rows
    int32_t* pf_pos_ = nullptr;
    int32_t* pf_pages_ = nullptr;
    float* pf_x_ = nullptr;
    float* pf_q_ = nullptr;
    float* pf_attn_ = nullptr;
    float* pf_act_ = nullptr;
    float* pf_logits_ = nullptr;
    unsigned long long* pf_slot_ = nullptr;
    int32_t* pf_next_ = nullptr;
    int32_t* pf_h_ = nullptr;     // pinned staging of ids / positions / page rows
    void* pf_fd_ws_ = nullptr;
    size_t pf_fd_bytes_ = 0;
    bool pf_attn_tc_ = false;  // prompt chunks take the tensor-core prompt attention
    bool short_attn_ = false;  // decode steps take the short-cache attention kernel
    void* pf_tc_ws_ = nullptr;
    void* pf_x2n_ = nullptr;  // gate/up -> down split activations of the prompt pass
    TcRoute pf_tc_route_ = {};
    std::vector<int32_t> pt_host_;  // host copy of the page table
    int allreduce_sum(float* buf, int count);
    int check_cuda(cudaError_t e, const char* what);
    // Wait for the engine's stream. Without tensor parallelism this is cudaStreamSynchronize;
    // with it, a bounded watched wait (watchdog.h) that aborts the communicator and marks the
    // engine failed when a peer never arrives.
    int sync();
    // After a sync: the sticky device status word; non-zero statuses are returned as errors
    // (a timed-out peer exchange also marks a tensor-parallel engine failed).
    int check_device_status(const char* what);
    // VSL_ERR_STATE once the engine has failed (a peer exchange timed out or the communicator
    // was aborted): the ranks are out of step and the engine must be recreated.
    int check_usable() const;
    // ncclResult_t of an enqueue on the non-blocking communicator: waits out ncclInProgress
    int nccl_result(int r, const char* what);
    void abort_comm();
    bool failed_ = false;
    int failed_code_ = 0;
    SparseMask sparse_{};  // long-context sparse attention (min_len 0: dense)
    int device_of_layer(int l) const;

    // weight upload helpers: a "source" is full-tensor rows in host (pinned or mapped) or
    // device memory; `copy_rows` / `copy_cols` place the rank's slice into the arena.
    int upload_tensor(const void* src, bool src_host, int dtype_src, size_t rows, size_t cols, void* dst,
                      size_t dst_ld, size_t row0, size_t nrows, size_t col0, size_t ncols);
    int upload_norm(const vk_symbiote::GGUFLoader& loader, const std::string& name, float* dst);

    vsl_model_config cfg_{};
    vsl_engine_options opt_{};
    int nh_l_ = 0, nkv_l_ = 0, ff_l_ = 0, v_l_ = 0, v_off_ = 0;
    int kvdtype_ = VSL_F16;
    int page_size_ = 64, max_pages_ = 0, n_pages_ = 0, split_len_ = 64;
    int fd_splits_ = 0;  // split-K attention: splits per (sequence, group); 0 = max_seq / split_len_
    int fd_grid_splits() const { return fd_splits_ > 0 ? fd_splits_ : (opt_.max_seq + split_len_ - 1) / split_len_; }
    size_t es_ = 2;  // bytes per weight element of the 16/32-bit types (1 for block-quantized)
    // bytes of a weight row of K elements in device layout (quantized rows include their scales)
    size_t wrow(size_t K) const { return weight_row_bytes(cfg_.wdtype, K); }

    cudaStream_t stream_ = nullptr;
    cudaStream_t copy_stream_ = nullptr;
    void* arena_ = nullptr;
    size_t arena_bytes_ = 0;
    void* kv_ = nullptr;
    size_t kv_bytes_ = 0;
    void* act_ = nullptr;  // activations and bookkeeping
    size_t act_bytes_ = 0;
    void* fd_ws_ = nullptr;
    size_t fd_ws_bytes_ = 0;
    void* host_layers_ = nullptr;  // pinned host copies of the streamed layers
    size_t host_layers_bytes_ = 0;
    char* slot_[2] = {nullptr, nullptr};
    cudaEvent_t ev_fork_ = nullptr, ev_copied_[2] = {nullptr, nullptr}, ev_done_[2] = {nullptr, nullptr};
    bool streaming_active_ = false;
    int activate_streaming();
    // tensor parallel: one-shot NVLink peer-memory all-reduces (residual sums, argmax keys)
    P2pPeers p2p_x_{}, p2p_s_{};
    void* p2p_x_local_ = nullptr;
    void* p2p_s_local_ = nullptr;
    void* p2p_x_opened_[P2P_MAX_RANKS] = {};
    void* p2p_s_opened_[P2P_MAX_RANKS] = {};
    bool p2p_ready_ = false;
    unsigned long long* ar_epochs_ = nullptr;  // per-chunk device call counters of the two all-reduces
    int setup_p2p();
    void* fdtc_ws_ = nullptr;  // long-context attention (tcgen05 scores) workspace; null = split-K kernel
    size_t fdtc_ws_bytes_ = 0;
    void* tc_ws_ = nullptr;  // tensor-core route of batched projections (batch >= 5, 16-bit weights)
    void* x2n_ = nullptr;    // gate/up -> down split activations of the decode step
    size_t tc_ws_bytes_ = 0;
    TcRoute tc_route_ = {};

    void* tok_embd_ = nullptr;
    void* lm_head_ = nullptr;
    float* out_norm_ = nullptr;
    std::vector<LayerPtrs> layers_;
    size_t layer_bytes_ = 0;

    float* rope_cos_ = nullptr;
    float* rope_sin_ = nullptr;
    int32_t* page_table_ = nullptr;

    float* x_ = nullptr;
    float* q_ = nullptr;
    float* attn_ = nullptr;
    float* act_ffn_ = nullptr;
    float* logits_ = nullptr;
    float* logits_full_ = nullptr;
    unsigned long long* slots_ = nullptr;
    int32_t* ids_ = nullptr;
    int32_t* pos_ = nullptr;
    int32_t* step_ = nullptr;
    int32_t* n_forced_ = nullptr;
    int32_t* forced_ = nullptr;
    int32_t* log_ = nullptr;
    int32_t* sampled_ = nullptr;
    int* status_ = nullptr;
    int l2_bytes_ = 0;  // the device's L2 capacity (caps the attention kernel's L2 prefetch)
    int log_cap_ = 0;

    // pinned host staging for step_host
    int32_t* h_ids_ = nullptr;
    int32_t* h_out_ = nullptr;
    float* h_logits_ = nullptr;

    std::vector<int32_t> pos_host_;
    int steps_host_ = 0;

    // one captured step per (batch, temperature, seed): the sampler parameters are baked
    // into the lm_head launch
    struct GraphKey {
        int B;
        float temperature;
        uint64_t seed;
        bool operator<(const GraphKey& o) const {
            if (B != o.B) return B < o.B;
            if (temperature != o.temperature) return temperature < o.temperature;
            return seed < o.seed;
        }
    };
    std::map<GraphKey, cudaGraphExec_t> graphs_;


    void* nccl_ = nullptr;  // ncclComm_t
    vk_symbiote::PackResidency residency_{};
};

int make_model_config_from_gguf(const vk_symbiote::GGUFLoader& loader, vsl_model_config* out);

}  // namespace vsl
