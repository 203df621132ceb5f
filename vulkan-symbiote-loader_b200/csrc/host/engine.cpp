// DecodeEngine implementation: HBM arena, weight upload (GGUF or seeded), paged KV cache,
// graph-captured decode step, tensor parallelism over NCCL.
//
// Replaces VulkanSymbioteEngine's load_model / load_all_weights / generate
// (vk_symbiote/src/VulkanSymbioteEngine.cpp:1114-1175, 2189-2213, 678-765). The reference
// uploads each tensor as fp32 with a blocking staging copy and re-runs the whole sequence
// with three host round trips per op; here weights keep their GGUF dtype in one arena and
// a decode step is a single graph launch with device-resident ids and positions.
#include "engine.h"

#include <type_traits>

#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <thread>

#include "kernels.h"
#include "status.h"
#include "watchdog.h"

namespace vsl {

int synth2d_impl(void* dst, int dtype, size_t dst_ld, uint64_t seed, uint64_t tid, size_t row0, size_t nrows,
                 size_t src_cols, size_t col0, size_t ncols, double sigma, cudaStream_t st);

static size_t align_up(size_t n, size_t a) { return (n + a - 1) / a * a; }
static size_t dtype_bytes(int dt) { return dt == VSL_F32 ? 4 : 2; }

// tensor ids of the seeded generator (vsl/synth.py)
static constexpr uint64_t TID_TOK_EMBD = 1, TID_OUTPUT = 2;
static uint64_t tid_layer(int l, int k) { return 256ull + 16ull * (uint64_t)l + (uint64_t)k; }
static uint64_t tid_kv(int l, int isv) { return 0x40000000ull + 2ull * (uint64_t)l + (uint64_t)isv; }
enum { K_Q = 1, K_K = 2, K_V = 3, K_O = 4, K_GATE = 6, K_UP = 7, K_DOWN = 8 };

int DecodeEngine::check_cuda(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return VSL_OK;
    if (e == cudaErrorMemoryAllocation) return set_error(VSL_ERR_OOM, "%s: %s", what, cudaGetErrorString(e));
    return set_error(VSL_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

static double seconds_now() {
    return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

static double nccl_timeout_s(const vsl_engine_options& o) {
    return (o.nccl_timeout_ms > 0 ? o.nccl_timeout_ms : 120000) * 1e-3;
}

void DecodeEngine::abort_comm() {
    if (nccl_) ncclCommAbort((ncclComm_t)nccl_);
    nccl_ = nullptr;
}

int DecodeEngine::check_usable() const {
    if (!failed_) return VSL_OK;
    return set_error(VSL_ERR_STATE,
                     "engine: a tensor-parallel exchange failed (status %d); the ranks are out of step, destroy and "
                     "recreate the engine on every rank",
                     failed_code_);
}

int DecodeEngine::nccl_result(int r0, const char* what) {
    ncclResult_t r = (ncclResult_t)r0;
    if (r == ncclInProgress && nccl_) {
        // non-blocking communicator: the call finishes in the background; bounded wait
        const double t0 = seconds_now(), limit = nccl_timeout_s(opt_);
        while (r == ncclInProgress) {
            ncclResult_t q = ncclCommGetAsyncError((ncclComm_t)nccl_, &r);
            if (q != ncclSuccess) r = q;
            if (r == ncclInProgress && seconds_now() - t0 > limit) {
                abort_comm();
                failed_ = true;
                failed_code_ = VSL_ERR_TIMEOUT;
                return set_error(VSL_ERR_TIMEOUT, "%s: not finished after %.1f s; communicator aborted", what, limit);
            }
            if (r == ncclInProgress) std::this_thread::yield();
        }
    }
    if (r == ncclSuccess) return VSL_OK;
    abort_comm();
    failed_ = true;
    failed_code_ = VSL_ERR_NCCL;
    return set_error(VSL_ERR_NCCL, "%s: %s; communicator aborted", what, ncclGetErrorString(r));
}

int DecodeEngine::sync() {
    if (!nccl_) return check_cuda(cudaStreamSynchronize(stream_), "cudaStreamSynchronize");
    cudaError_t qerr = cudaSuccess;
    ncclComm_t comm = (ncclComm_t)nccl_;
    const int rc = watched_wait(
        [&] {
            const cudaError_t e = cudaStreamQuery(stream_);
            if (e == cudaSuccess) return StreamPoll::Done;
            if (e == cudaErrorNotReady) return StreamPoll::Pending;
            qerr = e;
            return StreamPoll::Error;
        },
        [&] {
            ncclResult_t ae = ncclSuccess;
            if (ncclCommGetAsyncError(comm, &ae) != ncclSuccess) return true;
            return ae != ncclSuccess && ae != ncclInProgress;
        },
        [&] { abort_comm(); }, nccl_timeout_s(opt_), seconds_now,
        [](unsigned long long it) {
            // spin first (a decode step's wait is tens of microseconds), then back off
            if (it > 4096) std::this_thread::sleep_for(std::chrono::microseconds(50));
        });
    if (rc == VSL_OK) return VSL_OK;
    if (rc == VSL_ERR_CUDA) return check_cuda(qerr, "stream");
    failed_ = true;
    failed_code_ = rc;
    if (rc == VSL_ERR_TIMEOUT)
        return set_error(rc, "tensor-parallel work not finished after %.1f s: a rank is missing; communicator aborted, "
                             "recreate the engine", nccl_timeout_s(opt_));
    return set_error(rc, "NCCL reported an asynchronous error; communicator aborted, recreate the engine");
}

static int status_error(int st, const char* what) {
    const char* why = st == VSL_ERR_TIMEOUT  ? "a bounded wait expired (a peer rank or a co-operating CTA never arrived)"
                      : st == VSL_ERR_BOUNDS ? "an index was out of range (a position beyond max_seq)"
                                             : "a kernel reported an error";
    return set_error(st, "%s: %s (device status %d)", what, why, st);
}

int DecodeEngine::check_device_status(const char* what) {
    int st = 0;
    if (int rc = check_cuda(cudaMemcpy(&st, status_, 4, cudaMemcpyDeviceToHost), "status read")) return rc;
    if (st == 0) return VSL_OK;
    if (st == VSL_ERR_TIMEOUT && opt_.tp_size > 1) {
        failed_ = true;
        failed_code_ = st;
    }
    return status_error(st, what);
}

#define CK(expr)                                   \
    do {                                           \
        int _rc = check_cuda((expr), #expr);       \
        if (_rc) return _rc;                       \
    } while (0)
#define RC(expr)                 \
    do {                         \
        int _rc = (expr);        \
        if (_rc) return _rc;     \
    } while (0)

int DecodeEngine::create(const vsl_model_config& cfg, const vsl_engine_options& opt,
                         std::unique_ptr<DecodeEngine>& out) {
    std::unique_ptr<DecodeEngine> e(new DecodeEngine());
    int rc = e->init(cfg, opt);
    if (rc) return rc;
    out = std::move(e);
    return VSL_OK;
}

int DecodeEngine::init(const vsl_model_config& cfg, const vsl_engine_options& opt) {
    cfg_ = cfg;
    opt_ = opt;
    const int tp = std::max(1, opt.tp_size);
    opt_.tp_size = tp;
    if (cfg.n_layers <= 0 || cfg.d_model <= 0 || cfg.n_heads <= 0 || cfg.n_kv_heads <= 0 || cfg.ffn <= 0 ||
        cfg.vocab <= 0 || cfg.head_dim <= 0)
        return set_error(VSL_ERR_INVALID, "engine: empty model dimension");
    if (cfg.head_dim != 64 && cfg.head_dim != 128)
        return set_error(VSL_ERR_UNSUPPORTED, "engine: head_dim %d (64 or 128 supported)", cfg.head_dim);
    if (cfg.n_heads % cfg.n_kv_heads || cfg.n_heads / cfg.n_kv_heads > 8)
        return set_error(VSL_ERR_UNSUPPORTED, "engine: %d query heads over %d KV heads", cfg.n_heads, cfg.n_kv_heads);
    if (opt.tp_rank < 0 || opt.tp_rank >= tp) return set_error(VSL_ERR_INVALID, "engine: tp_rank %d of %d", opt.tp_rank, tp);
    if (cfg.n_heads % tp || cfg.n_kv_heads % tp || cfg.ffn % tp || cfg.vocab % tp)
        return set_error(VSL_ERR_UNSUPPORTED, "engine: heads %d, kv heads %d, ffn %d and vocab %d must divide by tp %d",
                         cfg.n_heads, cfg.n_kv_heads, cfg.ffn, cfg.vocab, tp);
    if (opt.max_batch <= 0 || opt.max_batch > 1024 || opt.max_seq <= 0)
        return set_error(VSL_ERR_INVALID, "engine: max_batch %d / max_seq %d", opt.max_batch, opt.max_seq);
    if (cfg.wdtype != VSL_F32 && cfg.wdtype != VSL_F16 && cfg.wdtype != VSL_BF16 && !is_quant(cfg.wdtype))
        return set_error(VSL_ERR_UNSUPPORTED, "engine: weight dtype %d", cfg.wdtype);
    es_ = is_quant(cfg.wdtype) ? 1 : dtype_bytes(cfg.wdtype);  // 16-bit paths test es_ == 2
    if (is_quant(cfg.wdtype) && (cfg.d_model % QBLK || (cfg.ffn / tp) % QBLK || (cfg.n_heads / tp * cfg.head_dim) % QBLK))
        return set_error(VSL_ERR_UNSUPPORTED, "engine: quantized projections need inner dimensions divisible by 32");
    for (size_t k : {(size_t)cfg.d_model, (size_t)cfg.ffn / tp, (size_t)cfg.n_heads / tp * cfg.head_dim})
        if (weight_row_bytes(cfg.wdtype, k) % 16)
            return set_error(VSL_ERR_UNSUPPORTED, "engine: projection inner dimensions must be 16-byte multiples");
    nh_l_ = cfg.n_heads / tp;
    nkv_l_ = cfg.n_kv_heads / tp;
    ff_l_ = cfg.ffn / tp;
    v_l_ = cfg.vocab / tp;
    v_off_ = opt.tp_rank * v_l_;
    kvdtype_ = opt.kv_dtype >= 0 ? opt.kv_dtype : (cfg.wdtype == VSL_F32 ? VSL_F32 : VSL_F16);
    if (kvdtype_ != VSL_F32 && kvdtype_ != VSL_F16) return set_error(VSL_ERR_UNSUPPORTED, "engine: kv dtype %d", kvdtype_);
    page_size_ = opt.page_size > 0 ? opt.page_size : 64;
    if (page_size_ % 64) return set_error(VSL_ERR_INVALID, "engine: page_size %d must be a multiple of 64", page_size_);
    max_pages_ = (opt.max_seq + page_size_ - 1) / page_size_;
    n_pages_ = max_pages_ * opt.max_batch;
    fd_splits_ = 0;  // fixed splits of split_len_ positions over max_seq
    if (opt.split_len > 0) {
        split_len_ = opt.split_len;
    } else {
        // about four CTAs per SM over the whole cache at full length. Many short splits beat fewer
        // long ones at every length measured: a CTA's chunks run one after another through a chain
        // of dependent shared-memory steps, while the splits run on separate SMs (7B batch 1 at
        // ~150 positions: 96 CTAs of one chunk each, 11 us per layer including the combine, against
        // 19 us for 32 CTAs of three chunks)
        const int groups = opt.max_batch * nkv_l_;
        int splits = std::max(1, (4 * 148 + groups - 1) / groups);
        split_len_ = (int)align_up((size_t)((opt.max_seq + splits - 1) / splits), 64);
    }
    if (split_len_ % 64) return set_error(VSL_ERR_INVALID, "engine: split_len %d must be a multiple of 64", split_len_);
    set_pdl_enabled(opt.use_pdl != 0);
    if (opt.attn_route < 0 || opt.attn_route > 3) return set_error(VSL_ERR_INVALID, "engine: attn_route %d", opt.attn_route);
    if (opt.use_fused)
        return set_error(VSL_ERR_UNSUPPORTED, "engine: use_fused (the persistent single-kernel step was removed)");
    if (opt.sparse_min_len < 0 || opt.sparse_window < 0 || opt.sparse_global < 0 || opt.sparse_block < 0)
        return set_error(VSL_ERR_INVALID, "engine: negative sparse attention parameter");
    if (opt.sparse_min_len > 0)  // zeros take the reference's values (Common.h:71-74)
        sparse_ = SparseMask{opt.sparse_min_len, opt.sparse_window ? opt.sparse_window : 512,
                             opt.sparse_global ? opt.sparse_global : 16, opt.sparse_block ? opt.sparse_block : 1024};

    CK(cudaSetDevice(opt.device));
    CK(cudaDeviceGetAttribute(&l2_bytes_, cudaDevAttrL2CacheSize, opt.device));
    CK(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
    CK(cudaStreamCreateWithFlags(&copy_stream_, cudaStreamNonBlocking));
    if (tp > 1) {
        if (!opt.nccl_id) return set_error(VSL_ERR_INVALID, "engine: tp_size %d needs an NCCL unique id", tp);
        ncclUniqueId id;
        memcpy(&id, opt.nccl_id, sizeof(id));
        // non-blocking, so that no host call can wait on a peer without a bound (sync())
        ncclConfig_t ncfg = NCCL_CONFIG_INITIALIZER;
        ncfg.blocking = 0;
        ncclComm_t comm = nullptr;
        ncclResult_t r = ncclCommInitRankConfig(&comm, tp, id, opt.tp_rank, &ncfg);
        nccl_ = comm;
        RC(nccl_result(r, "ncclCommInitRankConfig"));
    }
    RC(alloc_buffers());
    if (nccl_ && opt_.use_p2p && tp <= P2P_MAX_RANKS) RC(setup_p2p());
    return VSL_OK;
}

// Receive buffers of the peer-memory all-reduces, exchanged with the other ranks by CUDA IPC.
int DecodeEngine::setup_p2p() {
    RC(p2p_setup(&p2p_x_, &p2p_x_local_, p2p_x_opened_, opt_.tp_rank, opt_.tp_size, opt_.max_batch * cfg_.d_model, 4,
                 nccl_, ar_epochs_, status_, stream_));
    RC(p2p_setup(&p2p_s_, &p2p_s_local_, p2p_s_opened_, opt_.tp_rank, opt_.tp_size, opt_.max_batch, 8, nccl_,
                 ar_epochs_ + P2P_MAX_CHUNKS, status_, stream_));
    if (opt_.p2p_chunk_bytes > 0) {  // the same value on every rank: the layout does not depend on it
        const int want = (opt_.p2p_chunk_bytes / 4 + 1) / 2 * 2;
        const int whole = (int)(p2p_x_.slot_bytes / 8);
        p2p_x_.chunk_words = std::max(p2p_x_.chunk_words, std::min(want, whole));
    }
    p2p_ready_ = true;
    return VSL_OK;
}

DecodeEngine::~DecodeEngine() {
    if (opt_.device >= 0) cudaSetDevice(opt_.device);
    if (stream_) cudaStreamSynchronize(stream_);
    for (auto& kv : graphs_) cudaGraphExecDestroy(kv.second);
    graphs_.clear();
    p2p_teardown(p2p_x_local_, p2p_x_opened_, opt_.tp_size);
    p2p_teardown(p2p_s_local_, p2p_s_opened_, opt_.tp_size);
    if (nccl_) {
        // non-blocking communicator: finalize (bounded), then free; abort if a peer is gone
        ncclComm_t comm = (ncclComm_t)nccl_;
        ncclResult_t r = ncclCommFinalize(comm);
        const auto t0 = std::chrono::steady_clock::now();
        while (r == ncclInProgress) {
            if (ncclCommGetAsyncError(comm, &r) != ncclSuccess) break;
            if (std::chrono::steady_clock::now() - t0 > std::chrono::seconds(10)) break;
            std::this_thread::yield();
        }
        if (r == ncclSuccess) ncclCommDestroy(comm);
        else ncclCommAbort(comm);
        nccl_ = nullptr;
    }
    cudaFree(arena_);
    cudaFree(kv_);
    cudaFree(act_);
    cudaFree(fd_ws_);
    cudaFree(tc_ws_);
    cudaFree(x2n_);
    cudaFree(pf_mem_);
    cudaFree(pf_fd_ws_);
    cudaFree(pf_tc_ws_);
    cudaFree(pf_x2n_);
    if (pf_h_) cudaFreeHost(pf_h_);
    cudaFree(fdtc_ws_);
    if (host_layers_) cudaFreeHost(host_layers_);
    for (cudaEvent_t ev : {ev_fork_, ev_copied_[0], ev_copied_[1], ev_done_[0], ev_done_[1]})
        if (ev) cudaEventDestroy(ev);
    cudaFreeHost(h_ids_);
    cudaFreeHost(h_out_);
    cudaFreeHost(h_logits_);
    if (stream_) cudaStreamDestroy(stream_);
    if (copy_stream_) cudaStreamDestroy(copy_stream_);
}

int DecodeEngine::alloc_buffers() {
    const vsl_model_config& c = cfg_;
    const size_t d = c.d_model, hd = c.head_dim, mb = opt_.max_batch;
    const size_t qkv_rows = (size_t)(nh_l_ + 2 * nkv_l_) * hd;
    const size_t qd_l = (size_t)nh_l_ * hd;
    const size_t A = 256;
    const size_t b_qkv = align_up(qkv_rows * wrow(d), A), b_wo = align_up(d * wrow(qd_l), A);
    const size_t b_wgu = align_up(2 * (size_t)ff_l_ * wrow(d), A), b_wd = align_up(d * wrow(ff_l_), A);
    const size_t b_norm = align_up(d * 4, A);
    layer_bytes_ = b_qkv + b_wo + b_wgu + b_wd + 2 * b_norm;
    const size_t b_emb = align_up((size_t)c.vocab * wrow(d), A), b_head = align_up((size_t)v_l_ * wrow(d), A);
    layers_.resize(c.n_layers);
    // paged KV cache: per layer K then V, each [n_pages][nkv_l][page][hd]
    const size_t kv_es = dtype_bytes(kvdtype_);
    const size_t b_kv_one = align_up((size_t)n_pages_ * nkv_l_ * page_size_ * hd * kv_es, A);
    kv_bytes_ = 2 * b_kv_one * c.n_layers;
    CK(cudaMalloc(&kv_, kv_bytes_));
    char* k = (char*)kv_;
    for (int l = 0; l < c.n_layers; l++) {
        layers_[l].k_cache = k; k += b_kv_one;
        layers_[l].v_cache = k; k += b_kv_one;
    }

    // activations and bookkeeping
    log_cap_ = opt_.max_seq;
    struct Item { void** dst; size_t bytes; };
    const size_t half = hd / 2;
    Item items[] = {
        {(void**)&x_, mb * d * 4},
        {(void**)&q_, mb * qd_l * 4},
        {(void**)&attn_, mb * qd_l * 4},
        {(void**)&act_ffn_, mb * ff_l_ * 4},
        {(void**)&logits_, mb * v_l_ * 4},
        {(void**)&logits_full_, opt_.tp_size > 1 ? mb * (size_t)c.vocab * 4 : 16},
        {(void**)&slots_, mb * 8},
        {(void**)&ids_, mb * 4},
        {(void**)&pos_, mb * 4},
        {(void**)&sampled_, mb * 4 + 4},  // sampled ids [mb], then the status word
        {(void**)&step_, 4},
        {(void**)&n_forced_, 4},
        {(void**)&forced_, (size_t)log_cap_ * mb * 4},
        {(void**)&log_, (size_t)log_cap_ * mb * 4},
        {(void**)&rope_cos_, (size_t)opt_.max_seq * half * 4},
        {(void**)&rope_sin_, (size_t)opt_.max_seq * half * 4},
        {(void**)&page_table_, mb * (size_t)max_pages_ * 4},
        {(void**)&ar_epochs_, 2 * P2P_MAX_CHUNKS * 8},
    };
    size_t total = 0;
    for (auto& it : items) total += align_up(it.bytes, A);
    act_bytes_ = total;
    CK(cudaMalloc(&act_, total));
    CK(cudaMemset(act_, 0, total));
    char* a = (char*)act_;
    for (auto& it : items) { *it.dst = a; a += align_up(it.bytes, A); }
    status_ = reinterpret_cast<int*>(sampled_ + mb);

    fd_ws_bytes_ = flash_decode_workspace_bytes(opt_.max_batch, nh_l_, nkv_l_, c.head_dim, fd_grid_splits());
    CK(cudaMalloc(&fd_ws_, fd_ws_bytes_));
    CK(cudaMemset(fd_ws_, 0, fd_ws_bytes_));

    // short caches: one CTA per (sequence, KV group), no split combine
    short_attn_ = opt_.attn_route == 3 || (opt_.attn_route == 0 && opt_.max_seq <= FS_MAX_LEN);
    // long caches of several sequences: attention with tcgen05 scores and an even split of the
    // KV over the SMs (with one or a few sequences its merge of many splits is the tail: at 70B
    // batch 1 over 2048 positions 114 us per layer against 38.5 us for the split-K kernel)
    const bool want_tc = opt_.attn_route == 2 ||
                         (opt_.attn_route == 0 && opt_.max_seq >= FDTC_MIN_SEQ && opt_.max_batch >= FDTC_MIN_BATCH);
    if (want_tc &&
        flash_decode_tc_supported(kvdtype_, c.head_dim, nh_l_, nkv_l_, opt_.max_batch, page_size_)) {
        fdtc_ws_bytes_ = flash_decode_tc_workspace_bytes(opt_.max_batch, nkv_l_);
        CK(cudaMalloc(&fdtc_ws_, fdtc_ws_bytes_));
        CK(cudaMemset(fdtc_ws_, 0, fdtc_ws_bytes_));
    }
    // batched projections (5..128 rows, 16-bit weights) run on the tensor cores: one workspace
    // sized for the largest projection of the model
    if (es_ == 2 && !is_quant(c.wdtype) && opt_.max_batch >= TC_MIN_BATCH) {
        const int tb = std::min(opt_.max_batch, TC_MAX_BATCH);
        const int n_max = std::max({(nh_l_ + 2 * nkv_l_) * c.head_dim, c.d_model, 2 * ff_l_, v_l_});
        const int k_max = std::max({c.d_model, nh_l_ * c.head_dim, ff_l_});
        tc_ws_bytes_ = tc_workspace_bytes(n_max, k_max, tb) + 1024;
        CK(cudaMalloc(&tc_ws_, tc_ws_bytes_));
        CK(cudaMemset(tc_ws_, 0, tc_ws_bytes_));
        char* base = reinterpret_cast<char*>(((uintptr_t)tc_ws_ + 1023) & ~(uintptr_t)1023);
        tc_route_ = TcRoute{base, tc_ws_bytes_ - 1024, TC_MIN_BATCH, status_};
        // the gate/up projection writes the down projection's split activations here
        const size_t x2n = 2 * tc_split_rows(tb) * (size_t)ff_l_ * 2;
        CK(cudaMalloc(&x2n_, x2n));
        tc_route_.x2_next = x2n_;
        tc_route_.x2_next_bytes = x2n;
    }


    // ---- weights: resident layers + embeddings + lm_head in one HBM arena; when the model
    // exceeds the HBM budget, the layers that do not fit live in pinned host memory and
    // stream through two rotating HBM slots (NomadPackManager plan) ----
    const size_t emb_bytes = b_emb + b_head + b_norm;
    const size_t fixed = kv_bytes_ + act_bytes_ + fd_ws_bytes_ + tc_ws_bytes_ + fdtc_ws_bytes_ + emb_bytes;
    residency_ = vk_symbiote::NomadPackManager::plan(layer_bytes_, (uint32_t)c.n_layers, fixed,
                                                     (uint64_t)(opt_.vram_budget_gb > 0 ? opt_.vram_budget_gb * 1e9 : 0));
    if (!residency_.feasible)
        return set_error(VSL_ERR_OOM,
                         "engine: a %.2f GB budget cannot hold the KV cache, activations and embeddings (%.2f GB) "
                         "plus two %.2f GB layer slots",
                         opt_.vram_budget_gb, fixed / 1e9, layer_bytes_ / 1e9);
    const int R = (int)residency_.resident_layers;
    const int n_slots = residency_.streamed_layers ? 2 : 0;
    arena_bytes_ = layer_bytes_ * (size_t)(R + n_slots) + emb_bytes;
    CK(cudaMalloc(&arena_, arena_bytes_));
    if (residency_.streamed_layers) {
        host_layers_bytes_ = layer_bytes_ * residency_.streamed_layers;
        CK(cudaHostAlloc(&host_layers_, host_layers_bytes_, cudaHostAllocMapped | cudaHostAllocPortable));
        for (int i = 0; i < 2; i++) {
            CK(cudaEventCreateWithFlags(&ev_copied_[i], cudaEventDisableTiming));
            CK(cudaEventCreateWithFlags(&ev_done_[i], cudaEventDisableTiming));
        }
        CK(cudaEventCreateWithFlags(&ev_fork_, cudaEventDisableTiming));
    }
    char* p = (char*)arena_;
    auto place = [&](LayerPtrs& L, char* base) {
        char* q = base;
        L.wqkv = q; q += b_qkv;
        L.wo = q; q += b_wo;
        L.wgu = q; q += b_wgu;
        L.wd = q; q += b_wd;
        L.attn_norm = (float*)q; q += b_norm;
        L.ffn_norm = (float*)q;
    };
    for (int l = 0; l < R; l++) {
        place(layers_[l], p);
        p += layer_bytes_;
    }
    for (int i = 0; i < n_slots; i++) {
        slot_[i] = p;
        p += layer_bytes_;
    }
    // streamed layers are loaded straight into pinned host memory (mapped, so the synthetic
    // fill kernels and the upload copies write there); activate_streaming() then points them
    // at their slot
    for (int l = R; l < c.n_layers; l++) {
        char* h = (char*)host_layers_ + (size_t)(l - R) * layer_bytes_;
        place(layers_[l], h);
        layers_[l].host = h;
        layers_[l].slot = (l - R) & 1;
    }
    tok_embd_ = p; p += b_emb;
    lm_head_ = p; p += b_head;
    out_norm_ = (float*)p;

    CK(cudaMallocHost((void**)&h_ids_, mb * 4));
    CK(cudaMallocHost((void**)&h_out_, (mb + 1) * 4));
    CK(cudaMallocHost((void**)&h_logits_, mb * (size_t)c.vocab * 4));

    // RoPE tables: cos/sin(pos * theta^(-2i/hd)) evaluated in double (Utils.cpp:101-110)
    std::vector<float> cs((size_t)opt_.max_seq * half), sn((size_t)opt_.max_seq * half);
    for (int ps = 0; ps < opt_.max_seq; ps++)
        for (size_t i = 0; i < half; i++) {
            const double f = std::pow((double)c.rope_theta, -(double)(2 * i) / (double)hd);
            const double ang = (double)ps * f;
            cs[(size_t)ps * half + i] = (float)std::cos(ang);
            sn[(size_t)ps * half + i] = (float)std::sin(ang);
        }
    CK(cudaMemcpy(rope_cos_, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(rope_sin_, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice));
    // identity page table: sequence b owns physical pages [b*max_pages, (b+1)*max_pages)
    std::vector<int32_t> pt(mb * (size_t)max_pages_);
    for (size_t b = 0; b < mb; b++)
        for (int i = 0; i < max_pages_; i++) pt[b * max_pages_ + i] = (int32_t)(b * max_pages_ + i);
    CK(cudaMemcpy(page_table_, pt.data(), pt.size() * 4, cudaMemcpyHostToDevice));
    pt_host_ = pt;
    pos_host_.assign(mb, 0);
    return VSL_OK;
}


// ---------------------------------------------------------------------------------------
// weight upload
// ---------------------------------------------------------------------------------------

// Copy rows [row0, row0+nrows) x cols [col0, col0+ncols) of a row-major [rows][cols] host
// tensor into dst (row pitch dst_ld bytes) through two pinned staging buffers.
int DecodeEngine::upload_tensor(const void* src, bool src_host, int dtype_src, size_t rows, size_t cols, void* dst,
                                size_t dst_ld, size_t row0, size_t nrows, size_t col0, size_t ncols) {
    const size_t es = dtype_bytes(dtype_src);
    if (row0 + nrows > rows || col0 + ncols > cols) return set_error(VSL_ERR_BOUNDS, "upload: slice out of range");
    const bool q = is_quant(dtype_src);
    if (q && (!src_host || cols % QBLK || col0 % QBLK || ncols % QBLK))
        return set_error(VSL_ERR_INVALID, "upload: quantized slices are host-side and block aligned");
    const size_t row_bytes = q ? weight_row_bytes(dtype_src, ncols) : ncols * es;
    if (!src_host) {
        CK(cudaMemcpy2DAsync(dst, dst_ld, (const char*)src + (row0 * cols + col0) * es, cols * es, row_bytes, nrows,
                             cudaMemcpyDefault, copy_stream_));
        CK(cudaStreamSynchronize(copy_stream_));
        return VSL_OK;
    }
    static constexpr size_t STAGE = 64ull << 20;
    void* stage[2] = {nullptr, nullptr};
    cudaEvent_t done[2] = {nullptr, nullptr};
    int rc = VSL_OK;
    for (int i = 0; i < 2 && !rc; i++) {
        rc = check_cuda(cudaMallocHost(&stage[i], STAGE), "pinned staging");
        if (!rc) rc = check_cuda(cudaEventCreateWithFlags(&done[i], cudaEventDisableTiming), "staging event");
    }
    const size_t chunk = std::max<size_t>(1, STAGE / row_bytes);
    int buf = 0;
    for (size_t r = 0; r < nrows && !rc; r += chunk, buf ^= 1) {
        const size_t n = std::min(chunk, nrows - r);
        if (n * row_bytes > STAGE) { rc = set_error(VSL_ERR_UNSUPPORTED, "upload: row larger than staging"); break; }
        rc = check_cuda(cudaEventSynchronize(done[buf]), "staging wait");
        if (rc) break;
        const char* s = (const char*)src + ((row0 + r) * cols + col0) * es;
        char* t = (char*)stage[buf];
        if (q) {  // GGUF blocks -> device row layout
            rc = repack_gguf_rows(dtype_src, src, cols, row0 + r, n, col0, ncols, t, row_bytes, opt_.legacy_q4);
            if (rc) break;
        } else if (ncols == cols) {
            memcpy(t, s, n * row_bytes);
        } else {
            for (size_t i = 0; i < n; i++) memcpy(t + i * row_bytes, s + i * cols * es, row_bytes);
        }
        rc = check_cuda(cudaMemcpy2DAsync((char*)dst + r * dst_ld, dst_ld, t, row_bytes, row_bytes, n,
                                          cudaMemcpyDefault, copy_stream_),
                        "upload copy");
        if (!rc) rc = check_cuda(cudaEventRecord(done[buf], copy_stream_), "staging record");
    }
    cudaStreamSynchronize(copy_stream_);
    for (int i = 0; i < 2; i++) {
        if (done[i]) cudaEventDestroy(done[i]);
        if (stage[i]) cudaFreeHost(stage[i]);
    }
    return rc;
}

int DecodeEngine::upload_norm(const vk_symbiote::GGUFLoader& loader, const std::string& name, float* dst) {
    const vk_symbiote::GGUFTensorInfo* t = loader.get_tensor(name);
    if (!t || t->element_count() != (uint64_t)cfg_.d_model)
        return set_error(VSL_ERR_FORMAT, "gguf: missing or mis-sized norm tensor %s", name.c_str());
    auto v = const_cast<vk_symbiote::GGUFLoader&>(loader).read_tensor_data(*t, true);
    if (!v) return set_error(VSL_ERR_FORMAT, "gguf: cannot read %s (%d)", name.c_str(), v.error());
    CK(cudaMemcpy(dst, v.value().data(), (size_t)cfg_.d_model * 4, cudaMemcpyDefault));
    return VSL_OK;
}

int make_model_config_from_gguf(const vk_symbiote::GGUFLoader& loader, vsl_model_config* out) {
    vk_symbiote::ModelConfig mc = loader.get_model_config();
    const vk_symbiote::GGUFTensorInfo* emb = loader.get_tensor("token_embd.weight");
    if (!emb) return set_error(VSL_ERR_FORMAT, "gguf: token_embd.weight missing");
    int dt;
    switch (emb->data_type) {
        case vk_symbiote::GGMLType::F32: dt = VSL_F32; break;
        case vk_symbiote::GGMLType::F16: dt = VSL_F16; break;
        case vk_symbiote::GGMLType::BF16: dt = VSL_BF16; break;
        case vk_symbiote::GGMLType::Q8_0: dt = VSL_Q8_0; break;
        case vk_symbiote::GGMLType::Q4_0: dt = VSL_Q4_0; break;
        case vk_symbiote::GGMLType::Q4_1: dt = VSL_Q4_1; break;
        default: return set_error(VSL_ERR_UNSUPPORTED, "gguf: token_embd dtype %u", (unsigned)emb->data_type);
    }
    vsl_model_config c = {};
    c.n_layers = (int)mc.num_layers;
    c.d_model = (int)mc.hidden_size;
    c.n_heads = (int)mc.num_attention_heads;
    c.n_kv_heads = (int)mc.num_key_value_heads;
    c.head_dim = (int)mc.head_dim;
    c.ffn = (int)mc.intermediate_size;
    c.vocab = (int)mc.vocab_size;
    c.rope_theta = mc.rope_theta;
    c.rms_eps = mc.rms_epsilon;
    c.wdtype = dt;
    if (const vk_symbiote::GGUFTensorInfo* g = loader.get_tensor("blk.0.ffn_gate.weight"))
        if (g->dimensions.size() == 2) c.ffn = (int)g->dimensions[1];
    *out = c;
    return VSL_OK;
}

int DecodeEngine::load_gguf(vk_symbiote::GGUFLoader& loader) {
    const vsl_model_config& c = cfg_;
    const int r = opt_.tp_rank;
    const size_t d = c.d_model, hd = c.head_dim, qd = (size_t)c.n_heads * hd, kvd = (size_t)c.n_kv_heads * hd;
    auto matrix = [&](const std::string& name, size_t N, size_t K, const void** data) -> int {
        const vk_symbiote::GGUFTensorInfo* t = loader.get_tensor(name);
        if (!t) return set_error(VSL_ERR_FORMAT, "gguf: tensor %s missing", name.c_str());
        if (t->dimensions.size() != 2 || t->dimensions[0] != K || t->dimensions[1] != N)
            return set_error(VSL_ERR_FORMAT, "gguf: %s has shape [%llu,%llu], expected ne=[%zu,%zu]", name.c_str(),
                             (unsigned long long)t->dimensions[0],
                             (unsigned long long)(t->dimensions.size() > 1 ? t->dimensions[1] : 0), K, N);
        const int want = c.wdtype;  // VSL dtype ids are the ggml tensor type ids
        if ((int)t->data_type != want)
            return set_error(VSL_ERR_UNSUPPORTED, "gguf: %s dtype %u differs from the model dtype %d", name.c_str(),
                             (unsigned)t->data_type, want);
        *data = loader.map_tensor(name);
        return VSL_OK;
    };
    const void* src = nullptr;
    RC(matrix("token_embd.weight", c.vocab, d, &src));
    RC(upload_tensor(src, true, c.wdtype, c.vocab, d, tok_embd_, wrow(d), 0, c.vocab, 0, d));
    const char* head_name = loader.get_tensor("output.weight") ? "output.weight" : "token_embd.weight";  // tied
    RC(matrix(head_name, c.vocab, d, &src));
    RC(upload_tensor(src, true, c.wdtype, c.vocab, d, lm_head_, wrow(d), (size_t)v_off_, v_l_, 0, d));
    RC(upload_norm(loader, "output_norm.weight", out_norm_));
    for (int l = 0; l < c.n_layers; l++) {
        const LayerPtrs& L = layers_[l];
        const std::string p = "blk." + std::to_string(l) + ".";
        char* qkv = (char*)L.wqkv;
        RC(matrix(p + "attn_q.weight", qd, d, &src));
        RC(upload_tensor(src, true, c.wdtype, qd, d, qkv, wrow(d), (size_t)r * nh_l_ * hd, (size_t)nh_l_ * hd, 0, d));
        qkv += (size_t)nh_l_ * hd * wrow(d);
        RC(matrix(p + "attn_k.weight", kvd, d, &src));
        RC(upload_tensor(src, true, c.wdtype, kvd, d, qkv, wrow(d), (size_t)r * nkv_l_ * hd, (size_t)nkv_l_ * hd, 0, d));
        qkv += (size_t)nkv_l_ * hd * wrow(d);
        RC(matrix(p + "attn_v.weight", kvd, d, &src));
        RC(upload_tensor(src, true, c.wdtype, kvd, d, qkv, wrow(d), (size_t)r * nkv_l_ * hd, (size_t)nkv_l_ * hd, 0, d));
        // attn_output (llama.cpp name) or attn_o (the reference's name, VulkanSymbioteEngine.cpp:2037)
        const std::string o_name = loader.get_tensor(p + "attn_output.weight") ? p + "attn_output.weight" : p + "attn_o.weight";
        RC(matrix(o_name, d, qd, &src));
        RC(upload_tensor(src, true, c.wdtype, d, qd, L.wo, wrow((size_t)nh_l_ * hd), 0, d, (size_t)r * nh_l_ * hd,
                         (size_t)nh_l_ * hd));
        RC(matrix(p + "ffn_gate.weight", c.ffn, d, &src));
        RC(upload_tensor(src, true, c.wdtype, c.ffn, d, L.wgu, 2 * wrow(d), (size_t)r * ff_l_, ff_l_, 0, d));
        RC(matrix(p + "ffn_up.weight", c.ffn, d, &src));
        RC(upload_tensor(src, true, c.wdtype, c.ffn, d, (char*)L.wgu + wrow(d), 2 * wrow(d), (size_t)r * ff_l_, ff_l_,
                         0, d));
        RC(matrix(p + "ffn_down.weight", d, c.ffn, &src));
        RC(upload_tensor(src, true, c.wdtype, d, c.ffn, L.wd, wrow(ff_l_), 0, d, (size_t)r * ff_l_, ff_l_));
        RC(upload_norm(loader, p + "attn_norm.weight", L.attn_norm));
        RC(upload_norm(loader, p + "ffn_norm.weight", L.ffn_norm));
    }
    CK(cudaDeviceSynchronize());
    return activate_streaming();
}

// After loading: streamed layers switch their weight pointers from the pinned host copy to
// their HBM slot (same offsets inside the layer block); the step copies host -> slot.
int DecodeEngine::activate_streaming() {
    if (streaming_active_) return VSL_OK;
    for (LayerPtrs& L : layers_) {
        if (L.slot < 0) continue;
        char* h = L.host;
        char* sl = slot_[L.slot];
        auto mv = [&](auto*& ptr) { ptr = reinterpret_cast<std::remove_reference_t<decltype(ptr)>>(sl + ((char*)ptr - h)); };
        mv(L.wqkv);
        mv(L.wo);
        mv(L.wgu);
        mv(L.wd);
        mv(L.attn_norm);
        mv(L.ffn_norm);
    }
    streaming_active_ = true;
    return VSL_OK;
}

int DecodeEngine::init_synthetic(uint64_t seed, double sigma) {
    const vsl_model_config& c = cfg_;
    const int r = opt_.tp_rank;
    const size_t d = c.d_model, hd = c.head_dim, qd = (size_t)c.n_heads * hd;
    const int dt = c.wdtype;
    cudaStream_t st = copy_stream_;
    // slice [row0, +nrows) x [col0, +ncols) of tensor tid ([*][src_cols]) into rows of ld bytes
    auto S = [&](void* dst, size_t ld, uint64_t tid, size_t row0, size_t nrows, size_t src_cols, size_t col0,
                 size_t ncols) {
        return is_quant(dt) ? synthq2d_impl(dst, dt, ld, seed, tid, row0, nrows, src_cols, col0, ncols, sigma, st)
                            : synth2d_impl(dst, dt, ld / es_, seed, tid, row0, nrows, src_cols, col0, ncols, sigma, st);
    };
    RC(S(tok_embd_, wrow(d), TID_TOK_EMBD, 0, c.vocab, d, 0, d));
    RC(S(lm_head_, wrow(d), TID_OUTPUT, (size_t)v_off_, v_l_, d, 0, d));
    std::vector<float> ones(d, 1.0f);
    CK(cudaMemcpy(out_norm_, ones.data(), d * 4, cudaMemcpyHostToDevice));
    for (int l = 0; l < c.n_layers; l++) {
        const LayerPtrs& L = layers_[l];
        char* qkv = (char*)L.wqkv;
        RC(S(qkv, wrow(d), tid_layer(l, K_Q), (size_t)r * nh_l_ * hd, (size_t)nh_l_ * hd, d, 0, d));
        qkv += (size_t)nh_l_ * hd * wrow(d);
        RC(S(qkv, wrow(d), tid_layer(l, K_K), (size_t)r * nkv_l_ * hd, (size_t)nkv_l_ * hd, d, 0, d));
        qkv += (size_t)nkv_l_ * hd * wrow(d);
        RC(S(qkv, wrow(d), tid_layer(l, K_V), (size_t)r * nkv_l_ * hd, (size_t)nkv_l_ * hd, d, 0, d));
        RC(S(L.wo, wrow((size_t)nh_l_ * hd), tid_layer(l, K_O), 0, d, qd, (size_t)r * nh_l_ * hd, (size_t)nh_l_ * hd));
        RC(S(L.wgu, 2 * wrow(d), tid_layer(l, K_GATE), (size_t)r * ff_l_, ff_l_, d, 0, d));
        RC(S((char*)L.wgu + wrow(d), 2 * wrow(d), tid_layer(l, K_UP), (size_t)r * ff_l_, ff_l_, d, 0, d));
        RC(S(L.wd, wrow(ff_l_), tid_layer(l, K_DOWN), 0, d, c.ffn, (size_t)r * ff_l_, ff_l_));
        CK(cudaMemcpyAsync(L.attn_norm, ones.data(), d * 4, cudaMemcpyDefault, st));
        CK(cudaMemcpyAsync(L.ffn_norm, ones.data(), d * 4, cudaMemcpyDefault, st));
        CK(cudaStreamSynchronize(st));  // `ones` is pageable; keep it alive across the copies
    }
    CK(cudaStreamSynchronize(st));
    return activate_streaming();
}

// ---------------------------------------------------------------------------------------
// state management
// ---------------------------------------------------------------------------------------

int DecodeEngine::reset() {
    RC(check_usable());
    CK(cudaSetDevice(opt_.device));
    RC(sync());
    const size_t mb = opt_.max_batch;
    CK(cudaMemsetAsync(pos_, 0, mb * 4, stream_));
    CK(cudaMemsetAsync(ids_, 0, mb * 4, stream_));
    CK(cudaMemsetAsync(step_, 0, 4, stream_));
    CK(cudaMemsetAsync(n_forced_, 0, 4, stream_));
    CK(cudaMemsetAsync(status_, 0, 4, stream_));
    if (tc_ws_) CK(cudaMemsetAsync(tc_ws_, 0, tc_ws_bytes_, stream_));  // arrival counters
    if (fdtc_ws_) CK(cudaMemsetAsync(fdtc_ws_, 0, fdtc_ws_bytes_, stream_));
    if (pf_tc_ws_) CK(cudaMemsetAsync(pf_tc_route_.ws, 0, pf_tc_route_.bytes, stream_));
    RC(sync());
    std::fill(pos_host_.begin(), pos_host_.end(), 0);
    steps_host_ = 0;
    return VSL_OK;
}

int DecodeEngine::fill_kv_synthetic(uint64_t seed, double sigma, int n_pos, int B) {
    if (n_pos < 0 || n_pos > opt_.max_seq || B <= 0 || B > opt_.max_batch)
        return set_error(VSL_ERR_INVALID, "fill_kv: n_pos %d / B %d out of range", n_pos, B);
    RC(check_usable());
    CK(cudaSetDevice(opt_.device));
    const vsl_model_config& c = cfg_;
    const size_t hd = c.head_dim;
    // element index of (b, global kv head G, t, e): ((b * n_kv + G) * n_pos + t) * hd + e;
    // a page holds [nkv_l][page][hd] so each (page, head) block is page*hd contiguous values
    for (int l = 0; l < c.n_layers; l++)
        for (int isv = 0; isv < 2; isv++) {
            char* cache = (char*)(isv ? layers_[l].v_cache : layers_[l].k_cache);
            for (int b = 0; b < B; b++)
                for (int g = 0; g < nkv_l_; g++) {
                    const int G = opt_.tp_rank * nkv_l_ + g;
                    for (int t0 = 0; t0 < n_pos; t0 += page_size_) {
                        const int n = std::min(page_size_, n_pos - t0);
                        const size_t page = (size_t)b * max_pages_ + t0 / page_size_;
                        const size_t off = ((page * nkv_l_ + g) * page_size_) * hd * dtype_bytes(kvdtype_);
                        const size_t start = (((size_t)b * c.n_kv_heads + G) * n_pos + t0) * hd;
                        RC(synth_impl(cache + off, kvdtype_, seed, tid_kv(l, isv), start, (size_t)n * hd, sigma,
                                      stream_));
                    }
                }
        }
    std::vector<int32_t> pos(opt_.max_batch, 0);
    CK(cudaMemcpy(pos.data(), pos_, pos.size() * 4, cudaMemcpyDeviceToHost));
    for (int b = 0; b < B; b++) pos[b] = n_pos;
    CK(cudaMemcpyAsync(pos_, pos.data(), pos.size() * 4, cudaMemcpyHostToDevice, stream_));
    RC(sync());
    for (int b = 0; b < B; b++) pos_host_[b] = n_pos;
    return VSL_OK;
}

int DecodeEngine::set_forced(const int32_t* ids, int n_steps, int B) {
    if (!ids || n_steps <= 0 || n_steps > log_cap_ || B <= 0 || B > opt_.max_batch)
        return set_error(VSL_ERR_INVALID, "set_forced: %d steps x %d sequences out of range", n_steps, B);
    RC(check_usable());
    CK(cudaSetDevice(opt_.device));
    RC(sync());
    CK(cudaMemcpy(forced_, ids, (size_t)n_steps * B * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(n_forced_, &n_steps, 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(ids_, ids, (size_t)B * 4, cudaMemcpyHostToDevice));
    CK(cudaMemset(step_, 0, 4));
    steps_host_ = 0;
    return VSL_OK;
}

// ---------------------------------------------------------------------------------------
// the decode step
// ---------------------------------------------------------------------------------------

int DecodeEngine::allreduce_sum(float* buf, int count) {
    if (!nccl_) return VSL_OK;
    if (p2p_ready_ && count <= p2p_x_.cap) return p2p_allreduce(p2p_x_, buf, count, 0, stream_);
    return nccl_result(ncclAllReduce(buf, buf, (size_t)count, ncclFloat, ncclSum, (ncclComm_t)nccl_, stream_),
                       "ncclAllReduce");
}

// The decoder layers for B activation rows held in `sb` (the decode step's buffers, or a
// prefill chunk's, where the rows are consecutive prompt positions of one sequence). Under
// tensor parallelism the row-parallel O and down projections leave partial residuals that the
// peer-memory all-reduce (or NCCL) sums on every rank.
int DecodeEngine::enqueue_layers(const StepBufs& sb, int B) {
    const vsl_model_config& c = cfg_;
    const int d = c.d_model, hd = c.head_dim;
    const int res_epi = opt_.tp_rank == 0 ? VSL_EPI_ADD : VSL_EPI_STORE;  // partial sums reduced into x
    cudaStream_t st = stream_;
    const TcRoute* tcr = sb.tc;
    // L2 prefetch hints: each kernel requests the head of the next projection's weights so
    // that the weight stream does not stall at kernel boundaries; the attention kernel
    // (which reads little from HBM) prefetches the output projection, up to half the L2
    // (a larger request would evict its own head before the projection reads it).
    const size_t qkv_b = (size_t)(nh_l_ + 2 * nkv_l_) * hd * wrow(d), wo_b = (size_t)d * wrow((size_t)nh_l_ * hd);
    const size_t wgu_b = 2 * (size_t)ff_l_ * wrow(d), wd_b = (size_t)d * wrow(ff_l_);
    const size_t head = 16ull << 20;
    auto H = [&](size_t bytes) { return std::min(bytes, head); };
    const size_t att_pf = opt_.attn_prefetch ? std::min(wo_b, (size_t)l2_bytes_ / 2) : 0;
    const bool streamed = residency_.streamed_layers > 0;
    if (streamed) {  // bring the copy stream into this step (and into a graph being captured)
        CK(cudaEventRecord(ev_fork_, st));
        CK(cudaStreamWaitEvent(copy_stream_, ev_fork_, 0));
    }
    const int R = (int)residency_.resident_layers;
    for (int l = 0; l < c.n_layers; l++) {
        const LayerPtrs& L = layers_[l];
        const bool last = l + 1 == c.n_layers;
        if (L.slot >= 0) {
            // host -> slot copy of this layer on the side stream, after the slot's previous
            // user (layer l - 2) has finished; it overlaps the compute of layer l - 1
            if (l - 2 >= R) CK(cudaStreamWaitEvent(copy_stream_, ev_done_[L.slot], 0));
            CK(cudaMemcpyAsync(slot_[L.slot], L.host, layer_bytes_, cudaMemcpyHostToDevice, copy_stream_));
            CK(cudaEventRecord(ev_copied_[L.slot], copy_stream_));
            CK(cudaStreamWaitEvent(st, ev_copied_[L.slot], 0));
        }
        RC(qkv_rope_append_status(c.wdtype, L.wqkv, nh_l_, nkv_l_, hd, d, sb.x, L.attn_norm, c.rms_eps, B, sb.pos,
                                  rope_cos_, rope_sin_, sb.q, L.k_cache, L.v_cache, kvdtype_, sb.pages, max_pages_,
                                  page_size_, status_, st, L.wo, H(wo_b), tcr));
        // a prompt chunk's attention writes the output projection's split activations straight
        // into the tensor-core workspace when that projection takes the tensor-core route
        const bool presplit = sb.shared_pages && pf_attn_tc_ && tc_route_taken(tcr, c.wdtype, d, nh_l_ * hd, B);
        if (sb.shared_pages && pf_attn_tc_)
            RC(flash_prefill_impl(sb.q, L.k_cache, L.v_cache, n_pages_, sb.pages, max_pages_, page_size_, sb.pos, B,
                                  nh_l_, nkv_l_, opt_.max_seq, presplit ? nullptr : sb.attn, status_, st, &sparse_,
                                  presplit ? tcr->ws : nullptr, c.wdtype == VSL_BF16 ? 1 : 0,
                                  (int)tc_split_rows(B)));
        else if (short_attn_ && !sb.shared_pages)
            RC(flash_decode_short_impl(sb.q, L.k_cache, L.v_cache, kvdtype_, sb.pages, max_pages_, page_size_, sb.pos,
                                       B, nh_l_, nkv_l_, hd, opt_.max_seq, sb.attn, st, L.wo, att_pf, &sparse_,
                                       status_));
        else if (sb.fdtc_ws)
            RC(flash_decode_tc_impl(sb.q, L.k_cache, L.v_cache, n_pages_, sb.pages, max_pages_, page_size_, sb.pos, B,
                                    nh_l_, nkv_l_, opt_.max_seq, sb.attn, sb.fdtc_ws, sb.fdtc_bytes, status_, st,
                                    &sparse_));
        else
            RC(flash_decode_impl(sb.q, L.k_cache, L.v_cache, kvdtype_, sb.pages, max_pages_, page_size_, sb.pos, B,
                                 nh_l_, nkv_l_, hd, opt_.max_seq, split_len_, sb.attn, sb.fd_ws, sb.fd_bytes, st, L.wo,
                                 att_pf, sb.shared_pages, &sparse_, fd_splits_, status_));
        RC(gemv_hint(c.wdtype, L.wo, d, nh_l_ * hd, sb.attn, B, sb.x, res_epi, nullptr, 0.0f, L.wgu, H(wgu_b), st, tcr,
                     presplit));
        RC(allreduce_sum(sb.x, B * d));
        // when both take the tensor-core route, gate/up writes the down projection's split
        // activations itself (no split launch before down)
        void* x2n = tcr && tcr->x2_next && tcr->x2_next_bytes >= 2 * tc_split_rows(B) * (size_t)ff_l_ * 2 &&
                            tc_route_taken(tcr, c.wdtype, 2 * ff_l_, d, B) && tc_route_taken(tcr, c.wdtype, d, ff_l_, B)
                        ? tcr->x2_next
                        : nullptr;
        RC(gemv_hint(c.wdtype, L.wgu, 2 * ff_l_, d, sb.x, B, sb.act, VSL_EPI_SWIGLU, L.ffn_norm, c.rms_eps, L.wd,
                     H(wd_b), st, tcr, false, nullptr, x2n));
        RC(gemv_hint(c.wdtype, L.wd, d, ff_l_, sb.act, B, sb.x, res_epi, nullptr, 0.0f,
                     last ? lm_head_ : layers_[l + 1].wqkv, last ? H((size_t)v_l_ * wrow(d)) : H(qkv_b), st, tcr,
                     x2n != nullptr, x2n));
        RC(allreduce_sum(sb.x, B * d));
        if (L.slot >= 0) CK(cudaEventRecord(ev_done_[L.slot], st));
    }
    return VSL_OK;
}

int DecodeEngine::enqueue_step(int B, float temperature, uint64_t seed) {
    const vsl_model_config& c = cfg_;
    const int d = c.d_model, hd = c.head_dim;
    cudaStream_t st = stream_;
    const size_t qkv_b = (size_t)(nh_l_ + 2 * nkv_l_) * hd * wrow(d);
    auto H = [&](size_t bytes) { return std::min(bytes, (size_t)16 << 20); };
    RC(embed_impl(c.wdtype, tok_embd_, c.vocab, d, ids_, B, x_, slots_, st));
    StepBufs sb{x_, q_, attn_, act_ffn_, pos_, page_table_, fd_ws_, fd_ws_bytes_, fdtc_ws_, fdtc_ws_bytes_,
                tc_ws_ ? &tc_route_ : nullptr, false};
    RC(enqueue_layers(sb, B));
    RC(lm_head_hint(c.wdtype, lm_head_, v_l_, d, x_, out_norm_, c.rms_eps, B, logits_, slots_, v_off_, temperature,
                    seed, step_, layers_[0].wqkv, H(qkv_b), st, sb.tc));
    if (p2p_ready_) {
        RC(p2p_allreduce(p2p_s_, slots_, B, 1, st));
    } else if (nccl_) {
        RC(nccl_result(ncclAllReduce(slots_, slots_, (size_t)B, ncclUint64, ncclMax, (ncclComm_t)nccl_, st),
                       "ncclAllReduce(argmax)"));
    }
    RC(finalize_impl(slots_, B, ids_, pos_, step_, forced_, n_forced_, log_, log_cap_, sampled_, opt_.max_seq, status_,
                     st));
    return VSL_OK;
}

int DecodeEngine::get_graph(int B, float temperature, uint64_t seed, cudaGraphExec_t* exec) {
    GraphKey key{B, temperature > 0.0f ? temperature : 0.0f, temperature > 0.0f ? seed : 0};
    auto it = graphs_.find(key);
    if (it != graphs_.end()) {
        *exec = it->second;
        return VSL_OK;
    }
    CK(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
    int rc = enqueue_step(B, temperature, seed);
    cudaGraph_t graph = nullptr;
    cudaError_t e = cudaStreamEndCapture(stream_, &graph);
    if (rc) {
        if (graph) cudaGraphDestroy(graph);
        return rc;
    }
    CK(e);
    cudaGraphExec_t g = nullptr;
    e = cudaGraphInstantiate(&g, graph, 0);
    cudaGraphDestroy(graph);
    CK(e);
    graphs_[key] = g;
    *exec = g;
    return VSL_OK;
}

int DecodeEngine::run(int n_steps, int B, float temperature, uint64_t seed) {
    if (n_steps < 0 || B <= 0 || B > opt_.max_batch)
        return set_error(VSL_ERR_INVALID, "run: %d steps for %d sequences (max batch %d)", n_steps, B, opt_.max_batch);
    for (int b = 0; b < B; b++)
        if (pos_host_[b] + n_steps > opt_.max_seq)
            return set_error(VSL_ERR_BOUNDS, "run: sequence %d at position %d cannot take %d more steps (max_seq %d)", b,
                             pos_host_[b], n_steps, opt_.max_seq);
    RC(check_usable());
    CK(cudaSetDevice(opt_.device));
    if (n_steps == 0) return VSL_OK;
    if (opt_.use_graph) {
        cudaGraphExec_t g;
        RC(get_graph(B, temperature, seed, &g));
        for (int i = 0; i < n_steps; i++) CK(cudaGraphLaunch(g, stream_));
    } else {
        for (int i = 0; i < n_steps; i++) RC(enqueue_step(B, temperature, seed));
    }
    for (int b = 0; b < B; b++) pos_host_[b] += n_steps;
    steps_host_ += n_steps;
    return VSL_OK;
}

// Buffers of the prompt pass, allocated on first use.
int DecodeEngine::alloc_prefill() {
    if (pf_mem_) return VSL_OK;
    const vsl_model_config& c = cfg_;
    const size_t P = PF_ROWS, d = c.d_model, qd = (size_t)nh_l_ * c.head_dim, A = 256;
    const size_t n_int = 2 * P + P * (size_t)max_pages_;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t o = off;
        off += align_up(bytes, A);
        return o;
    };
    const size_t o_ids = take(n_int * 4), o_x = take(P * d * 4), o_q = take(P * qd * 4), o_attn = take(P * qd * 4),
                 o_act = take(P * ff_l_ * 4), o_lg = take((size_t)v_l_ * 4), o_slot = take(16), o_next = take(4);
    CK(cudaMalloc(&pf_mem_, off));
    CK(cudaMemset(pf_mem_, 0, off));
    char* m = static_cast<char*>(pf_mem_);
    pf_ids_ = reinterpret_cast<int32_t*>(m + o_ids);
    pf_pos_ = pf_ids_ + P;
    pf_pages_ = pf_ids_ + 2 * P;
    pf_x_ = reinterpret_cast<float*>(m + o_x);
    pf_q_ = reinterpret_cast<float*>(m + o_q);
    pf_attn_ = reinterpret_cast<float*>(m + o_attn);
    pf_act_ = reinterpret_cast<float*>(m + o_act);
    pf_logits_ = reinterpret_cast<float*>(m + o_lg);
    pf_slot_ = reinterpret_cast<unsigned long long*>(m + o_slot);
    pf_next_ = reinterpret_cast<int32_t*>(m + o_next);
    CK(cudaMallocHost((void**)&pf_h_, n_int * 4 + 64));
    // prompt chunks: up to 128 rows of one sequence over the same pages, one query block of the
    // tensor-core prompt attention per head (fp16 KV, head_dim 128); otherwise the split-K kernel
    pf_attn_tc_ = flash_prefill_supported(kvdtype_, c.head_dim, nh_l_, nkv_l_, page_size_);
    if (!pf_attn_tc_) {
        pf_fd_bytes_ = flash_decode_workspace_bytes(PF_ROWS, nh_l_, nkv_l_, c.head_dim, fd_grid_splits());
        CK(cudaMalloc(&pf_fd_ws_, pf_fd_bytes_));
        CK(cudaMemset(pf_fd_ws_, 0, pf_fd_bytes_));
    }
    if (es_ == 2 && !is_quant(c.wdtype)) {
        const int n_max = std::max({(nh_l_ + 2 * nkv_l_) * c.head_dim, c.d_model, 2 * ff_l_, v_l_});
        const int k_max = std::max({c.d_model, nh_l_ * c.head_dim, ff_l_});
        const size_t bytes = tc_workspace_bytes(n_max, k_max, PF_ROWS) + 1024;
        CK(cudaMalloc(&pf_tc_ws_, bytes));
        CK(cudaMemset(pf_tc_ws_, 0, bytes));
        char* base = reinterpret_cast<char*>(((uintptr_t)pf_tc_ws_ + 1023) & ~(uintptr_t)1023);
        pf_tc_route_ = TcRoute{base, bytes - 1024, TC_MIN_BATCH, status_};
        const size_t x2n = 2 * tc_split_rows(PF_ROWS) * (size_t)ff_l_ * 2;
        CK(cudaMalloc(&pf_x2n_, x2n));
        pf_tc_route_.x2_next = pf_x2n_;
        pf_tc_route_.x2_next_bytes = x2n;
    }
    return VSL_OK;
}

int DecodeEngine::prefill(const int32_t* ids, int n, int seq, int32_t* next_id, float* out_logits, float temperature,
                          uint64_t seed) {
    if (!ids || n <= 0 || seq < 0 || seq >= opt_.max_batch)
        return set_error(VSL_ERR_INVALID, "prefill: %d ids for sequence %d", n, seq);
    if (pos_host_[seq] + n > opt_.max_seq)
        return set_error(VSL_ERR_BOUNDS, "prefill: sequence %d at %d + %d positions exceeds max_seq %d", seq,
                         pos_host_[seq], n, opt_.max_seq);
    RC(check_usable());
    const vsl_model_config& c = cfg_;
    CK(cudaSetDevice(opt_.device));
    RC(sync());
    RC(alloc_prefill());
    const int d = c.d_model, P = PF_ROWS;
    const int p0 = pos_host_[seq];
    for (int c0 = 0; c0 < n; c0 += P) {
        const int nc = std::min(P, n - c0);
        RC(sync());  // the staging buffer is reused
        for (int i = 0; i < nc; i++) {
            pf_h_[i] = ids[c0 + i];
            pf_h_[P + i] = p0 + c0 + i;
            memcpy(pf_h_ + 2 * P + (size_t)i * max_pages_, pt_host_.data() + (size_t)seq * max_pages_,
                   (size_t)max_pages_ * 4);
        }
        CK(cudaMemcpyAsync(pf_ids_, pf_h_, (2 * (size_t)P + (size_t)P * max_pages_) * 4, cudaMemcpyHostToDevice,
                           stream_));
        RC(embed_impl(c.wdtype, tok_embd_, c.vocab, d, pf_ids_, nc, pf_x_, nullptr, stream_));
        StepBufs sb{pf_x_, pf_q_, pf_attn_, pf_act_, pf_pos_, pf_pages_, pf_fd_ws_, pf_fd_bytes_, nullptr, 0,
                    pf_tc_ws_ ? &pf_tc_route_ : nullptr, true};
        RC(enqueue_layers(sb, nc));
        if (c0 + nc == n) {  // the last prompt token: logits, greedy next token
            CK(cudaMemsetAsync(pf_slot_, 0, 16, stream_));
            RC(lm_head_hint(c.wdtype, lm_head_, v_l_, d, pf_x_ + (size_t)(nc - 1) * d, out_norm_, c.rms_eps, 1,
                            pf_logits_, pf_slot_, v_off_, temperature, seed, step_, nullptr, 0, stream_));
            if (p2p_ready_) {
                RC(p2p_allreduce(p2p_s_, pf_slot_, 1, 1, stream_));
            } else if (nccl_) {
                RC(nccl_result(ncclAllReduce(pf_slot_, pf_slot_, 1, ncclUint64, ncclMax, (ncclComm_t)nccl_, stream_),
                               "ncclAllReduce(argmax)"));
            }
            RC(prefill_finish_impl(pf_slot_, ids_, pos_, seq, p0 + n, pf_next_, stream_));
        }
    }
    const float* lsrc = pf_logits_;
    if (out_logits && nccl_) {
        RC(nccl_result(ncclAllGather(pf_logits_, logits_full_, (size_t)v_l_, ncclFloat, (ncclComm_t)nccl_, stream_),
                       "ncclAllGather(logits)"));
        lsrc = logits_full_;  // [rank][v_l] = [vocab]
    }
    if (out_logits) CK(cudaMemcpyAsync(h_logits_, lsrc, (size_t)c.vocab * 4, cudaMemcpyDeviceToHost, stream_));
    CK(cudaMemcpyAsync(h_out_, pf_next_, 4, cudaMemcpyDeviceToHost, stream_));
    RC(sync());
    RC(check_device_status("prefill"));
    if (next_id) *next_id = h_out_[0];
    if (out_logits) memcpy(out_logits, h_logits_, (size_t)c.vocab * 4);
    pos_host_[seq] = p0 + n;
    return VSL_OK;
}

int DecodeEngine::reset_seq(int seq) {
    if (seq < 0 || seq >= opt_.max_batch) return set_error(VSL_ERR_INVALID, "reset_seq: sequence %d", seq);
    RC(check_usable());
    CK(cudaSetDevice(opt_.device));
    RC(sync());
    CK(cudaMemsetAsync(pos_ + seq, 0, 4, stream_));
    CK(cudaMemsetAsync(ids_ + seq, 0, 4, stream_));
    RC(sync());
    pos_host_[seq] = 0;
    return VSL_OK;
}

// Batched generation (the reference's generate_text_batch, VulkanSymbioteEngine.cpp:850-935,
// runs its prompts one after another): every sequence gets its own prompt pass into its own
// pages, then all of them decode together, one graph-launched step per token for the whole
// batch. A sequence that emits a stop id stops collecting ids; the batch ends when every
// sequence has stopped or produced max_new ids.
int DecodeEngine::generate_batch(const int32_t* prompts, const int* lens, int n_seq, int max_new, float temperature,
                                 uint64_t seed, const int32_t* stop_ids, int n_stop, int32_t* out_ids, int* n_out) {
    if (!prompts || !lens || !out_ids || !n_out || n_seq <= 0 || n_seq > opt_.max_batch || max_new < 0 ||
        (n_stop > 0 && !stop_ids))
        return set_error(VSL_ERR_INVALID, "generate_batch: %d sequences (max batch %d)", n_seq, opt_.max_batch);
    int longest = 0;
    for (int b = 0; b < n_seq; b++) {
        if (lens[b] <= 0) return set_error(VSL_ERR_INVALID, "generate_batch: empty prompt %d", b);
        longest = std::max(longest, lens[b]);
    }
    if (longest + max_new - 1 > opt_.max_seq)
        return set_error(VSL_ERR_BOUNDS, "generate_batch: prompt %d + %d new tokens exceed max_seq %d", longest,
                         max_new, opt_.max_seq);
    for (int b = 0; b < n_seq; b++) n_out[b] = 0;
    if (max_new == 0) return VSL_OK;
    auto is_stop = [&](int32_t t) {
        for (int s = 0; s < n_stop; s++)
            if (t == stop_ids[s]) return true;
        return false;
    };
    RC(reset());
    std::vector<char> done(n_seq, 0);
    int live = n_seq;
    size_t off = 0;
    for (int b = 0; b < n_seq; b++) {
        RC(prefill(prompts + off, lens[b], b, &out_ids[(size_t)b * max_new], nullptr, temperature, seed));
        off += lens[b];
        n_out[b] = 1;
        if (is_stop(out_ids[(size_t)b * max_new])) {
            done[b] = 1;
            live--;
        }
    }
    const int total = max_new - 1;
    const int chunk = n_stop > 0 ? 16 : std::max(total, 1);
    std::vector<int32_t> log;
    int steps = 0;
    while (steps < total && live > 0) {
        const int n = std::min(chunk, total - steps);
        RC(run(n, n_seq, temperature, seed));
        log.resize((size_t)(steps + n) * n_seq);
        RC(read_tokens(steps + n, n_seq, log.data()));
        RC(check_device_status("generate_batch"));
        for (int t = steps; t < steps + n; t++)
            for (int b = 0; b < n_seq; b++) {
                if (done[b]) continue;
                const int32_t id = log[(size_t)t * n_seq + b];
                out_ids[(size_t)b * max_new + 1 + t] = id;
                n_out[b] = 2 + t;
                if (is_stop(id)) {
                    done[b] = 1;
                    live--;
                }
            }
        steps += n;
    }
    return VSL_OK;
}

int DecodeEngine::step_host(const int32_t* ids, int B, int32_t* out_ids, float* out_logits) {
    if (!ids || B <= 0 || B > opt_.max_batch) return set_error(VSL_ERR_INVALID, "step_host: bad batch %d", B);
    for (int b = 0; b < B; b++)
        if (pos_host_[b] + 1 > opt_.max_seq)
            return set_error(VSL_ERR_BOUNDS, "step_host: sequence %d is at max_seq %d", b, opt_.max_seq);
    RC(check_usable());
    CK(cudaSetDevice(opt_.device));
    memcpy(h_ids_, ids, (size_t)B * 4);
    CK(cudaMemcpyAsync(ids_, h_ids_, (size_t)B * 4, cudaMemcpyHostToDevice, stream_));
    RC(run(1, B, 0.0f, 0));
    // the sampled ids and the status word behind them in one copy
    CK(cudaMemcpyAsync(h_out_, sampled_, ((size_t)opt_.max_batch + 1) * 4, cudaMemcpyDeviceToHost, stream_));
    const float* lsrc = logits_;
    if (out_logits && nccl_) {
        RC(nccl_result(ncclAllGather(logits_, logits_full_, (size_t)B * v_l_, ncclFloat, (ncclComm_t)nccl_, stream_),
                       "ncclAllGather(logits)"));
        lsrc = logits_full_;
    }
    if (out_logits)
        CK(cudaMemcpyAsync(h_logits_, lsrc, (size_t)B * cfg_.vocab * 4, cudaMemcpyDeviceToHost, stream_));
    RC(sync());
    if (const int st = h_out_[opt_.max_batch]) {
        if (st == VSL_ERR_TIMEOUT && opt_.tp_size > 1) {
            failed_ = true;
            failed_code_ = st;
        }
        return status_error(st, "step_host");
    }
    if (out_ids) memcpy(out_ids, h_out_, (size_t)B * 4);
    if (out_logits) {
        if (!nccl_) {
            memcpy(out_logits, h_logits_, (size_t)B * cfg_.vocab * 4);
        } else {  // gathered layout [rank][b][v_l] -> [b][vocab]
            const int tp = opt_.tp_size;
            for (int rk = 0; rk < tp; rk++)
                for (int b = 0; b < B; b++)
                    memcpy(out_logits + (size_t)b * cfg_.vocab + (size_t)rk * v_l_,
                           h_logits_ + ((size_t)rk * B + b) * v_l_, (size_t)v_l_ * 4);
        }
    }
    return VSL_OK;
}

int DecodeEngine::read_tokens(int n, int B, int32_t* out) {
    if (!out || n < 0 || n > log_cap_ || B <= 0 || B > opt_.max_batch)
        return set_error(VSL_ERR_INVALID, "read_tokens: %d x %d out of range", n, B);
    CK(cudaSetDevice(opt_.device));
    RC(sync());
    if (n) CK(cudaMemcpy(out, log_, (size_t)n * B * 4, cudaMemcpyDeviceToHost));
    return VSL_OK;
}

int DecodeEngine::positions(int B, int32_t* out) {
    if (!out || B <= 0 || B > opt_.max_batch) return set_error(VSL_ERR_INVALID, "positions: bad batch");
    CK(cudaSetDevice(opt_.device));
    RC(sync());
    CK(cudaMemcpy(out, pos_, (size_t)B * 4, cudaMemcpyDeviceToHost));
    return VSL_OK;
}

int DecodeEngine::device_status(int* status) {
    CK(cudaSetDevice(opt_.device));
    RC(sync());
    CK(cudaMemcpy(status, status_, 4, cudaMemcpyDeviceToHost));
    return VSL_OK;
}

int DecodeEngine::inject_status(int code) {
    CK(cudaSetDevice(opt_.device));
    RC(sync());
    CK(cudaMemcpy(status_, &code, 4, cudaMemcpyHostToDevice));
    return VSL_OK;
}

// generate (VulkanSymbioteEngine.cpp:678-765): clear the cache, feed the prompt, decode up to
// max_new tokens, stop after emitting a stop id (the reference stops on 0 or 2, :747-749).
int DecodeEngine::generate(const int32_t* prompt, int n_prompt, int max_new, float temperature, uint64_t seed,
                           const int32_t* stop_ids, int n_stop, int32_t* out_ids, int* n_out) {
    if (!prompt || n_prompt <= 0 || max_new < 0 || !out_ids || !n_out)
        return set_error(VSL_ERR_INVALID, "generate: empty prompt or null output");
    // the prompt takes positions 0..n_prompt-1 and every new token but the last takes one more
    // (the last one is sampled, never fed back): like generate_batch
    if (n_prompt + max_new - 1 > opt_.max_seq)
        return set_error(VSL_ERR_BOUNDS, "generate: prompt %d + %d new tokens exceed max_seq %d", n_prompt, max_new,
                         opt_.max_seq);
    RC(check_usable());
    *n_out = 0;
    if (max_new == 0) return VSL_OK;
    RC(reset());
    // the prompt in one prompt pass (chunks of 128 rows), which also samples the first new
    // token; then one graph-launched decode step per token, in chunks of 16 when stop ids can
    // end the loop early
    auto is_stop = [&](int32_t t) {
        for (int s = 0; s < n_stop; s++)
            if (t == stop_ids[s]) return true;
        return false;
    };
    RC(prefill(prompt, n_prompt, 0, &out_ids[0], nullptr, temperature, seed));
    *n_out = 1;
    if (is_stop(out_ids[0])) return VSL_OK;
    const int total = max_new - 1;
    const int chunk = n_stop > 0 ? 16 : std::max(total, 1);
    std::vector<int32_t> log;
    int done = 0;
    while (done < total) {
        const int n = std::min(chunk, total - done);
        RC(run(n, 1, temperature, seed));
        log.resize(done + n);
        RC(read_tokens(done + n, 1, log.data()));
        RC(check_device_status("generate"));
        for (int i = done; i < done + n; i++) {
            out_ids[1 + i] = log[i];
            *n_out = 2 + i;
            if (is_stop(log[i])) return VSL_OK;
        }
        done += n;
    }
    return VSL_OK;
}

int DecodeEngine::step_stats(int B, int* kernels, double* bytes) {
    if (B <= 0 || B > opt_.max_batch) return set_error(VSL_ERR_INVALID, "step_stats: bad batch");
    const vsl_model_config& c = cfg_;
    const double d = c.d_model, hd = c.head_dim;
    // weight bytes per step (quantized rows include their scales), norms, the embedding rows
    const double rd = (double)wrow(c.d_model);
    const double qkv = (double)(nh_l_ + 2 * nkv_l_) * hd * rd, wo = d * (double)wrow((size_t)nh_l_ * c.head_dim),
                 wgu = 2.0 * ff_l_ * rd, wd = d * (double)wrow(ff_l_);
    double w = c.n_layers * (qkv + wo + wgu + wd + 2 * d * 4) + (double)v_l_ * rd + d * 4 + B * rd;
    double kv = 0;
    const double kv_es = (double)dtype_bytes(kvdtype_);
    for (int b = 0; b < B; b++) kv += 2.0 * c.n_layers * nkv_l_ * hd * kv_es * (pos_host_[b] + 1);
    if (kernels) {
        // GEMV launches cover at most 4 activation rows (fewer when K is large), see gemv.cu;
        // batches on the tensor-core route take two launches per projection (split + GEMM)
        const bool tc = tc_ws_ && B >= TC_MIN_BATCH && B <= TC_MAX_BATCH;
        auto chunks = [&](int K) {
            if (tc) return 2;
            int cmax = (int)std::min<size_t>(4, (200 * 1024) / ((size_t)K * 4));
            return (B + cmax - 1) / cmax;
        };
        *kernels = 1 /*embed*/ +
                   c.n_layers * (chunks(c.d_model) /*qkv*/ + 1 /*attention*/ + chunks(nh_l_ * c.head_dim) /*o*/ +
                                 chunks(c.d_model) /*gate-up*/ + chunks(ff_l_) /*down*/) +
                   chunks(c.d_model) /*lm_head*/ + 1 /*finalize*/;
        // tensor parallel over peer memory: the residual all-reduces and the argmax exchange
        // (NCCL's kernels are not counted)
        if (p2p_ready_) *kernels += 1 + 2 * c.n_layers;
    }
    if (bytes) *bytes = w + kv;
    return VSL_OK;
}

int DecodeEngine::device_of_layer(int) const { return opt_.device; }


}  // namespace vsl
