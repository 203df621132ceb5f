// VulkanSymbioteEngine and Tokenizer: the reference's C++ class API
// (vk_symbiote/include/vk_symbiote/VulkanSymbioteEngine.h, Tokenizer.h) on top of the C ABI.
#include "../../../include/vk_symbiote/VulkanSymbioteEngine.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <iostream>
#include <sstream>
#include <stdexcept>

#include "../../../include/vk_symbiote/Tokenizer.h"
#include "../../../include/vsl.h"

namespace vk_symbiote {

// ---------------------------------------------------------------------------------------
// VulkanSymbioteEngine
// ---------------------------------------------------------------------------------------
static void throw_vsl(const char* what) {
    throw std::runtime_error(std::string(what) + ": " + vsl_last_error_string());
}

VulkanSymbioteEngine::VulkanSymbioteEngine(const Path& model_path) { open(model_path, DeviceOptions{}); }

VulkanSymbioteEngine::VulkanSymbioteEngine(const Path& model_path, const DeviceOptions& options) {
    open(model_path, options);
}

VulkanSymbioteEngine::~VulkanSymbioteEngine() {
    if (engine_) vsl_engine_destroy(engine_);
}

void VulkanSymbioteEngine::open(const Path& model_path, const DeviceOptions& opt) {
    ConfigManager& cm = ConfigManager::instance();
    if (!cm.performance().enable_gpu)
        throw std::runtime_error(
            "VulkanSymbioteEngine: the GPU is disabled (--disable-gpu / enable_gpu = false) and this build has no "
            "CPU decode path");
    GGUFLoader loader(model_path);
    auto st = loader.load();
    if (!st) throw std::runtime_error("VulkanSymbioteEngine: cannot load GGUF " + model_path.string());
    config_ = loader.get_model_config();
    vsl_engine_options o;
    vsl_engine_default_options(&o);
    o.device = opt.device >= 0 ? opt.device : (int)cm.parallel().device;
    o.tp_size = opt.tp_size > 0 ? opt.tp_size : (int)std::max<uint32_t>(1, cm.parallel().tp_size);
    o.tp_rank = opt.tp_rank;
    if (o.tp_size > 1) {
        if (opt.nccl_id.size() != 128)
            throw std::runtime_error("VulkanSymbioteEngine: tensor parallelism needs the 128-byte NCCL unique id");
        o.nccl_id = opt.nccl_id.data();
    }
    o.max_batch = (int)std::max<uint32_t>(1, opt.max_batch);
    max_batch_ = (uint32_t)o.max_batch;
    max_seq_ = opt.max_seq ? opt.max_seq : std::min<uint32_t>(std::max<uint32_t>(config_.max_position_embeddings, 64), 4096);
    o.max_seq = (int)max_seq_;
    o.vram_budget_gb =
        opt.vram_budget_gb >= 0 ? opt.vram_budget_gb : (cm.vram_budget_explicit() ? cm.memory().vram_budget_gb : 0.0);
    o.use_graph = opt.use_graph ? 1 : 0;
    if (opt.sparse_attention && config_.use_sparse_attention) {
        o.sparse_min_len = (int)opt.sparse_min_len;
        o.sparse_window = (int)config_.sparse_window_size;
        o.sparse_global = (int)config_.sparse_global_tokens;
        o.sparse_block = (int)config_.sparse_block_size;
    }
    if (vsl_engine_create_gguf(model_path.c_str(), &o, &engine_) != VSL_OK) throw_vsl("VulkanSymbioteEngine");
    tokenizer_ = Tokenizer::from_gguf(model_path);
    peak_vram_gb_ = get_peak_vram_usage();
}

std::vector<uint32_t> VulkanSymbioteEngine::encode(const std::string& text) { return tokenizer_->encode(text); }

std::string VulkanSymbioteEngine::decode(const std::vector<uint32_t>& tokens) { return tokenizer_->decode(tokens); }

std::vector<uint32_t> VulkanSymbioteEngine::text_stop_ids() const {
    if (tokenizer_ && tokenizer_->is_byte_bpe()) return {tokenizer_->eos_id()};
    return {0u, 2u};
}

std::vector<uint32_t> VulkanSymbioteEngine::generate_ids(const std::vector<uint32_t>& prompt, uint32_t max_new_tokens,
                                                         float temperature, const std::vector<uint32_t>& stop_ids,
                                                         uint64_t seed) {
    if (prompt.empty() || max_new_tokens == 0) return {};
    // the last new token is sampled, never fed back: it takes no KV position
    if (prompt.size() + max_new_tokens - 1 > max_seq_)
        throw std::runtime_error("generate_ids: prompt + new tokens exceed the engine's max_seq");
    std::vector<int32_t> p(prompt.begin(), prompt.end()), stops(stop_ids.begin(), stop_ids.end());
    std::vector<int32_t> out(max_new_tokens);
    int n = 0;
    const uint64_t t0 = get_current_time_ns();
    if (vsl_engine_generate(engine_, p.data(), (int)p.size(), (int)max_new_tokens, temperature, seed,
                            stops.empty() ? nullptr : stops.data(), (int)stops.size(), out.data(), &n) != VSL_OK)
        throw_vsl("generate_ids");
    const uint64_t dt = get_current_time_ns() - t0;
    int kernels = 0;
    double bytes = 0;
    vsl_engine_step_stats(engine_, 1, &kernels, &bytes);
    performance_metrics_.update(dt, (uint32_t)n);
    const double steps = (double)prompt.size() + n - 1;
    if (dt > 0) performance_metrics_.memory_bandwidth_gbps = (float)(bytes * steps / (dt * 1e-9) / 1e9);
    return std::vector<uint32_t>(out.begin(), out.begin() + n);
}

std::string VulkanSymbioteEngine::generate(const std::string& prompt, uint32_t max_tokens, float /*temperature*/) {
    std::vector<uint32_t> ids = encode(prompt);
    if (ids.size() >= max_seq_) ids.resize(max_seq_ - 1);
    const uint32_t room = (uint32_t)(max_seq_ - ids.size());
    const uint32_t n = std::min(max_tokens, room);
    std::string result = prompt;
    if (n == 0) return result;
    // greedy for every temperature, and stop after emitting 0 or 2 (VulkanSymbioteEngine.cpp:747-749),
    // the unknown and end-of-sequence ids of the SentencePiece vocabularies the reference has in
    // view; in a byte-level BPE vocabulary those ids are ordinary tokens ("!" and "#"), so there
    // the vocabulary's own end-of-text id stops generation instead
    const std::vector<uint32_t> out = generate_ids(ids, n, 0.0f, text_stop_ids());
    result += tokenizer_->decode_continuation(ids, out);
    return result;
}

std::vector<std::string> VulkanSymbioteEngine::generate_text_batch(const std::vector<std::string>& prompts,
                                                                   uint32_t max_tokens_per_prompt, float temperature) {
    // up to max_batch prompts decode together (one prompt pass each, then batched steps);
    // greedy and stop ids 0/2 as in generate()
    std::vector<std::string> out;
    out.reserve(prompts.size());
    for (size_t p0 = 0; p0 < prompts.size(); p0 += max_batch_) {
        const size_t nb = std::min<size_t>(max_batch_, prompts.size() - p0);
        std::vector<int32_t> flat;
        std::vector<int> lens(nb);
        std::vector<std::vector<uint32_t>> prompt_ids(nb);
        uint32_t longest = 0;
        for (size_t b = 0; b < nb; b++) {
            std::vector<uint32_t>& ids = prompt_ids[b];
            ids = encode(prompts[p0 + b]);
            if (ids.size() >= max_seq_) ids.resize(max_seq_ - 1);
            lens[b] = (int)ids.size();
            longest = std::max<uint32_t>(longest, (uint32_t)ids.size());
            flat.insert(flat.end(), ids.begin(), ids.end());
        }
        const uint32_t n = std::min<uint32_t>(max_tokens_per_prompt, max_seq_ - longest);
        std::vector<int32_t> ids_out(nb * std::max<uint32_t>(n, 1));
        std::vector<int> n_out(nb, 0);
        const std::vector<uint32_t> sv = text_stop_ids();
        const std::vector<int32_t> stops(sv.begin(), sv.end());
        const uint64_t t0 = get_current_time_ns();
        if (n > 0 && vsl_engine_generate_batch(engine_, flat.data(), lens.data(), (int)nb, (int)n, 0.0f, 0, stops.data(),
                                               (int)stops.size(), ids_out.data(), n_out.data()) != VSL_OK)
            throw_vsl("generate_text_batch");
        uint32_t produced = 0;
        for (size_t b = 0; b < nb; b++) {
            std::string r = prompts[p0 + b];
            const std::vector<uint32_t> gen(ids_out.begin() + b * n, ids_out.begin() + b * n + n_out[b]);
            r += tokenizer_->decode_continuation(prompt_ids[b], gen);
            produced += (uint32_t)n_out[b];
            out.push_back(std::move(r));
        }
        performance_metrics_.update(get_current_time_ns() - t0, produced);
    }
    (void)temperature;
    return out;
}

BenchmarkStats VulkanSymbioteEngine::run_benchmark_detailed(uint32_t warmup_tokens, uint32_t benchmark_tokens,
                                                           uint32_t iterations) {
    // run_benchmark_detailed (VulkanSymbioteEngine.cpp:942-1063): a fixed prompt, warm-up,
    // then `iterations` timed runs of `benchmark_tokens` decode steps.
    BenchmarkStats st;
    std::vector<uint32_t> prompt = encode("The quick brown fox jumps over the lazy dog");
    const size_t need = prompt.size() + warmup_tokens + (size_t)benchmark_tokens * iterations;
    if (need > max_seq_) throw std::runtime_error("run_benchmark: prompt + tokens exceed the engine's max_seq");
    if (vsl_engine_reset(engine_) != VSL_OK) throw_vsl("run_benchmark");
    std::vector<int32_t> p(prompt.begin(), prompt.end());
    if (vsl_engine_set_forced(engine_, p.data(), (int)p.size(), 1) != VSL_OK) throw_vsl("run_benchmark");
    if (vsl_engine_run(engine_, (int)p.size() + (int)warmup_tokens, 1, 0.0f, 0) != VSL_OK) throw_vsl("run_benchmark");
    cudaStream_t s = (cudaStream_t)vsl_engine_stream(engine_);
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    std::vector<double> rates, lat;
    for (uint32_t it = 0; it < iterations && benchmark_tokens > 0; it++) {
        cudaEventRecord(e0, s);
        if (vsl_engine_run(engine_, (int)benchmark_tokens, 1, 0.0f, 0) != VSL_OK) throw_vsl("run_benchmark");
        cudaEventRecord(e1, s);
        cudaEventSynchronize(e1);
        float ms = 0;
        cudaEventElapsedTime(&ms, e0, e1);
        rates.push_back(benchmark_tokens / (ms * 1e-3));
        lat.push_back(ms / benchmark_tokens);
    }
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    if (!rates.empty()) {
        double sum = 0, sq = 0, lsum = 0;
        for (double r : rates) sum += r;
        for (double l : lat) lsum += l;
        st.avg_tokens_per_sec = sum / rates.size();
        for (double r : rates) sq += (r - st.avg_tokens_per_sec) * (r - st.avg_tokens_per_sec);
        st.std_dev_tokens_per_sec = std::sqrt(sq / rates.size());
        st.min_tokens_per_sec = *std::min_element(rates.begin(), rates.end());
        st.max_tokens_per_sec = *std::max_element(rates.begin(), rates.end());
        st.avg_latency_ms = lsum / lat.size();
    }
    st.peak_vram_gb = get_peak_vram_usage();
    st.avg_vram_usage_gb = st.peak_vram_gb;
    return st;
}

BenchmarkResult VulkanSymbioteEngine::run_benchmark(uint32_t warmup_tokens, uint32_t benchmark_tokens,
                                                    uint32_t iterations) {
    BenchmarkStats s = run_benchmark_detailed(warmup_tokens, benchmark_tokens, iterations);
    BenchmarkResult r;
    r.warmup_tokens = warmup_tokens;
    r.benchmark_tokens = benchmark_tokens;
    r.iterations = iterations;
    r.avg_tokens_per_sec = s.avg_tokens_per_sec;
    r.min_tokens_per_sec = s.min_tokens_per_sec;
    r.max_tokens_per_sec = s.max_tokens_per_sec;
    r.std_dev_tokens_per_sec = s.std_dev_tokens_per_sec;
    r.avg_latency_ms = s.avg_latency_ms;
    r.peak_vram_gb = s.peak_vram_gb;
    return r;
}

void BenchmarkStats::print() const {
    std::cout << "tok/s avg " << avg_tokens_per_sec << " (min " << min_tokens_per_sec << ", max " << max_tokens_per_sec
              << ", std " << std_dev_tokens_per_sec << "), latency " << avg_latency_ms << " ms, peak HBM "
              << peak_vram_gb << " GB" << std::endl;
}

MemoryPoolStats VulkanSymbioteEngine::get_vram_stats() {
    MemoryPoolStats m;
    size_t free_b = 0, total_b = 0, w = 0, kv = 0, other = 0;
    vsl_engine_memory_stats(engine_, &w, &kv, &other);
    if (cudaMemGetInfo(&free_b, &total_b) == cudaSuccess) {
        m.total_size = total_b;
        m.free_size = free_b;
    }
    m.used_size = w + kv + other;
    m.allocation_count = 4;  // weight arena, KV cache, activations, attention workspace
    m.fragmentation_ratio = 0.0f;
    return m;
}

double VulkanSymbioteEngine::get_peak_vram_usage() {
    size_t w = 0, kv = 0, other = 0;
    vsl_engine_memory_stats(engine_, &w, &kv, &other);
    peak_vram_gb_ = std::max(peak_vram_gb_, (w + kv + other) / 1e9);
    return peak_vram_gb_;
}

void VulkanSymbioteEngine::clear_kv_cache() {
    if (vsl_engine_reset(engine_) != VSL_OK) throw_vsl("clear_kv_cache");
}

size_t VulkanSymbioteEngine::get_kv_cache_memory_usage() const {
    size_t kv = 0;
    vsl_engine_memory_stats(engine_, nullptr, &kv, nullptr);
    return kv;
}

}  // namespace vk_symbiote
