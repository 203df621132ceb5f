// Decode engine with the reference's VulkanSymbioteEngine API
// (vk_symbiote/include/vk_symbiote/VulkanSymbioteEngine.h:72-118,193-194), running the
// B200 kernels of libvsl.so. The constructor taking Vulkan handles (:77-82) has no
// counterpart without Vulkan; DeviceOptions takes its place (device, tensor-parallel rank
// and size, NCCL id, KV capacity). Constructors throw std::runtime_error on failure, like
// the reference (VulkanSymbioteEngine.cpp:426-434).
#pragma once

#include <cstdint>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "Common.h"
#include "ConfigManager.h"
#include "GGUFLoader.h"
#include "NomadPack.h"

struct vsl_engine;

namespace vk_symbiote {

class Tokenizer;

struct BenchmarkResult {
    uint32_t warmup_tokens = 0;
    uint32_t benchmark_tokens = 0;
    uint32_t iterations = 0;
    double avg_tokens_per_sec = 0.0;
    double min_tokens_per_sec = 0.0;
    double max_tokens_per_sec = 0.0;
    double std_dev_tokens_per_sec = 0.0;
    double avg_latency_ms = 0.0;
    double peak_vram_gb = 0.0;
    double cache_hit_rate = 0.0;
    double cache_size_mb = 0.0;
    std::unordered_map<std::string, double> power_mode_results;
    double memory_pressure_result = 0.0;
};

struct VSL_CPP_API BenchmarkStats {
    double avg_tokens_per_sec = 0.0;
    double min_tokens_per_sec = 0.0;
    double max_tokens_per_sec = 0.0;
    double std_dev_tokens_per_sec = 0.0;
    double avg_latency_ms = 0.0;
    double peak_vram_gb = 0.0;
    double avg_vram_usage_gb = 0.0;
    double fragmentation_ratio = 0.0;
    double cache_hit_rate = 0.0;
    uint64_t total_evictions = 0;
    double eviction_rate = 0.0;
    void print() const;
};

struct DeviceOptions {
    int device = -1;               // -1: ConfigManager parallel().device
    int tp_rank = 0;
    int tp_size = 0;               // 0: ConfigManager parallel().tp_size
    std::vector<uint8_t> nccl_id;  // 128 bytes from vsl_nccl_unique_id when tp_size > 1
    uint32_t max_batch = 1;
    uint32_t max_seq = 0;          // 0: min(llama.context_length, 4096)
    double vram_budget_gb = -1.0;  // < 0: ConfigManager budget if explicitly set, else no cap
    bool use_graph = true;
    // Long-context sparse attention with the model config's window (use_sparse_attention,
    // sparse_window_size, sparse_global_tokens, sparse_block_size; Common.h): the reference
    // switches to it above 8192 positions (VulkanSymbioteEngine.cpp:788). Off by default here:
    // dense attention at every length, as a standard Llama.
    bool sparse_attention = false;
    uint32_t sparse_min_len = 8192;
};

class VSL_CPP_API VulkanSymbioteEngine {
public:
    explicit VulkanSymbioteEngine(const Path& model_path);
    VulkanSymbioteEngine(const Path& model_path, const DeviceOptions& options);
    ~VulkanSymbioteEngine();
    VulkanSymbioteEngine(const VulkanSymbioteEngine&) = delete;
    VulkanSymbioteEngine& operator=(const VulkanSymbioteEngine&) = delete;

    // generate (VulkanSymbioteEngine.cpp:678-765): returns prompt + decoded tokens; stops
    // after emitting id 0 or 2 (with a byte-level BPE vocabulary, where those are ordinary
    // tokens: after its end-of-text id). Any temperature gives the reference's result, the
    // argmax (its top_k_sampling hands back the most probable token first, :1548-1552).
    std::string generate(const std::string& prompt, uint32_t max_tokens = 256, float temperature = 0.7f);

    // Token-id generation: temperature > 0 samples with the seeded Gumbel-max sampler;
    // stop_ids end the generation after the first one emitted.
    std::vector<uint32_t> generate_ids(const std::vector<uint32_t>& prompt, uint32_t max_new_tokens,
                                       float temperature = 0.0f, const std::vector<uint32_t>& stop_ids = {},
                                       uint64_t seed = 0);

    std::vector<uint32_t> encode(const std::string& text);
    std::string decode(const std::vector<uint32_t>& tokens);

    const ModelConfig& config() const noexcept { return config_; }
    ModelConfig& config() noexcept { return config_; }

    BenchmarkResult run_benchmark(uint32_t warmup_tokens = 10, uint32_t benchmark_tokens = 100,
                                  uint32_t iterations = 3);
    BenchmarkStats run_benchmark_detailed(uint32_t warmup_tokens, uint32_t benchmark_tokens, uint32_t iterations);

    // generate_text_batch (VulkanSymbioteEngine.cpp:850-935): one result per prompt.
    std::vector<std::string> generate_text_batch(const std::vector<std::string>& prompts,
                                                 uint32_t max_tokens_per_prompt = 256, float temperature = 0.7f);

    MemoryPoolStats get_vram_stats();
    double get_peak_vram_usage();
    void clear_kv_cache();
    size_t get_kv_cache_memory_usage() const;

    const PerformanceMetrics& get_performance_metrics() const { return performance_metrics_; }
    void reset_performance_metrics() { performance_metrics_.reset(); }

    // The C ABI engine underneath (include/vsl.h), for callers mixing both layers.
    vsl_engine* native_handle() noexcept { return engine_; }

private:
    void open(const Path& model_path, const DeviceOptions& options);

    vsl_engine* engine_ = nullptr;
    std::unique_ptr<Tokenizer> tokenizer_;
    // ids that end generate() / generate_text_batch(): 0 and 2 as in the reference, or the
    // end-of-text id of a byte-level BPE vocabulary (where 0 and 2 are ordinary tokens)
    std::vector<uint32_t> text_stop_ids() const;
    ModelConfig config_;
    PerformanceMetrics performance_metrics_;
    uint32_t max_seq_ = 0;
    uint32_t max_batch_ = 1;
    double peak_vram_gb_ = 0.0;
};

}  // namespace vk_symbiote
