// Process-wide configuration with the reference's ConfigManager API
// (vk_symbiote/include/vk_symbiote/ConfigManager.h:13-270): INI/TOML-subset files, command
// line flags, typed section structs and generic getters.
//
// Differences, each deliberate:
//   - numeric budgets accept integer or float values (the reference reads only integers,
//     ConfigManager.cpp:277-326, and parses --vram-gb with stoull);
//   - --disable-gpu is parsed (documented by the reference but never parsed,
//     ConfigManager.cpp:669-689); this build has no CPU decode path, so an engine refuses
//     to start when the GPU is disabled;
//   - --tp N sets the tensor-parallel world size (ParallelConfig);
//   - vram_budget_explicit() tells whether a budget was set by a file, a flag or
//     set_memory(); only then does an engine cap its HBM use (the reference hard-codes
//     4 GiB, VulkanSymbioteEngine.cpp:1130).
#pragma once

#include <cstdint>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <variant>

#include "Common.h"

namespace vk_symbiote {

enum class LogLevel { DEBUG = 0, INFO = 1, WARNING = 2, ERROR = 3, FATAL = 4 };

struct MemoryConfig {
    float vram_budget_gb = 4.0f;
    float ram_budget_gb = 16.0f;
    // Parsed and saved for compatibility; the engine does not use it. Layers over the budget
    // stream through two HBM slots (the copy of layer l + 1 overlaps the compute of layer l),
    // which already keeps the host link busy (0.999 of the measured pinned copy bandwidth for the
    // 70B model under a 64 GB cap); each deeper slot would take a layer's HBM from the resident
    // set and add that layer to the bytes streamed per token.
    uint32 prefetch_lookahead = 3;
    float eviction_aggression = 0.7f;
    bool enable_compression = true;
    std::string compression_algorithm = "hybrid";
    uint32 max_packs_in_memory = 1000;
    bool enable_defrag = true;
    uint32 defrag_interval_ms = 5000;
};

struct PerformanceConfig {
    bool enable_gpu = true;
    bool enable_profiling = false;
    uint32 workgroup_size_x = 256;
    uint32 workgroup_size_y = 1;
    uint32 workgroup_size_z = 1;
    bool use_subgroup_ops = true;
    uint32 subgroup_size = 32;
    // Parsed and saved for compatibility; the engine does not use it: weights keep their stored
    // type (fp16 / bf16 / fp32 / block-quantized) and every dot product accumulates in fp32.
    bool use_fp16_math = true;
    float scale_factor = 1.0f;
    uint32 thread_pool_size = 0;
};

struct PowerConfig {
    bool enable_power_management = true;
    bool enable_power_saver = false;
    bool auto_detect_battery = true;
    uint32 power_profile = 1;
    float battery_threshold_low = 0.25f;
    float battery_threshold_critical = 0.10f;
    bool throttle_on_thermal = true;
    bool reduce_workgroup_on_battery = true;
    uint32 min_workgroup_size_battery = 64;
    uint32 prefetch_reduction_factor = 2;
    bool disable_profiling_on_battery = true;
    uint32 battery_threshold_percent = 30;
    uint32 max_workgroup_size_battery = 64;
    uint32 prefetch_lookahead_battery = 1;
};

struct BenchmarkConfig {
    bool enable_benchmark_mode = false;
    uint32 warmup_tokens = 10;
    uint32 benchmark_tokens = 100;
    uint32 iterations = 3;
    bool output_json = true;
    std::string output_file = "benchmark_results.json";
    bool test_power_modes = false;
    bool test_memory_pressure = false;
    bool detailed_layer_stats = false;
};

struct LoggingConfig {
    LogLevel log_level = LogLevel::INFO;
    bool log_to_file = false;
    std::string log_file_path = "vk_symbiote.log";
    bool log_performance = false;
    bool log_memory_usage = false;
    uint32 max_log_file_size_mb = 100;
    bool log_to_console = true;
};

struct CodecConfig {
    std::string codec = "hybrid";
    uint32 compression_level = 5;
    bool enable_blosc2 = true;
    std::string blosc2_compressor = "lz4";
    bool blosc2_shuffle = true;
    bool enable_zfp = false;
    uint32 zfp_precision = 16;
    float zfp_rate = 0.0f;
    bool enable_hybrid = true;
    std::string hybrid_mode = "auto";
    uint32 decompression_threads = 0;
    bool enable_compression = true;
    std::string algorithm = "hybrid";
    float hybrid_compression_ratio = 0.5f;
};

struct BatchConfig {
    bool enable_batching = true;
    uint32 max_batch_size = 8;
    bool dynamic_batch_size = true;
    uint32 batch_timeout_ms = 100;
    bool prefetch_for_batch = true;
    bool share_kv_cache = false;
    uint32 max_sequence_length = 8192;
};

struct VitalityConfig {
    bool enabled = true;
    float learning_rate = 0.001f;
    float momentum = 0.9f;
    bool use_adam = false;
    std::string model_path = "vitality_model.toml";
};

struct ShaderConfig {
    std::string cache_dir = ".shader_cache";
    bool enable_cache = true;
    bool use_cooperative_matrix = true;
    uint32 coop_matrix_m = 16;
    uint32 coop_matrix_n = 16;
    uint32 coop_matrix_k = 16;
    bool auto_tune = true;
    std::string tuning_file = "shader_tuning.conf";
};

// Tensor parallelism of the B200 engine (no counterpart in the reference).
struct ParallelConfig {
    uint32 tp_size = 1;
    uint32 device = 0;
};

class VSL_CPP_API ConfigManager {
public:
    using Value = std::variant<int64_t, double, bool, std::string>;

    static ConfigManager& instance();

    bool load_from_file(const Path& config_path);
    bool save_to_file(const Path& config_path);
    bool load_from_toml(const Path& config_path);
    bool save_to_toml(const Path& config_path);
    void load_from_args(int argc, char* argv[]);
    void set_defaults();

    const MemoryConfig& memory() const { return memory_config_; }
    void set_memory(const MemoryConfig& config) {
        memory_config_ = config;
        vram_budget_explicit_ = true;
    }
    const PerformanceConfig& performance() const { return perf_config_; }
    void set_performance(const PerformanceConfig& config) { perf_config_ = config; }
    const LoggingConfig& logging() const { return logging_config_; }
    void set_logging(const LoggingConfig& config) { logging_config_ = config; }
    const PowerConfig& power() const { return power_config_; }
    void set_power(const PowerConfig& config) { power_config_ = config; }
    const BenchmarkConfig& benchmark() const { return benchmark_config_; }
    void set_benchmark(const BenchmarkConfig& config) { benchmark_config_ = config; }
    const CodecConfig& codec() const { return codec_config_; }
    void set_codec(const CodecConfig& config) { codec_config_ = config; }
    const BatchConfig& batch() const { return batch_config_; }
    void set_batch(const BatchConfig& config) { batch_config_ = config; }
    const VitalityConfig& vitality() const { return vitality_config_; }
    void set_vitality(const VitalityConfig& config) { vitality_config_ = config; }
    const ShaderConfig& shader() const { return shader_config_; }
    void set_shader(const ShaderConfig& config) { shader_config_ = config; }
    const ParallelConfig& parallel() const { return parallel_config_; }
    void set_parallel(const ParallelConfig& config) { parallel_config_ = config; }

    const std::string& model_path() const { return model_path_; }
    void set_model_path(const std::string& path) { model_path_ = path; }
    const std::string& model_type() const { return model_type_; }
    void set_model_type(const std::string& type) { model_type_ = type; }

    int get_int(const std::string& section, const std::string& key, int default_value) const;
    float get_float(const std::string& section, const std::string& key, float default_value) const;
    bool get_bool(const std::string& section, const std::string& key, bool default_value) const;
    std::string get_string(const std::string& section, const std::string& key, const std::string& default_value) const;

    // Reference bounds (ConfigManager.cpp:773-787): VRAM 1-64 GB, RAM 1-128 GB.
    bool validate_config() const;
    void print_config() const;
    std::string get_current_timestamp() const;

    bool vram_budget_explicit() const { return vram_budget_explicit_; }

    struct PrivateTag {};
    explicit ConfigManager(PrivateTag) {}

private:
    void apply_document();

    MemoryConfig memory_config_;
    PerformanceConfig perf_config_;
    LoggingConfig logging_config_;
    PowerConfig power_config_;
    BenchmarkConfig benchmark_config_;
    CodecConfig codec_config_;
    BatchConfig batch_config_;
    VitalityConfig vitality_config_;
    ShaderConfig shader_config_;
    ParallelConfig parallel_config_;
    std::string model_path_;
    std::string model_type_;
    bool vram_budget_explicit_ = false;
    std::unordered_map<std::string, std::unordered_map<std::string, Value>> toml_data_;

    static std::unique_ptr<ConfigManager> instance_;
    static std::mutex instance_mutex_;
};

}  // namespace vk_symbiote
