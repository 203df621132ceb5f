// ConfigManager: INI/TOML-subset parser and command-line flags with the reference's API
// (vk_symbiote/src/ConfigManager.cpp:15-120 file grammar, :669-689 flags, :773-787 bounds).
#include "../../../include/vk_symbiote/ConfigManager.h"

#include <chrono>
#include <ctime>
#include <fstream>
#include <iomanip>
#include <limits>
#include <iostream>
#include <sstream>

namespace vk_symbiote {

std::unique_ptr<ConfigManager> ConfigManager::instance_ = nullptr;
std::mutex ConfigManager::instance_mutex_;

ConfigManager& ConfigManager::instance() {
    std::lock_guard<std::mutex> lock(instance_mutex_);
    if (!instance_) {
        instance_ = std::make_unique<ConfigManager>(PrivateTag{});
        instance_->set_defaults();
    }
    return *instance_;
}

void ConfigManager::set_defaults() {
    memory_config_ = MemoryConfig{};
    perf_config_ = PerformanceConfig{};
    logging_config_ = LoggingConfig{};
    power_config_ = PowerConfig{};
    benchmark_config_ = BenchmarkConfig{};
    codec_config_ = CodecConfig{};
    batch_config_ = BatchConfig{};
    vitality_config_ = VitalityConfig{};
    shader_config_ = ShaderConfig{};
    parallel_config_ = ParallelConfig{};
    model_path_.clear();
    model_type_.clear();
    vram_budget_explicit_ = false;
    toml_data_.clear();
}

static std::string trim(const std::string& s) {
    const size_t a = s.find_first_not_of(" \t\r\n");
    if (a == std::string::npos) return "";
    const size_t b = s.find_last_not_of(" \t\r\n");
    return s.substr(a, b - a + 1);
}

// Value grammar of the reference parser: true/false, integers (digits and '-'), floats
// (anything with . e E that parses), otherwise a string with optional quotes. A trailing
// '# comment' after a value is dropped.
static ConfigManager::Value parse_value(std::string v) {
    if (!v.empty() && v[0] != '"' && v[0] != '\'') {
        const size_t hash = v.find('#');
        if (hash != std::string::npos) v = trim(v.substr(0, hash));
    }
    if (v == "true") return true;
    if (v == "false") return false;
    if (!v.empty() && v.find_first_not_of("0123456789-") == std::string::npos) {
        try {
            return (int64_t)std::stoll(v);
        } catch (...) {
        }
    }
    if (v.find_first_of(".eE") != std::string::npos) {
        try {
            size_t used = 0;
            double d = std::stod(v, &used);
            if (used == v.size()) return d;
        } catch (...) {
        }
    }
    if (v.size() >= 2 && ((v.front() == '"' && v.back() == '"') || (v.front() == '\'' && v.back() == '\'')))
        v = v.substr(1, v.size() - 2);
    return v;
}

bool ConfigManager::load_from_file(const Path& config_path) {
    std::ifstream f(config_path.string());
    if (!f.is_open()) {
        std::cerr << "Warning: Could not open config file: " << config_path.string() << std::endl;
        return false;
    }
    std::string line, section;
    while (std::getline(f, line)) {
        line = trim(line);
        if (line.empty() || line[0] == '#') continue;
        if (line.front() == '[' && line.back() == ']') {
            section = trim(line.substr(1, line.size() - 2));
            continue;
        }
        const size_t eq = line.find('=');
        if (eq == std::string::npos || section.empty()) continue;
        toml_data_[section][trim(line.substr(0, eq))] = parse_value(trim(line.substr(eq + 1)));
    }
    apply_document();
    return validate_config();
}

bool ConfigManager::load_from_toml(const Path& config_path) { return load_from_file(config_path); }

namespace {
struct Section {
    const std::unordered_map<std::string, ConfigManager::Value>* t = nullptr;
    const ConfigManager::Value* get(const char* k) const {
        if (!t) return nullptr;
        auto it = t->find(k);
        return it == t->end() ? nullptr : &it->second;
    }
    template <typename T>
    bool num(const char* k, T& dst) const {
        const ConfigManager::Value* v = get(k);
        if (!v) return false;
        if (std::holds_alternative<int64_t>(*v)) { dst = (T)std::get<int64_t>(*v); return true; }
        if (std::holds_alternative<double>(*v)) { dst = (T)std::get<double>(*v); return true; }
        return false;
    }
    void flag(const char* k, bool& dst) const {
        const ConfigManager::Value* v = get(k);
        if (v && std::holds_alternative<bool>(*v)) dst = std::get<bool>(*v);
    }
    void str(const char* k, std::string& dst) const {
        const ConfigManager::Value* v = get(k);
        if (v && std::holds_alternative<std::string>(*v)) dst = std::get<std::string>(*v);
    }
};
}  // namespace

void ConfigManager::apply_document() {
    auto sec = [&](const char* name) {
        Section s;
        auto it = toml_data_.find(name);
        if (it != toml_data_.end()) s.t = &it->second;
        return s;
    };
    Section m = sec("memory");
    if (m.num("vram_budget_gb", memory_config_.vram_budget_gb)) vram_budget_explicit_ = true;
    m.num("ram_budget_gb", memory_config_.ram_budget_gb);
    m.num("prefetch_lookahead", memory_config_.prefetch_lookahead);
    m.num("eviction_aggression", memory_config_.eviction_aggression);
    m.flag("enable_compression", memory_config_.enable_compression);
    m.str("compression_algorithm", memory_config_.compression_algorithm);
    m.num("max_packs_in_memory", memory_config_.max_packs_in_memory);
    m.flag("enable_defrag", memory_config_.enable_defrag);
    m.num("defrag_interval_ms", memory_config_.defrag_interval_ms);

    Section p = sec("performance");
    p.flag("enable_gpu", perf_config_.enable_gpu);
    p.flag("enable_profiling", perf_config_.enable_profiling);
    p.num("workgroup_size_x", perf_config_.workgroup_size_x);
    p.num("workgroup_size_y", perf_config_.workgroup_size_y);
    p.num("workgroup_size_z", perf_config_.workgroup_size_z);
    p.flag("use_subgroup_ops", perf_config_.use_subgroup_ops);
    p.num("subgroup_size", perf_config_.subgroup_size);
    p.flag("use_fp16_math", perf_config_.use_fp16_math);
    p.num("scale_factor", perf_config_.scale_factor);
    p.num("thread_pool_size", perf_config_.thread_pool_size);

    Section l = sec("logging");
    int level = (int)logging_config_.log_level;
    if (l.num("log_level", level)) logging_config_.log_level = (LogLevel)level;
    l.flag("log_to_file", logging_config_.log_to_file);
    l.str("log_file_path", logging_config_.log_file_path);
    l.flag("log_performance", logging_config_.log_performance);
    l.flag("log_memory_usage", logging_config_.log_memory_usage);
    l.num("max_log_file_size_mb", logging_config_.max_log_file_size_mb);
    l.flag("log_to_console", logging_config_.log_to_console);

    Section w = sec("power");
    w.flag("enable_power_management", power_config_.enable_power_management);
    w.flag("enable_power_saver", power_config_.enable_power_saver);
    w.flag("auto_detect_battery", power_config_.auto_detect_battery);
    w.num("power_profile", power_config_.power_profile);
    w.num("battery_threshold_low", power_config_.battery_threshold_low);
    w.num("battery_threshold_critical", power_config_.battery_threshold_critical);
    w.flag("throttle_on_thermal", power_config_.throttle_on_thermal);

    Section b = sec("benchmark");
    b.flag("enable_benchmark_mode", benchmark_config_.enable_benchmark_mode);
    b.num("warmup_tokens", benchmark_config_.warmup_tokens);
    b.num("benchmark_tokens", benchmark_config_.benchmark_tokens);
    b.num("iterations", benchmark_config_.iterations);
    b.flag("output_json", benchmark_config_.output_json);
    b.str("output_file", benchmark_config_.output_file);
    b.flag("test_power_modes", benchmark_config_.test_power_modes);
    b.flag("test_memory_pressure", benchmark_config_.test_memory_pressure);
    b.flag("detailed_layer_stats", benchmark_config_.detailed_layer_stats);

    Section c = sec("codec");
    c.str("codec", codec_config_.codec);
    c.num("compression_level", codec_config_.compression_level);
    c.flag("enable_blosc2", codec_config_.enable_blosc2);
    c.str("blosc2_compressor", codec_config_.blosc2_compressor);
    c.flag("enable_zfp", codec_config_.enable_zfp);
    c.num("zfp_precision", codec_config_.zfp_precision);
    c.flag("enable_hybrid", codec_config_.enable_hybrid);

    Section t = sec("batch");
    t.flag("enable_batching", batch_config_.enable_batching);
    t.num("max_batch_size", batch_config_.max_batch_size);
    t.flag("dynamic_batch_size", batch_config_.dynamic_batch_size);
    t.num("batch_timeout_ms", batch_config_.batch_timeout_ms);
    t.flag("share_kv_cache", batch_config_.share_kv_cache);
    t.num("max_sequence_length", batch_config_.max_sequence_length);

    Section v = sec("vitality");
    v.flag("enabled", vitality_config_.enabled);
    v.num("learning_rate", vitality_config_.learning_rate);
    v.num("momentum", vitality_config_.momentum);
    v.flag("use_adam", vitality_config_.use_adam);
    v.str("model_path", vitality_config_.model_path);

    Section s = sec("shader");
    s.str("cache_dir", shader_config_.cache_dir);
    s.flag("enable_cache", shader_config_.enable_cache);
    s.flag("use_cooperative_matrix", shader_config_.use_cooperative_matrix);
    s.flag("auto_tune", shader_config_.auto_tune);
    s.str("tuning_file", shader_config_.tuning_file);

    Section md = sec("model");
    md.str("path", model_path_);
    md.str("type", model_type_);

    Section par = sec("parallel");
    par.num("tp_size", parallel_config_.tp_size);
    par.num("device", parallel_config_.device);
}

bool ConfigManager::save_to_toml(const Path& config_path) {
    std::ofstream f(config_path.string());
    if (!f.is_open()) return false;
    f << "# Vulkan-Symbiote B200 configuration\n";
    // floats with enough digits to read back the same value (a fixed 2 decimals did not)
    f << std::setprecision(std::numeric_limits<float>::max_digits10);
    f << "[memory]\nvram_budget_gb = " << memory_config_.vram_budget_gb
      << "\nram_budget_gb = " << memory_config_.ram_budget_gb
      << "\nprefetch_lookahead = " << memory_config_.prefetch_lookahead
      << "\neviction_aggression = " << memory_config_.eviction_aggression
      << "\nenable_compression = " << (memory_config_.enable_compression ? "true" : "false") << "\n\n";
    f << "[performance]\nenable_gpu = " << (perf_config_.enable_gpu ? "true" : "false")
      << "\nenable_profiling = " << (perf_config_.enable_profiling ? "true" : "false")
      << "\nuse_fp16_math = " << (perf_config_.use_fp16_math ? "true" : "false") << "\n\n";
    f << "[benchmark]\nwarmup_tokens = " << benchmark_config_.warmup_tokens
      << "\nbenchmark_tokens = " << benchmark_config_.benchmark_tokens
      << "\niterations = " << benchmark_config_.iterations << "\n\n";
    f << "[parallel]\ntp_size = " << parallel_config_.tp_size << "\ndevice = " << parallel_config_.device << "\n";
    if (!model_path_.empty()) f << "\n[model]\npath = \"" << model_path_ << "\"\n";
    return (bool)f;
}

bool ConfigManager::save_to_file(const Path& config_path) { return save_to_toml(config_path); }

// Flags of the reference (:669-689) plus --disable-gpu and --tp; --vram-gb/--ram-gb take floats.
void ConfigManager::load_from_args(int argc, char* argv[]) {
    for (int i = 1; i < argc; ++i) {
        const std::string a = argv[i];
        const bool more = i + 1 < argc;
        try {
            if (a == "--model" && more) model_path_ = argv[++i];
            else if (a == "--config" && more) load_from_file(argv[++i]);
            else if (a == "--vram-gb" && more) {
                memory_config_.vram_budget_gb = std::stof(argv[++i]);
                vram_budget_explicit_ = true;
            } else if (a == "--ram-gb" && more) memory_config_.ram_budget_gb = std::stof(argv[++i]);
            else if (a == "--verbose" || a == "-v") logging_config_.log_level = LogLevel::DEBUG;
            else if (a == "--power-profile" && more) power_config_.power_profile = (uint32)std::stoul(argv[++i]);
            else if (a == "--benchmark") benchmark_config_.enable_benchmark_mode = true;
            else if (a == "--disable-gpu") perf_config_.enable_gpu = false;
            else if (a == "--tp" && more) parallel_config_.tp_size = (uint32)std::stoul(argv[++i]);
            else if (a == "--device" && more) parallel_config_.device = (uint32)std::stoul(argv[++i]);
        } catch (const std::exception&) {
            std::cerr << "Warning: ignoring malformed value for " << a << std::endl;
        }
    }
}

int ConfigManager::get_int(const std::string& section, const std::string& key, int def) const {
    auto s = toml_data_.find(section);
    if (s == toml_data_.end()) return def;
    auto k = s->second.find(key);
    if (k == s->second.end() || !std::holds_alternative<int64_t>(k->second)) return def;
    return (int)std::get<int64_t>(k->second);
}

float ConfigManager::get_float(const std::string& section, const std::string& key, float def) const {
    auto s = toml_data_.find(section);
    if (s == toml_data_.end()) return def;
    auto k = s->second.find(key);
    if (k == s->second.end() || !std::holds_alternative<double>(k->second)) return def;
    return (float)std::get<double>(k->second);
}

bool ConfigManager::get_bool(const std::string& section, const std::string& key, bool def) const {
    auto s = toml_data_.find(section);
    if (s == toml_data_.end()) return def;
    auto k = s->second.find(key);
    if (k == s->second.end() || !std::holds_alternative<bool>(k->second)) return def;
    return std::get<bool>(k->second);
}

std::string ConfigManager::get_string(const std::string& section, const std::string& key,
                                      const std::string& def) const {
    auto s = toml_data_.find(section);
    if (s == toml_data_.end()) return def;
    auto k = s->second.find(key);
    if (k == s->second.end() || !std::holds_alternative<std::string>(k->second)) return def;
    return std::get<std::string>(k->second);
}

bool ConfigManager::validate_config() const {
    bool ok = true;
    if (memory_config_.vram_budget_gb <= 0.0f || memory_config_.vram_budget_gb > 64.0f) {
        std::cerr << "Error: VRAM budget must be between 1-64 GB" << std::endl;
        ok = false;
    }
    if (memory_config_.ram_budget_gb <= 0.0f || memory_config_.ram_budget_gb > 128.0f) {
        std::cerr << "Error: RAM budget must be between 1-128 GB" << std::endl;
        ok = false;
    }
    if (parallel_config_.tp_size == 0) {
        std::cerr << "Error: tensor-parallel size must be at least 1" << std::endl;
        ok = false;
    }
    return ok;
}

void ConfigManager::print_config() const {
    std::cout << "=== Vulkan Symbiote (B200) Configuration ===\n"
              << "Memory:\n  VRAM Budget: " << memory_config_.vram_budget_gb << " GB"
              << (vram_budget_explicit_ ? "" : " (not set: no cap)") << "\n  RAM Budget: " << memory_config_.ram_budget_gb
              << " GB\n  Prefetch Lookahead: " << memory_config_.prefetch_lookahead
              << "\nPerformance:\n  GPU Enabled: " << (perf_config_.enable_gpu ? "Yes" : "No")
              << "\n  FP16 Math: " << (perf_config_.use_fp16_math ? "Yes" : "No")
              << "\nParallel:\n  TP size: " << parallel_config_.tp_size << "\n  Device: " << parallel_config_.device
              << "\nModel: " << (model_path_.empty() ? "(none)" : model_path_) << std::endl;
}

std::string ConfigManager::get_current_timestamp() const {
    const auto now = std::chrono::system_clock::now();
    const std::time_t t = std::chrono::system_clock::to_time_t(now);
    std::tm tm{};
    localtime_r(&t, &tm);
    std::ostringstream os;
    os << std::put_time(&tm, "%Y-%m-%d %H:%M:%S");
    return os.str();
}

}  // namespace vk_symbiote
