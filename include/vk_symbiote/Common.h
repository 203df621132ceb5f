// Shared types of the drop-in C++ API, re-declared without Vulkan headers.
// Mirrors vk_symbiote/include/vk_symbiote/Common.h of the reference: ModelConfig (:56-76),
// InferenceParams (:78-86), Expected<T> / ExpectedVoid (:88-193), Path (:195-202),
// PerformanceMetrics (:285-318). Vulkan-specific helpers (vk_result_to_string, ErrorContext
// with VkResult) have no counterpart: errors are VSL_ERR_* codes from include/vsl.h.
#pragma once

#include <chrono>
#include <cmath>
#include <cstddef>
#include <cstdint>
#include <filesystem>
#include <new>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

// Symbols of the C++ API exported from libvsl.so (built with hidden visibility).
#if defined(__GNUC__)
#define VSL_CPP_API __attribute__((visibility("default")))
#else
#define VSL_CPP_API
#endif

namespace vk_symbiote {

using uint8 = uint8_t;
using uint32 = uint32_t;
using uint64 = uint64_t;
using int8 = int8_t;
using int32 = int32_t;
using int64 = int64_t;
using float16 = uint16_t;

struct ModelConfig {
    uint32 hidden_size = 4096;
    uint32 num_layers = 32;
    uint32 num_attention_heads = 32;
    uint32 num_key_value_heads = 32;
    uint32 intermediate_size = 11008;
    uint32 vocab_size = 32000;
    float rope_theta = 10000.0f;
    uint32 max_position_embeddings = 2048;
    std::string model_type = "llama";
    uint32 head_dim = 128;
    bool use_fp16 = true;
    float rms_epsilon = 1e-5f;

    // Sparse long-context attention (reference defaults). The B200 engine runs dense
    // attention; these fields are kept for source compatibility.
    bool use_sparse_attention = true;
    uint32 sparse_window_size = 512;
    uint32 sparse_global_tokens = 16;
    uint32 sparse_block_size = 1024;
    bool use_ring_attention = true;
};

struct InferenceParams {
    uint32 max_new_tokens = 256;
    float temperature = 0.7f;
    float top_p = 0.9f;
    uint32 top_k = 40;
    bool do_sample = true;
    float repetition_penalty = 1.1f;
    uint32 context_length = 2048;
};

// Value-or-error-code, same shape as the reference's Expected<T>.
template <typename T>
class Expected {
public:
    Expected() : has_value_(true), error_code_(0) { new (storage_) T(); }
    Expected(const T& v) : has_value_(true), error_code_(0) { new (storage_) T(v); }
    Expected(T&& v) : has_value_(true), error_code_(0) { new (storage_) T(std::move(v)); }
    Expected(int err) : has_value_(false), error_code_(err) {}
    ~Expected() { reset(); }
    Expected(const Expected& o) : has_value_(o.has_value_), error_code_(o.error_code_) {
        if (has_value_) new (storage_) T(*o.ptr());
    }
    Expected(Expected&& o) noexcept : has_value_(o.has_value_), error_code_(o.error_code_) {
        if (has_value_) new (storage_) T(std::move(*o.ptr()));
    }
    Expected& operator=(const Expected& o) {
        if (this != &o) {
            reset();
            has_value_ = o.has_value_;
            error_code_ = o.error_code_;
            if (has_value_) new (storage_) T(*o.ptr());
        }
        return *this;
    }
    Expected& operator=(Expected&& o) noexcept {
        if (this != &o) {
            reset();
            has_value_ = o.has_value_;
            error_code_ = o.error_code_;
            if (has_value_) new (storage_) T(std::move(*o.ptr()));
        }
        return *this;
    }
    bool has_value() const noexcept { return has_value_; }
    explicit operator bool() const noexcept { return has_value_; }
    T& value() {
        if (!has_value_) throw std::runtime_error("Expected::value() called on error state");
        return *ptr();
    }
    const T& value() const {
        if (!has_value_) throw std::runtime_error("Expected::value() called on error state");
        return *ptr();
    }
    int error() const noexcept { return error_code_; }

private:
    T* ptr() { return reinterpret_cast<T*>(storage_); }
    const T* ptr() const { return reinterpret_cast<const T*>(storage_); }
    void reset() {
        if (has_value_) ptr()->~T();
        has_value_ = false;
    }
    bool has_value_;
    alignas(T) unsigned char storage_[sizeof(T)];
    int error_code_;
};

template <>
class Expected<void> {
public:
    Expected() : error_code_(0), has_value_(true) {}
    Expected(int err) : error_code_(err), has_value_(false) {}
    bool has_value() const noexcept { return has_value_; }
    explicit operator bool() const noexcept { return has_value_; }
    int error() const noexcept { return error_code_; }

private:
    int error_code_;
    bool has_value_;
};

using ExpectedVoid = Expected<void>;

struct Path : public std::filesystem::path {
    Path() : std::filesystem::path() {}
    Path(const std::string& p) : std::filesystem::path(p) {}
    Path(const char* p) : std::filesystem::path(p) {}
    Path(const std::filesystem::path& p) : std::filesystem::path(p) {}
    const char* c_str() const noexcept { return native().c_str(); }
};

inline uint64 get_current_time_ns() {
    return std::chrono::duration_cast<std::chrono::nanoseconds>(
               std::chrono::steady_clock::now().time_since_epoch())
        .count();
}

inline float silu(float x) { return x / (1.0f + std::exp(-x)); }

struct PerformanceMetrics {
    uint64_t total_inference_time_ns = 0;
    uint64_t total_gpu_time_ns = 0;
    uint64_t total_cpu_time_ns = 0;
    uint32_t total_inferences = 0;
    uint32_t successful_inferences = 0;
    float average_tokens_per_second = 0.0f;
    float gpu_utilization_percent = 0.0f;
    // achieved algorithmic HBM bandwidth of the decode loop (weights + KV read per token)
    float memory_bandwidth_gbps = 0.0f;

    void reset() { *this = PerformanceMetrics(); }
    void update(uint64_t inference_time_ns, uint32_t tokens_generated) {
        total_inferences++;
        if (inference_time_ns > 0) {
            total_inference_time_ns += inference_time_ns;
            successful_inferences++;
            if (tokens_generated > 0)
                average_tokens_per_second = (float)tokens_generated / ((float)inference_time_ns / 1e9f);
        }
    }
};

// Memory pool statistics (reference NomadPack.h:53-57), filled from the HBM arena.
struct MemoryPoolStats {
    uint64 total_size = 0, used_size = 0, free_size = 0;
    uint32 allocation_count = 0;
    float fragmentation_ratio = 0.0f;
};

}  // namespace vk_symbiote
