// GGUF model reader with the reference's GGUFLoader API
// (vk_symbiote/include/vk_symbiote/GGUFLoader.h:265-333).
//
// Differences from the reference, each a documented compatibility decision:
//   - tensor types use ggml's ids (F32 0, F16 1, Q4_0 2, Q4_1 3, Q8_0 8, BF16 30); the
//     reference cast them into its metadata enum (GGUFLoader.cpp:901-903). Files written
//     with the reference's ids (FLOAT32 6, FLOAT16 48, BFLOAT16 47) load when
//     set_legacy_dtype_ids(true) is called first;
//   - the data section starts at the next multiple of general.alignment (default 32);
//   - metadata arrays are parsed with their element type and count.
// The bulk path for the B200 engine is map_tensor(): a pointer into the memory-mapped file
// (native dtype, no upcast) that the engine stages through pinned memory into HBM.
#pragma once

#include <cstdint>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "Common.h"
#include "NomadPack.h"

namespace vk_symbiote {

// Metadata value types (GGUF spec; identical to the reference's ids 0..12).
enum class GGUFValueType : uint32 {
    UINT8 = 0, INT8 = 1, UINT16 = 2, INT16 = 3, UINT32 = 4, INT32 = 5, FLOAT32 = 6, BOOL = 7,
    STRING = 8, ARRAY = 9, UINT64 = 10, INT64 = 11, FLOAT64 = 12
};

// Tensor element types (ggml ids).
enum class GGMLType : uint32 { F32 = 0, F16 = 1, Q4_0 = 2, Q4_1 = 3, Q8_0 = 8, BF16 = 30, UNKNOWN = 0xffffffffu };

struct GGUFHeader {
    uint32 magic = 0;
    uint32 version = 0;
    uint64 tensor_count = 0;
    uint64 metadata_kv_count = 0;
};

struct VSL_CPP_API GGUFTensorInfo {
    std::string name;
    uint32 n_dimensions = 0;
    std::vector<uint64> dimensions;  // ne[0] is the contiguous dimension
    GGMLType data_type = GGMLType::UNKNOWN;
    uint64 offset = 0;       // relative to the data section
    uint64 data_offset = 0;  // absolute offset in the file
    uint64 data_size = 0;    // bytes
    bool is_compressed = false;
    uint32 compression_codec = 0;
    uint64 element_count() const;
};

struct VSL_CPP_API GGUFMetadataKV {
    std::string key;
    GGUFValueType value_type = GGUFValueType::UINT8;
    std::vector<uint8_t> raw_value;  // scalar bytes; string bytes; array: element bytes
    GGUFValueType array_type = GGUFValueType::UINT8;
    uint64 array_count = 0;
    std::vector<std::string> array_strings;  // string arrays

    std::string get_string() const;
    uint32_t get_uint32() const;
    int32_t get_int32() const;
    float get_float32() const;
    bool get_bool() const;
    double get_number() const;  // any numeric scalar as double
    std::vector<uint8_t> get_array_data() const;
    GGUFValueType get_array_element_type() const;
};

struct VocabularyEntry {
    std::string token;
    std::vector<uint8_t> bytes;
    float score = 0.0f;
    uint32_t token_type = 0;
    bool is_special = false;
};

struct TokenizerConfig {
    std::string model_type = "gpt2";
    bool add_bos_token = false;
    bool add_eos_token = false;
    uint32_t bos_token_id = 0;
    uint32_t eos_token_id = 0;
    uint32_t pad_token_id = 0;
    uint32_t unk_token_id = 0;
    std::string chat_template;
    std::string pre_tokenizer;
    bool add_space_prefix = true;
    bool remove_extra_whitespaces = false;
    std::vector<std::pair<std::string, uint32_t>> added_tokens;
};

struct TensorCacheConfig {
    size_t max_entries = 256;
    size_t max_memory_bytes = 4ULL * 1024 * 1024 * 1024;
    uint64_t ttl_seconds = 300;
    bool enable_compression = false;
};

class VSL_CPP_API GGUFLoader {
public:
    explicit GGUFLoader(const Path& file_path);
    ~GGUFLoader();
    GGUFLoader(const GGUFLoader&) = delete;
    GGUFLoader& operator=(const GGUFLoader&) = delete;

    ExpectedVoid load();
    ExpectedVoid close();

    ModelConfig get_model_config() const;
    std::vector<PackMetadata> generate_packs(const ModelConfig& config);

    uint64 tensor_count() const;
    uint64 metadata_count() const;

    const GGUFTensorInfo* get_tensor(const std::string& name) const;
    // Host fp32 copy of a tensor (F32 / F16 / BF16 / Q8_0 / Q4_0 / Q4_1). With
    // fp16_to_fp32 == false, F16/BF16 tensors are returned as their raw bits widened to
    // float values of the 16-bit pattern (reference behaviour is to always upcast).
    Expected<std::vector<float>> read_tensor_data(const GGUFTensorInfo& tensor, bool fp16_to_fp32 = true);
    Expected<std::vector<float>> read_tensor_cached(const std::string& tensor_name, bool fp16_to_fp32 = true);
    std::vector<Expected<std::vector<float>>> read_tensors_parallel(const std::vector<std::string>& tensor_names,
                                                                    bool fp16_to_fp32 = true);

    // Pointer into the mapped file at the tensor's data (native encoding), or nullptr.
    const void* map_tensor(const std::string& name) const;

    const std::vector<VocabularyEntry>& get_vocabulary() const;
    const TokenizerConfig& get_tokenizer_config() const;

    void clear_tensor_cache();
    size_t get_tensor_cache_size() const;
    void configure_cache(const TensorCacheConfig& config);

    std::vector<std::string> get_tensor_names() const;
    std::vector<std::string> get_metadata_keys() const;
    const GGUFMetadataKV* get_metadata(const std::string& key) const;

    static uint64 align_offset(uint64 offset, uint64 alignment);
    uint32_t get_version() const;
    bool is_valid() const;

    // Accept the reference's own tensor type ids (FLOAT32 6, FLOAT16 48, BFLOAT16 47).
    void set_legacy_dtype_ids(bool on);

    struct Impl;

private:
    Path file_path_;
    std::unique_ptr<Impl> pimpl_;
};

}  // namespace vk_symbiote
