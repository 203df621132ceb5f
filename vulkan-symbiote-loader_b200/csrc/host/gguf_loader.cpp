// GGUF reader behind the reference's GGUFLoader API (vk_symbiote/src/GGUFLoader.cpp).
// The file is memory-mapped once; tensor data is never copied on the host except into the
// engine's pinned staging buffers (bulk path) or for the fp32 compatibility accessors.
#include "../../../include/vk_symbiote/GGUFLoader.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <functional>
#include <list>
#include <mutex>
#include <thread>

#include "../../../include/vsl.h"
#include "status.h"

namespace vk_symbiote {

uint64 GGUFTensorInfo::element_count() const {
    uint64 n = 1;
    for (uint64 d : dimensions) n *= d;
    return n;
}

// ---- metadata accessors ----
static double scalar_as_double(GGUFValueType t, const uint8_t* p) {
    switch (t) {
        case GGUFValueType::UINT8: return *p;
        case GGUFValueType::INT8: return (int8_t)*p;
        case GGUFValueType::BOOL: return *p;
        case GGUFValueType::UINT16: { uint16_t v; memcpy(&v, p, 2); return v; }
        case GGUFValueType::INT16: { int16_t v; memcpy(&v, p, 2); return v; }
        case GGUFValueType::UINT32: { uint32_t v; memcpy(&v, p, 4); return v; }
        case GGUFValueType::INT32: { int32_t v; memcpy(&v, p, 4); return v; }
        case GGUFValueType::FLOAT32: { float v; memcpy(&v, p, 4); return v; }
        case GGUFValueType::UINT64: { uint64_t v; memcpy(&v, p, 8); return (double)v; }
        case GGUFValueType::INT64: { int64_t v; memcpy(&v, p, 8); return (double)v; }
        case GGUFValueType::FLOAT64: { double v; memcpy(&v, p, 8); return v; }
        default: return 0.0;
    }
}

std::string GGUFMetadataKV::get_string() const {
    if (value_type != GGUFValueType::STRING) return {};
    return std::string(raw_value.begin(), raw_value.end());
}
double GGUFMetadataKV::get_number() const {
    if (value_type == GGUFValueType::STRING || value_type == GGUFValueType::ARRAY || raw_value.empty()) return 0.0;
    return scalar_as_double(value_type, raw_value.data());
}
uint32_t GGUFMetadataKV::get_uint32() const { return (uint32_t)get_number(); }
int32_t GGUFMetadataKV::get_int32() const { return (int32_t)get_number(); }
float GGUFMetadataKV::get_float32() const { return (float)get_number(); }
bool GGUFMetadataKV::get_bool() const { return get_number() != 0.0; }
std::vector<uint8_t> GGUFMetadataKV::get_array_data() const {
    return value_type == GGUFValueType::ARRAY ? raw_value : std::vector<uint8_t>{};
}
GGUFValueType GGUFMetadataKV::get_array_element_type() const { return array_type; }

// ---- implementation ----
struct GGUFLoader::Impl {
    int fd = -1;
    const uint8_t* map = nullptr;
    size_t size = 0;
    GGUFHeader header;
    uint64 alignment = 32;
    uint64 data_start = 0;
    bool legacy_ids = false;
    bool loaded = false;
    std::vector<GGUFMetadataKV> kvs;
    std::unordered_map<std::string, size_t> kv_index;
    std::vector<GGUFTensorInfo> tensors;
    std::unordered_map<std::string, size_t> tensor_index;
    std::vector<VocabularyEntry> vocab;
    TokenizerConfig tok_cfg;
    // LRU cache of fp32 copies (read_tensor_cached)
    TensorCacheConfig cache_cfg;
    std::list<std::pair<std::string, std::vector<float>>> lru;
    std::unordered_map<std::string, std::list<std::pair<std::string, std::vector<float>>>::iterator> lru_map;
    size_t cache_bytes = 0;
    std::mutex cache_mu;

    const uint8_t* p = nullptr;
    const uint8_t* end = nullptr;
    bool err = false;

    template <typename T>
    T rd() {
        T v{};
        if (p + sizeof(T) > end) { err = true; return v; }
        memcpy(&v, p, sizeof(T));
        p += sizeof(T);
        return v;
    }
    std::string rd_str() {
        uint64_t n = rd<uint64_t>();
        if (err || n > (uint64_t)(end - p)) { err = true; return {}; }
        std::string s((const char*)p, (size_t)n);
        p += n;
        return s;
    }
    static size_t scalar_size(GGUFValueType t) {
        switch (t) {
            case GGUFValueType::UINT8: case GGUFValueType::INT8: case GGUFValueType::BOOL: return 1;
            case GGUFValueType::UINT16: case GGUFValueType::INT16: return 2;
            case GGUFValueType::UINT32: case GGUFValueType::INT32: case GGUFValueType::FLOAT32: return 4;
            case GGUFValueType::UINT64: case GGUFValueType::INT64: case GGUFValueType::FLOAT64: return 8;
            default: return 0;
        }
    }
    bool parse_value(GGUFMetadataKV& kv) {
        if (kv.value_type == GGUFValueType::STRING) {
            std::string s = rd_str();
            kv.raw_value.assign(s.begin(), s.end());
        } else if (kv.value_type == GGUFValueType::ARRAY) {
            kv.array_type = (GGUFValueType)rd<uint32_t>();
            kv.array_count = rd<uint64_t>();
            if (err) return false;
            if (kv.array_type == GGUFValueType::STRING) {
                kv.array_strings.reserve((size_t)std::min<uint64_t>(kv.array_count, 1u << 22));
                for (uint64_t i = 0; i < kv.array_count && !err; i++) kv.array_strings.push_back(rd_str());
            } else {
                size_t es = scalar_size(kv.array_type);
                if (!es || kv.array_count > (uint64_t)(end - p) / es) { err = true; return false; }
                kv.raw_value.assign(p, p + es * kv.array_count);
                p += es * kv.array_count;
            }
        } else {
            size_t es = scalar_size(kv.value_type);
            if (!es || p + es > end) { err = true; return false; }
            kv.raw_value.assign(p, p + es);
            p += es;
        }
        return !err;
    }
    GGMLType map_type(uint32_t t) const {
        if (legacy_ids) {  // reference ids (GGUFLoader.h:25,66-67)
            if (t == 6) return GGMLType::F32;
            if (t == 48) return GGMLType::F16;
            if (t == 47) return GGMLType::BF16;
        }
        switch (t) {
            case 0: return GGMLType::F32;
            case 1: return GGMLType::F16;
            case 2: return GGMLType::Q4_0;
            case 3: return GGMLType::Q4_1;
            case 8: return GGMLType::Q8_0;
            case 30: return GGMLType::BF16;
            default: return GGMLType::UNKNOWN;
        }
    }
    static uint64 data_bytes(GGMLType t, uint64 n) {
        switch (t) {
            case GGMLType::F32: return n * 4;
            case GGMLType::F16: case GGMLType::BF16: return n * 2;
            case GGMLType::Q8_0: return n / 32 * 34;
            case GGMLType::Q4_0: return n / 32 * 18;
            case GGMLType::Q4_1: return n / 32 * 20;
            default: return 0;
        }
    }
    const GGUFMetadataKV* meta(const std::string& k) const {
        auto it = kv_index.find(k);
        return it == kv_index.end() ? nullptr : &kvs[it->second];
    }
};

GGUFLoader::GGUFLoader(const Path& file_path) : file_path_(file_path), pimpl_(new Impl) {}
GGUFLoader::~GGUFLoader() { close(); }

ExpectedVoid GGUFLoader::close() {
    Impl& m = *pimpl_;
    if (m.map) munmap((void*)m.map, m.size);
    if (m.fd >= 0) ::close(m.fd);
    m.map = nullptr;
    m.fd = -1;
    m.loaded = false;
    return ExpectedVoid();
}

void GGUFLoader::set_legacy_dtype_ids(bool on) { pimpl_->legacy_ids = on; }

uint64 GGUFLoader::align_offset(uint64 offset, uint64 alignment) {
    return alignment ? (offset + alignment - 1) / alignment * alignment : offset;
}

// GGUFLoaderImpl::load (GGUFLoader.cpp:625-663): header, metadata, tensor infos, data offsets.
ExpectedVoid GGUFLoader::load() {
    Impl& m = *pimpl_;
    close();
    m.fd = ::open(file_path_.c_str(), O_RDONLY);
    if (m.fd < 0) return ExpectedVoid(VSL_ERR_IO);
    struct stat st;
    if (fstat(m.fd, &st) != 0 || st.st_size < 24) { close(); return ExpectedVoid(VSL_ERR_FORMAT); }
    m.size = (size_t)st.st_size;
    void* mp = mmap(nullptr, m.size, PROT_READ, MAP_SHARED, m.fd, 0);
    if (mp == MAP_FAILED) { m.map = nullptr; close(); return ExpectedVoid(VSL_ERR_IO); }
    m.map = (const uint8_t*)mp;
    m.p = m.map;
    m.end = m.map + m.size;
    m.err = false;
    m.kvs.clear(); m.kv_index.clear(); m.tensors.clear(); m.tensor_index.clear(); m.vocab.clear();
    m.header.magic = m.rd<uint32_t>();
    m.header.version = m.rd<uint32_t>();
    if (m.header.magic != 0x46554747u) { close(); return ExpectedVoid(VSL_ERR_FORMAT); }
    if (m.header.version < 2 || m.header.version > 3) { close(); return ExpectedVoid(VSL_ERR_FORMAT); }
    m.header.tensor_count = m.rd<uint64_t>();
    m.header.metadata_kv_count = m.rd<uint64_t>();
    if (m.err || m.header.tensor_count > (1u << 24) || m.header.metadata_kv_count > (1u << 24)) {
        close();
        return ExpectedVoid(VSL_ERR_FORMAT);
    }
    for (uint64_t i = 0; i < m.header.metadata_kv_count; i++) {
        GGUFMetadataKV kv;
        kv.key = m.rd_str();
        kv.value_type = (GGUFValueType)m.rd<uint32_t>();
        if (m.err || (uint32_t)kv.value_type > 12 || !m.parse_value(kv)) { close(); return ExpectedVoid(VSL_ERR_FORMAT); }
        m.kv_index[kv.key] = m.kvs.size();
        m.kvs.push_back(std::move(kv));
    }
    if (auto a = m.meta("general.alignment")) m.alignment = a->get_uint32() ? a->get_uint32() : 32;
    for (uint64_t i = 0; i < m.header.tensor_count; i++) {
        GGUFTensorInfo t;
        t.name = m.rd_str();
        t.n_dimensions = m.rd<uint32_t>();
        if (m.err || t.n_dimensions == 0 || t.n_dimensions > 4) { close(); return ExpectedVoid(VSL_ERR_FORMAT); }
        for (uint32_t d = 0; d < t.n_dimensions; d++) t.dimensions.push_back(m.rd<uint64_t>());
        t.data_type = m.map_type(m.rd<uint32_t>());
        t.offset = m.rd<uint64_t>();
        if (m.err) { close(); return ExpectedVoid(VSL_ERR_FORMAT); }
        m.tensor_index[t.name] = m.tensors.size();
        m.tensors.push_back(std::move(t));
    }
    m.data_start = align_offset((uint64)(m.p - m.map), m.alignment);
    for (auto& t : m.tensors) {
        t.data_offset = m.data_start + t.offset;
        t.data_size = Impl::data_bytes(t.data_type, t.element_count());
        if (t.data_type != GGMLType::UNKNOWN && t.data_offset + t.data_size > m.size) {
            close();
            return ExpectedVoid(VSL_ERR_FORMAT);  // truncated file
        }
    }
    // vocabulary (tokenizer.ggml.*), parsed with its real element type and count
    if (auto toks = m.meta("tokenizer.ggml.tokens")) {
        const GGUFMetadataKV* scores = m.meta("tokenizer.ggml.scores");
        const GGUFMetadataKV* types = m.meta("tokenizer.ggml.token_type");
        for (size_t i = 0; i < toks->array_strings.size(); i++) {
            VocabularyEntry e;
            e.token = toks->array_strings[i];
            e.bytes.assign(e.token.begin(), e.token.end());
            if (scores && scores->array_type == GGUFValueType::FLOAT32 && i < scores->array_count)
                memcpy(&e.score, scores->raw_value.data() + 4 * i, 4);
            if (types && types->array_type == GGUFValueType::INT32 && i < types->array_count)
                memcpy(&e.token_type, types->raw_value.data() + 4 * i, 4);
            m.vocab.push_back(std::move(e));
        }
    }
    if (auto v = m.meta("tokenizer.ggml.model")) m.tok_cfg.model_type = v->get_string();
    if (auto v = m.meta("tokenizer.ggml.bos_token_id")) m.tok_cfg.bos_token_id = v->get_uint32();
    if (auto v = m.meta("tokenizer.ggml.eos_token_id")) m.tok_cfg.eos_token_id = v->get_uint32();
    if (auto v = m.meta("tokenizer.ggml.unknown_token_id")) m.tok_cfg.unk_token_id = v->get_uint32();
    if (auto v = m.meta("tokenizer.ggml.padding_token_id")) m.tok_cfg.pad_token_id = v->get_uint32();
    if (auto v = m.meta("tokenizer.ggml.add_bos_token")) m.tok_cfg.add_bos_token = v->get_bool();
    if (auto v = m.meta("tokenizer.ggml.add_eos_token")) m.tok_cfg.add_eos_token = v->get_bool();
    if (auto v = m.meta("tokenizer.ggml.add_space_prefix")) m.tok_cfg.add_space_prefix = v->get_bool();
    if (auto v = m.meta("tokenizer.ggml.pre")) m.tok_cfg.pre_tokenizer = v->get_string();
    if (auto v = m.meta("tokenizer.chat_template")) m.tok_cfg.chat_template = v->get_string();
    m.loaded = true;
    return ExpectedVoid();
}

// get_model_config (GGUFLoader.cpp:673-728): same keys; head_dim = d / heads (:725). The
// vocabulary size falls back to the token array length, then to token_embd's rows.
ModelConfig GGUFLoader::get_model_config() const {
    const Impl& m = *pimpl_;
    ModelConfig c;
    if (auto kv = m.meta("llama.embedding_length")) c.hidden_size = kv->get_uint32();
    else if (auto kv2 = m.meta("general.embedding_length")) c.hidden_size = kv2->get_uint32();
    if (auto kv = m.meta("llama.block_count")) c.num_layers = kv->get_uint32();
    else if (auto kv2 = m.meta("general.block_count")) c.num_layers = kv2->get_uint32();
    if (auto kv = m.meta("llama.attention.head_count")) c.num_attention_heads = kv->get_uint32();
    if (auto kv = m.meta("llama.attention.head_count_kv")) c.num_key_value_heads = kv->get_uint32();
    else c.num_key_value_heads = c.num_attention_heads;
    if (auto kv = m.meta("llama.feed_forward_length")) c.intermediate_size = kv->get_uint32();
    if (auto kv = m.meta("llama.vocab_size")) c.vocab_size = kv->get_uint32();
    else if (auto kv2 = m.meta("tokenizer.ggml.tokens")) c.vocab_size = (uint32)kv2->array_count;
    else if (auto t = get_tensor("token_embd.weight"); t && t->dimensions.size() == 2)
        c.vocab_size = (uint32)t->dimensions[1];
    if (auto kv = m.meta("llama.rope.freq_base")) c.rope_theta = kv->get_float32();
    if (auto kv = m.meta("llama.context_length")) c.max_position_embeddings = kv->get_uint32();
    if (auto kv = m.meta("llama.attention.layer_norm_rms_epsilon")) c.rms_epsilon = kv->get_float32();
    if (auto kv = m.meta("general.architecture")) c.model_type = kv->get_string();
    if (c.num_attention_heads) c.head_dim = c.hidden_size / c.num_attention_heads;
    if (auto t = get_tensor("token_embd.weight")) c.use_fp16 = t->data_type != GGMLType::F32;
    return c;
}

static PackType classify(const std::string& n) {
    if (n.find("attn_q.") != std::string::npos) return PackType::ATTENTION_Q;
    if (n.find("attn_k.") != std::string::npos) return PackType::ATTENTION_K;
    if (n.find("attn_v.") != std::string::npos) return PackType::ATTENTION_V;
    if (n.find("attn_output.") != std::string::npos || n.find("attn_o.") != std::string::npos)
        return PackType::ATTENTION_O;
    if (n.find("ffn_gate") != std::string::npos) return PackType::FEED_FORWARD_GATE;
    if (n.find("ffn_up") != std::string::npos) return PackType::FEED_FORWARD_UP;
    if (n.find("ffn_down") != std::string::npos) return PackType::FEED_FORWARD_DOWN;
    if (n.find("norm") != std::string::npos) return PackType::NORM_GAMMA;
    if (n.find("token_embd") != std::string::npos) return PackType::EMBEDDING;
    if (n.rfind("output.", 0) == 0) return PackType::HEAD;
    return PackType::UNKNOWN;
}

// generate_packs (GGUFLoader.cpp:730-751): one pack per tensor, id = hash of the name.
std::vector<PackMetadata> GGUFLoader::generate_packs(const ModelConfig&) {
    std::vector<PackMetadata> packs;
    for (const auto& t : pimpl_->tensors) {
        PackMetadata p;
        p.pack_id = std::hash<std::string>{}(t.name);
        p.tensor_name = t.name;
        if (t.name.rfind("blk.", 0) == 0) p.layer_idx = (uint32)std::strtoul(t.name.c_str() + 4, nullptr, 10);
        p.compressed_size = p.decompressed_size = t.data_size;
        p.file_offset = t.data_offset;
        p.type = classify(t.name);
        p.base_priority = (p.type == PackType::EMBEDDING || p.type == PackType::HEAD) ? 1.0f : 0.5f;
        p.n_dimensions = t.n_dimensions;
        p.dimensions = t.dimensions;
        packs.push_back(std::move(p));
    }
    return packs;
}

uint64 GGUFLoader::tensor_count() const { return pimpl_->tensors.size(); }
uint64 GGUFLoader::metadata_count() const { return pimpl_->kvs.size(); }
uint32_t GGUFLoader::get_version() const { return pimpl_->header.version; }
bool GGUFLoader::is_valid() const { return pimpl_->loaded; }

const GGUFTensorInfo* GGUFLoader::get_tensor(const std::string& name) const {
    auto it = pimpl_->tensor_index.find(name);
    return it == pimpl_->tensor_index.end() ? nullptr : &pimpl_->tensors[it->second];
}

const void* GGUFLoader::map_tensor(const std::string& name) const {
    const GGUFTensorInfo* t = get_tensor(name);
    if (!t || !pimpl_->map) return nullptr;
    return pimpl_->map + t->data_offset;
}

static float half_to_float(uint16_t h) {
    // exact IEEE binary16 -> binary32 (convert_fp16_to_fp32, GGUFLoader.cpp:1225-1262)
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1fu, mant = h & 0x3ffu, bits;
    if (e == 0) {
        if (mant == 0) bits = sign;
        else {
            int ee = 113;
            while (!(mant & 0x400u)) { mant <<= 1; ee--; }
            bits = sign | ((uint32_t)ee << 23) | ((mant & 0x3ffu) << 13);
        }
    } else if (e == 31) bits = sign | 0x7f800000u | (mant << 13);
    else bits = sign | ((e + 112u) << 23) | (mant << 13);
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

// read_tensor_data (GGUFLoader.cpp:761-793) with the Q8_0/Q4_0/Q4_1 dequantisers
// (:1121-1223): blocks of 32 elements with an fp16 scale (and minimum for Q4_1).
Expected<std::vector<float>> GGUFLoader::read_tensor_data(const GGUFTensorInfo& t, bool fp16_to_fp32) {
    const Impl& m = *pimpl_;
    if (!m.map) return Expected<std::vector<float>>(VSL_ERR_STATE);
    const uint8_t* src = m.map + t.data_offset;
    const uint64 n = t.element_count();
    std::vector<float> out((size_t)n);
    switch (t.data_type) {
        case GGMLType::F32: memcpy(out.data(), src, n * 4); break;
        case GGMLType::F16:
            for (uint64 i = 0; i < n; i++) {
                uint16_t h; memcpy(&h, src + 2 * i, 2);
                out[i] = fp16_to_fp32 ? half_to_float(h) : (float)h;
            }
            break;
        case GGMLType::BF16:
            for (uint64 i = 0; i < n; i++) {
                uint16_t h; memcpy(&h, src + 2 * i, 2);
                uint32_t bits = (uint32_t)h << 16;
                float f; memcpy(&f, &bits, 4);
                out[i] = fp16_to_fp32 ? f : (float)h;
            }
            break;
        case GGMLType::Q8_0:
            for (uint64 b = 0; b < n / 32; b++) {
                const uint8_t* blk = src + b * 34;
                uint16_t d; memcpy(&d, blk, 2);
                const float s = half_to_float(d);
                for (int i = 0; i < 32; i++) out[b * 32 + i] = s * (float)(int8_t)blk[2 + i];
            }
            break;
        case GGMLType::Q4_0:
            for (uint64 b = 0; b < n / 32; b++) {
                const uint8_t* blk = src + b * 18;
                uint16_t d; memcpy(&d, blk, 2);
                const float s = half_to_float(d);
                for (int i = 0; i < 16; i++) {
                    out[b * 32 + i] = s * (float)((int)(blk[2 + i] & 0xf) - 8);
                    out[b * 32 + 16 + i] = s * (float)((int)(blk[2 + i] >> 4) - 8);
                }
            }
            break;
        case GGMLType::Q4_1:
            for (uint64 b = 0; b < n / 32; b++) {
                const uint8_t* blk = src + b * 20;
                uint16_t d, mn; memcpy(&d, blk, 2); memcpy(&mn, blk + 2, 2);
                const float s = half_to_float(d), mm = half_to_float(mn);
                for (int i = 0; i < 16; i++) {
                    out[b * 32 + i] = s * (float)(blk[4 + i] & 0xf) + mm;
                    out[b * 32 + 16 + i] = s * (float)(blk[4 + i] >> 4) + mm;
                }
            }
            break;
        default: return Expected<std::vector<float>>(VSL_ERR_UNSUPPORTED);
    }
    return Expected<std::vector<float>>(std::move(out));
}

// read_tensor_cached (GGUFLoader.cpp:1371-1392): LRU over fp32 copies.
Expected<std::vector<float>> GGUFLoader::read_tensor_cached(const std::string& name, bool fp16_to_fp32) {
    Impl& m = *pimpl_;
    const std::string key = name + (fp16_to_fp32 ? "#f32" : "#raw");
    {
        std::lock_guard<std::mutex> lk(m.cache_mu);
        auto it = m.lru_map.find(key);
        if (it != m.lru_map.end()) {
            m.lru.splice(m.lru.begin(), m.lru, it->second);
            return Expected<std::vector<float>>(it->second->second);
        }
    }
    const GGUFTensorInfo* t = get_tensor(name);
    if (!t) return Expected<std::vector<float>>(VSL_ERR_INVALID);
    auto r = read_tensor_data(*t, fp16_to_fp32);
    if (!r) return r;
    std::lock_guard<std::mutex> lk(m.cache_mu);
    const size_t bytes = r.value().size() * sizeof(float);
    // another thread may have read and cached the same tensor meanwhile: keep one copy
    if (bytes <= m.cache_cfg.max_memory_bytes && m.lru_map.find(key) == m.lru_map.end()) {
        m.lru.emplace_front(key, r.value());
        m.lru_map[key] = m.lru.begin();
        m.cache_bytes += bytes;
        while (!m.lru.empty() &&
               (m.cache_bytes > m.cache_cfg.max_memory_bytes || m.lru.size() > m.cache_cfg.max_entries)) {
            m.cache_bytes -= m.lru.back().second.size() * sizeof(float);
            m.lru_map.erase(m.lru.back().first);
            m.lru.pop_back();
        }
    }
    return r;
}

std::vector<Expected<std::vector<float>>> GGUFLoader::read_tensors_parallel(const std::vector<std::string>& names,
                                                                           bool fp16_to_fp32) {
    std::vector<Expected<std::vector<float>>> out(names.size(), Expected<std::vector<float>>(VSL_ERR_STATE));
    std::vector<std::thread> th;
    const size_t nt = std::max<size_t>(1, std::min<size_t>(names.size(), std::thread::hardware_concurrency()));
    for (size_t w = 0; w < nt; w++)
        th.emplace_back([&, w] {
            for (size_t i = w; i < names.size(); i += nt) {
                const GGUFTensorInfo* t = get_tensor(names[i]);
                out[i] = t ? read_tensor_data(*t, fp16_to_fp32) : Expected<std::vector<float>>(VSL_ERR_INVALID);
            }
        });
    for (auto& t : th) t.join();
    return out;
}

const std::vector<VocabularyEntry>& GGUFLoader::get_vocabulary() const { return pimpl_->vocab; }
const TokenizerConfig& GGUFLoader::get_tokenizer_config() const { return pimpl_->tok_cfg; }

void GGUFLoader::clear_tensor_cache() {
    std::lock_guard<std::mutex> lk(pimpl_->cache_mu);
    pimpl_->lru.clear();
    pimpl_->lru_map.clear();
    pimpl_->cache_bytes = 0;
}
size_t GGUFLoader::get_tensor_cache_size() const {
    std::lock_guard<std::mutex> lk(pimpl_->cache_mu);
    return pimpl_->lru.size();
}
void GGUFLoader::configure_cache(const TensorCacheConfig& c) {
    std::lock_guard<std::mutex> lk(pimpl_->cache_mu);
    pimpl_->cache_cfg = c;
}

std::vector<std::string> GGUFLoader::get_tensor_names() const {
    std::vector<std::string> v;
    for (const auto& t : pimpl_->tensors) v.push_back(t.name);
    return v;
}
std::vector<std::string> GGUFLoader::get_metadata_keys() const {
    std::vector<std::string> v;
    for (const auto& k : pimpl_->kvs) v.push_back(k.key);
    return v;
}
const GGUFMetadataKV* GGUFLoader::get_metadata(const std::string& key) const { return pimpl_->meta(key); }

}  // namespace vk_symbiote
