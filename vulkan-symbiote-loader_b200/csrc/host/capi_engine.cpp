// C ABI over DecodeEngine (vsl_engine_*). No exception crosses this boundary.
#include <nccl.h>

#include <cstring>
#include <memory>
#include <new>

#include "../../../include/vsl.h"
#include "engine.h"
#include "status.h"

struct vsl_engine {
    std::unique_ptr<vsl::DecodeEngine> impl;
};

using vsl::set_error;

#define GUARD_BEGIN try {
#define GUARD_END                                                                        \
    }                                                                                    \
    catch (const std::bad_alloc&) { return set_error(VSL_ERR_OOM, "host allocation failed"); } \
    catch (const std::exception& ex) { return set_error(VSL_ERR_STATE, "exception: %s", ex.what()); } \
    catch (...) { return set_error(VSL_ERR_STATE, "unknown exception"); }

extern "C" void vsl_engine_default_options(vsl_engine_options* o) {
    if (!o) return;
    memset(o, 0, sizeof(*o));
    o->device = 0;
    o->max_batch = 1;
    o->max_seq = 4096;
    o->kv_dtype = -1;
    o->page_size = 64;
    o->split_len = 0;
    o->tp_rank = 0;
    o->tp_size = 1;
    o->nccl_id = nullptr;
    o->vram_budget_gb = 0.0;
    o->use_graph = 1;
    o->use_pdl = 1;
    o->use_fused = 0;
    o->use_p2p = 1;
    o->legacy_q4 = 0;
    o->sparse_min_len = 0;  // dense attention at every length
    o->sparse_window = 512;
    o->sparse_global = 16;
    o->sparse_block = 1024;
    o->attn_route = 0;
    o->attn_prefetch = 0;  // 7B batch 1: 330.5 tok/s without, 325.4 with (the prefetch delays the
                           // attention kernel's own cache reads)
    o->p2p_chunk_bytes = 0;
    o->nccl_timeout_ms = 120000;
}

extern "C" int vsl_nccl_unique_id(void* out128) {
    if (!out128) return set_error(VSL_ERR_INVALID, "nccl_unique_id: null output");
    static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
    ncclUniqueId id;
    ncclResult_t r = ncclGetUniqueId(&id);
    if (r != ncclSuccess) return set_error(VSL_ERR_NCCL, "ncclGetUniqueId: %s", ncclGetErrorString(r));
    memcpy(out128, &id, sizeof(id));
    return VSL_OK;
}

static int check_engine(const vsl_engine* e) {
    if (!e || !e->impl) return set_error(VSL_ERR_INVALID, "null engine");
    return VSL_OK;
}

extern "C" int vsl_engine_create_gguf(const char* path, const vsl_engine_options* opt, vsl_engine** out) {
    GUARD_BEGIN
    if (!path || !out) return set_error(VSL_ERR_INVALID, "create_gguf: null argument");
    *out = nullptr;
    vsl_engine_options o;
    if (opt) o = *opt; else vsl_engine_default_options(&o);
    vk_symbiote::GGUFLoader loader(path);
    auto st = loader.load();
    if (!st) return set_error(st.error() == VSL_ERR_IO ? VSL_ERR_IO : VSL_ERR_FORMAT, "GGUF load of %s failed (%d)",
                              path, st.error());
    vsl_model_config cfg;
    int rc = vsl::make_model_config_from_gguf(loader, &cfg);
    if (rc) return rc;
    std::unique_ptr<vsl::DecodeEngine> eng;
    rc = vsl::DecodeEngine::create(cfg, o, eng);
    if (rc) return rc;
    rc = eng->load_gguf(loader);
    if (rc) return rc;
    rc = eng->reset();
    if (rc) return rc;
    *out = new vsl_engine{std::move(eng)};
    return VSL_OK;
    GUARD_END
}

extern "C" int vsl_engine_create_synthetic(const vsl_model_config* cfg, uint64_t seed, double sigma,
                                           const vsl_engine_options* opt, vsl_engine** out) {
    GUARD_BEGIN
    if (!cfg || !out) return set_error(VSL_ERR_INVALID, "create_synthetic: null argument");
    *out = nullptr;
    vsl_engine_options o;
    if (opt) o = *opt; else vsl_engine_default_options(&o);
    std::unique_ptr<vsl::DecodeEngine> eng;
    int rc = vsl::DecodeEngine::create(*cfg, o, eng);
    if (rc) return rc;
    rc = eng->init_synthetic(seed, sigma);
    if (rc) return rc;
    rc = eng->reset();
    if (rc) return rc;
    *out = new vsl_engine{std::move(eng)};
    return VSL_OK;
    GUARD_END
}

extern "C" int vsl_engine_destroy(vsl_engine* e) {
    GUARD_BEGIN
    delete e;
    return VSL_OK;
    GUARD_END
}

extern "C" int vsl_engine_get_config(const vsl_engine* e, vsl_model_config* out) {
    if (int rc = check_engine(e)) return rc;
    if (!out) return set_error(VSL_ERR_INVALID, "get_config: null output");
    *out = e->impl->config();
    return VSL_OK;
}

extern "C" int vsl_engine_reset(vsl_engine* e) {
    GUARD_BEGIN
    if (int rc = check_engine(e)) return rc;
    return e->impl->reset();
    GUARD_END
}

extern "C" int vsl_engine_fill_kv_synthetic(vsl_engine* e, uint64_t seed, double sigma, int n_pos, int B) {
    GUARD_BEGIN
    if (int rc = check_engine(e)) return rc;
    return e->impl->fill_kv_synthetic(seed, sigma, n_pos, B);
    GUARD_END
}

extern "C" int vsl_engine_set_forced(vsl_engine* e, const int32_t* ids, int n_steps, int B) {
    GUARD_BEGIN
    if (int rc = check_engine(e)) return rc;
    return e->impl->set_forced(ids, n_steps, B);
    GUARD_END
}

extern "C" int vsl_engine_run(vsl_engine* e, int n_steps, int B, float temperature, uint64_t seed) {
    GUARD_BEGIN
    if (int rc = check_engine(e)) return rc;
    return e->impl->run(n_steps, B, temperature, seed);
    GUARD_END
}

extern "C" int vsl_engine_step_host(vsl_engine* e, const int32_t* ids, int B, int32_t* out_ids, float* out_logits) {
    GUARD_BEGIN
    if (int rc = check_engine(e)) return rc;
    return e->impl->step_host(ids, B, out_ids, out_logits);
    GUARD_END
}

extern "C" int vsl_engine_read_tokens(vsl_engine* e, int n, int B, int32_t* out) {
    GUARD_BEGIN
    if (int rc = check_engine(e)) return rc;
    return e->impl->read_tokens(n, B, out);
    GUARD_END
}

extern "C" int vsl_engine_positions(vsl_engine* e, int B, int32_t* out) {
    GUARD_BEGIN
    if (int rc = check_engine(e)) return rc;
    return e->impl->positions(B, out);
    GUARD_END
}

extern "C" int vsl_engine_generate(vsl_engine* e, const int32_t* prompt, int n_prompt, int max_new, float temperature,
                                   uint64_t seed, const int32_t* stop_ids, int n_stop, int32_t* out_ids, int* n_out) {
    GUARD_BEGIN
    if (int rc = check_engine(e)) return rc;
    return e->impl->generate(prompt, n_prompt, max_new, temperature, seed, stop_ids, n_stop, out_ids, n_out);
    GUARD_END
}

extern "C" void* vsl_engine_stream(vsl_engine* e) {
    if (!e || !e->impl) return nullptr;
    return (void*)e->impl->stream();
}

extern "C" int vsl_engine_step_stats(vsl_engine* e, int B, int* kernels_per_step, double* bytes_per_step) {
    GUARD_BEGIN
    if (int rc = check_engine(e)) return rc;
    return e->impl->step_stats(B, kernels_per_step, bytes_per_step);
    GUARD_END
}

extern "C" int vsl_engine_device_status(vsl_engine* e, int* status) {
    GUARD_BEGIN
    if (int rc = check_engine(e)) return rc;
    if (!status) return set_error(VSL_ERR_INVALID, "device_status: null output");
    return e->impl->device_status(status);
    GUARD_END
}

extern "C" int vsl_engine_inject_status(vsl_engine* e, int code) {
    GUARD_BEGIN
    if (int rc = check_engine(e)) return rc;
    if (code > 0 || code < VSL_ERR_STATE) return set_error(VSL_ERR_INVALID, "inject_status: %d is not a status", code);
    return e->impl->inject_status(code);
    GUARD_END
}

extern "C" int vsl_gguf_model_config(const char* path, vsl_model_config* out) {
    GUARD_BEGIN
    if (!path || !out) return set_error(VSL_ERR_INVALID, "gguf_model_config: null argument");
    vk_symbiote::GGUFLoader loader(path);
    auto st = loader.load();
    if (!st) return set_error(st.error() == VSL_ERR_IO ? VSL_ERR_IO : VSL_ERR_FORMAT, "GGUF load of %s failed (%d)",
                              path, st.error());
    return vsl::make_model_config_from_gguf(loader, out);
    GUARD_END
}

extern "C" int vsl_gguf_tensor_info(const char* path, const char* name, int* ggml_type, uint64_t ne[4],
                                    uint64_t* file_offset) {
    GUARD_BEGIN
    if (!path || !name) return set_error(VSL_ERR_INVALID, "gguf_tensor_info: null argument");
    vk_symbiote::GGUFLoader loader(path);
    auto st = loader.load();
    if (!st) return set_error(st.error() == VSL_ERR_IO ? VSL_ERR_IO : VSL_ERR_FORMAT, "GGUF load of %s failed (%d)",
                              path, st.error());
    const vk_symbiote::GGUFTensorInfo* t = loader.get_tensor(name);
    if (!t) return set_error(VSL_ERR_INVALID, "gguf_tensor_info: no tensor named %s", name);
    if (ggml_type) *ggml_type = (int)t->data_type;
    if (ne)
        for (int i = 0; i < 4; i++) ne[i] = i < (int)t->dimensions.size() ? t->dimensions[i] : 0;
    if (file_offset) *file_offset = t->data_offset;
    return VSL_OK;
    GUARD_END
}

extern "C" int vsl_engine_memory_stats(vsl_engine* e, size_t* weight_bytes, size_t* kv_bytes, size_t* other_bytes) {
    if (int rc = check_engine(e)) return rc;
    if (weight_bytes) *weight_bytes = e->impl->arena_bytes();
    if (kv_bytes) *kv_bytes = e->impl->kv_bytes();
    if (other_bytes) *other_bytes = e->impl->other_bytes();
    return VSL_OK;
}

extern "C" int vsl_engine_prefill(vsl_engine* e, const int32_t* ids, int n, int seq, int32_t* next_id,
                                  float* logits) {
    GUARD_BEGIN
    if (int rc = check_engine(e)) return rc;
    return e->impl->prefill(ids, n, seq, next_id, logits);
    GUARD_END
}

extern "C" int vsl_engine_reset_seq(vsl_engine* e, int seq) {
    GUARD_BEGIN
    if (int rc = check_engine(e)) return rc;
    return e->impl->reset_seq(seq);
    GUARD_END
}

extern "C" int vsl_engine_generate_batch(vsl_engine* e, const int32_t* prompts, const int* lens, int n_seq,
                                         int max_new, float temperature, uint64_t seed, const int32_t* stop_ids,
                                         int n_stop, int32_t* out_ids, int* n_out) {
    GUARD_BEGIN
    if (int rc = check_engine(e)) return rc;
    return e->impl->generate_batch(prompts, lens, n_seq, max_new, temperature, seed, stop_ids, n_stop, out_ids, n_out);
    GUARD_END
}

extern "C" int vsl_engine_residency(vsl_engine* e, uint32_t* resident_layers, uint32_t* streamed_layers,
                                    uint64_t* streamed_bytes_per_step, uint64_t* host_bytes) {
    if (int rc = check_engine(e)) return rc;
    const vk_symbiote::PackResidency r = e->impl->residency();
    if (resident_layers) *resident_layers = r.resident_layers;
    if (streamed_layers) *streamed_layers = r.streamed_layers;
    if (streamed_bytes_per_step) *streamed_bytes_per_step = r.streamed_bytes_per_step;
    if (host_bytes) *host_bytes = r.streamed_bytes_per_step;  // one pinned copy of every streamed layer
    return VSL_OK;
}

extern "C" int vsl_pack_plan(uint64_t layer_bytes, uint32_t n_layers, uint64_t fixed_bytes, double budget_gb,
                             uint32_t* resident_layers, uint32_t* streamed_layers) {
    if (!resident_layers || !streamed_layers || budget_gb < 0)
        return set_error(VSL_ERR_INVALID, "pack_plan: null output or negative budget");
    const vk_symbiote::PackResidency r = vk_symbiote::NomadPackManager::plan(
        layer_bytes, n_layers, fixed_bytes, (uint64_t)(budget_gb > 0 ? budget_gb * 1e9 : 0));
    if (!r.feasible) return set_error(VSL_ERR_OOM, "pack_plan: budget below the fixed part plus two layer slots");
    *resident_layers = r.resident_layers;
    *streamed_layers = r.streamed_layers;
    return VSL_OK;
}

