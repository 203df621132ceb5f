// Weight-pack metadata and the HBM streaming pack manager.
// Mirrors the parts of the reference's vk_symbiote/include/vk_symbiote/NomadPack.h that the
// decode path touches: PackType / MemoryTier / PackMetadata (:25-44) and the PackManager
// roles prefetch_packs / evict_until / get_vram_stats (:218-266). The Vulkan memory
// machinery (VMA buffers, timeline semaphores, multi-queue, defragmentation) is replaced
// by CUDA streams and events inside the engine: when a model exceeds the HBM budget, the
// layers that do not fit stay in pinned host memory and are copied into two rotating HBM
// slots on a side stream, one layer ahead of the compute stream.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "Common.h"

namespace vk_symbiote {

enum class PackType : uint8 {
    ATTENTION_Q = 0, ATTENTION_K = 1, ATTENTION_V = 2, ATTENTION_O = 3,
    FEED_FORWARD_GATE = 4, FEED_FORWARD_UP = 5, FEED_FORWARD_DOWN = 6,
    NORM_GAMMA = 7, NORM_BETA = 8, ROPE = 9, EMBEDDING = 10, HEAD = 11, UNKNOWN = 255
};

enum class MemoryTier : uint8 { VRAM_HOT = 0, RAM_WARM = 1, DISK_COLD = 2, UNLOADED = 3 };

struct PackMetadata {
    uint64 pack_id = 0;
    PackType type = PackType::UNKNOWN;
    uint32 layer_idx = 0, head_idx = 0, head_group_idx = 0;
    size_t compressed_size = 0, decompressed_size = 0;
    uint64 file_offset = 0;
    std::string tensor_name;
    float base_priority = 0.5f;
    uint32 alignment = 256;
    uint32 n_dimensions = 0;
    std::vector<uint64_t> dimensions;
};

// Residency plan of the engine's weights (what NomadPackManager decided at load time).
struct PackResidency {
    uint32 resident_layers = 0;   // layers kept in HBM (layers 0 .. resident_layers-1)
    uint32 streamed_layers = 0;   // layers copied from pinned host memory every step
    uint64 resident_bytes = 0;    // HBM for weights: resident layers, embeddings, lm_head, slots
    uint64 streamed_bytes_per_step = 0;
    uint64 slot_bytes = 0;        // size of one streaming slot (one layer), 0 when nothing streams
    bool feasible = true;         // false: the budget cannot hold the fixed part and two slots
};

// Decides which decoder layers stay in HBM (replaces the prefetch/evict policy of the
// reference's PackManager, NomadPack.cpp:1190-1249, and the engine's schedule_prefetch /
// evict_low_priority, VulkanSymbioteEngine.cpp:1555-1599). Decode visits every layer once per
// token in order, so recency/frequency scores carry no information here: the plan keeps the
// first layers resident, and the others stream through two rotating HBM slots, each copy
// overlapping the compute of the layer before it.
class VSL_CPP_API NomadPackManager {
public:
    // layer_bytes: one decoder layer's weights; fixed_bytes: everything else that must live in
    // HBM (KV cache, activations, workspaces, embeddings, lm_head, final norm); budget_bytes:
    // the cap (0 = none). Streaming engages only when the whole model does not fit.
    static PackResidency plan(uint64 layer_bytes, uint32 n_layers, uint64 fixed_bytes, uint64 budget_bytes);
};

}  // namespace vk_symbiote
