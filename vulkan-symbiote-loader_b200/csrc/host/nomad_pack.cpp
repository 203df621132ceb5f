// Residency planner of the decoder layers under an HBM budget (include/vk_symbiote/NomadPack.h).
#include "../../../include/vk_symbiote/NomadPack.h"

namespace vk_symbiote {

PackResidency NomadPackManager::plan(uint64 layer_bytes, uint32 n_layers, uint64 fixed_bytes, uint64 budget_bytes) {
    PackResidency r;
    const uint64 all = fixed_bytes + layer_bytes * (uint64)n_layers;
    if (budget_bytes == 0 || all <= budget_bytes || n_layers == 0) {
        r.resident_layers = n_layers;
        r.resident_bytes = all;
        return r;
    }
    // two rotating slots: the layer being computed and the one being copied in
    const uint64 slots = 2 * layer_bytes;
    if (fixed_bytes + slots > budget_bytes) {
        r.feasible = false;
        return r;
    }
    uint64 fit = (budget_bytes - fixed_bytes - slots) / (layer_bytes ? layer_bytes : 1);
    if (fit >= n_layers) fit = n_layers - 1;  // cannot happen (all > budget), kept as a guard
    r.resident_layers = (uint32)fit;
    r.streamed_layers = n_layers - (uint32)fit;
    r.slot_bytes = layer_bytes;
    r.resident_bytes = fixed_bytes + layer_bytes * fit + slots;
    r.streamed_bytes_per_step = layer_bytes * (uint64)r.streamed_layers;
    return r;
}

}  // namespace vk_symbiote
