// Long-context sparse attention mask shared by the attention kernels and the engine.
#pragma once

#if defined(__CUDACC__)
#define VSL_SPARSE_HD __host__ __device__
#else
#define VSL_SPARSE_HD
#endif

namespace vsl {

// Long-context sparse attention mask of the reference (vk_symbiote/shaders/sparse_attention.comp:77-131),
// selected there when the sequence is longer than a threshold (use_sparse_attention && seq_len >
// 8192, VulkanSymbioteEngine.cpp:788; window 512, 16 global tokens, 1024-position blocks,
// vk_symbiote/include/vk_symbiote/Common.h:71-74). For a query at position pos of a sequence of
// pos + 1 tokens, the shader's index arithmetic selects one contiguous range [first, pos]:
//   get_attention_window: window_start = pos > W ? pos - W : 0; a query among the first G tokens
//     starts at 0, any other at min(G, window_start); the range ends at pos + 1;
//   compute_ring_attention: block_start = (pos / BLK) * BLK raises the start to block_start - W
//     when block_start > W; the end is cut at the block's end, which is never below pos + 1.
// min_len <= 0 is dense attention (first = 0).
struct SparseMask {
    int min_len, window, global_tokens, block;
};
VSL_SPARSE_HD inline int sparse_first(const SparseMask& m, int pos) {
    if (m.min_len <= 0 || pos + 1 <= m.min_len) return 0;
    const int ws = pos > m.window ? pos - m.window : 0;
    const int start = pos < m.global_tokens ? 0 : (m.global_tokens < ws ? m.global_tokens : ws);
    const int bs = (pos / m.block) * m.block;
    const int clamp = bs > m.window ? bs - m.window : 0;
    return start > clamp ? start : clamp;
}

}  // namespace vsl
