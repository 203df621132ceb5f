// Tensor map of a paged fp16 KV cache for TMA (attention_tc.cu).
#pragma once
#include <cuda.h>

namespace vsl {

// KV cache [rows = n_pages * n_kv * page_size][128] fp16 as 64-row x 64-column boxes with the
// 128-byte swizzle (one box = one 64-position piece of a page, half of the head dims).
int kv_tensor_map(CUtensorMap* m, const void* base, long long rows);

}  // namespace vsl
