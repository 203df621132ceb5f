// Device layout of GGUF block-quantized weights (Q8_0 and Q4_0, 32 elements per block), shared
// by the host (upload, sizing) and the kernels.
//
// GGUF stores a row of K elements as K/32 blocks of {fp16 scale d; quants} (34 bytes for Q8_0,
// 18 for Q4_0), which leaves the 16-bit scale in front of every block and the quants off the
// 16-byte alignment that vectorised loads need. Rows are repacked once at upload into
//   [quants: K bytes (Q8_0) or K/2 bytes (Q4_0)][scales: K/32 fp16, padded to 16 bytes]
// so a weight row is two aligned, contiguous streams. Quant order inside a block is ggml's:
// Q8_0 element i = int8 qs[i]; Q4_0 element i = low nibble of qs[i] - 8 and element i + 16 =
// high nibble of qs[i] - 8 (i < 16). Value = quant * d (GGUFLoader.cpp:1141-1181 dequantises
// the same way, q * scale in fp32).
#pragma once

#include <cstddef>

#include "../../../include/vsl.h"

#ifdef __CUDACC__
#define VSL_HD __host__ __device__ __forceinline__
#else
#define VSL_HD inline
#endif

namespace vsl {

constexpr int QBLK = 32;

VSL_HD bool is_quant(int dt) { return dt == VSL_Q8_0 || dt == VSL_Q4_0; }
// bytes of the quant part of a row of K elements
VSL_HD size_t quant_bytes(int dt, size_t K) { return dt == VSL_Q8_0 ? K : K / 2; }
// bytes of the scale part (K/32 fp16 values, padded to a 16-byte multiple)
VSL_HD size_t scale_bytes(size_t K) { return ((K / QBLK) * 2 + 15) / 16 * 16; }
// bytes of one weight row of K elements in device layout, any weight type
VSL_HD size_t weight_row_bytes(int dt, size_t K) {
    return is_quant(dt) ? quant_bytes(dt, K) + scale_bytes(K) : K * (dt == VSL_F32 ? 4 : 2);
}
// bytes of one GGUF block
VSL_HD size_t gguf_block_bytes(int dt) { return dt == VSL_Q8_0 ? 34 : 18; }

}  // namespace vsl
