// Device layout of GGUF block-quantized weights (Q8_0, Q4_0 and Q4_1, 32 elements per block),
// shared by the host (upload, sizing) and the kernels.
//
// GGUF stores a row of K elements as K/32 blocks of {fp16 scale d; [fp16 minimum m;] quants}
// (34 bytes for Q8_0, 18 for Q4_0, 20 for Q4_1), which leaves 16-bit values in front of every
// block and the quants off the 16-byte alignment that vectorised loads need. Rows are repacked
// once at upload into
//   [quants: K bytes (Q8_0) or K/2 bytes (Q4_x)][scales: K/32 fp16, padded to 16 bytes]
//   [Q4_1 only: minimums: K/32 fp16, padded to 16 bytes]
// so a weight row is two or three aligned, contiguous streams. Quant order inside a block is
// ggml's: Q8_0 element i = int8 qs[i]; Q4_x element i = low nibble of qs[i] and element i + 16 =
// high nibble of qs[i] (i < 16). Value = int8 * d (Q8_0), (nibble - 8) * d (Q4_0), nibble * d + m
// (Q4_1) (GGUFLoader.cpp:1150-1207 dequantises the same way in fp32).
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

VSL_HD bool is_quant(int dt) { return dt == VSL_Q8_0 || dt == VSL_Q4_0 || dt == VSL_Q4_1; }
// whether blocks carry a minimum (value = nibble * d + m)
VSL_HD bool has_min(int dt) { return dt == VSL_Q4_1; }
// bytes of the quant part of a row of K elements
VSL_HD size_t quant_bytes(int dt, size_t K) { return dt == VSL_Q8_0 ? K : K / 2; }
// bytes of the scale part (K/32 fp16 values, padded to a 16-byte multiple); the minimums of a
// Q4_1 row take the same room after the scales
VSL_HD size_t scale_bytes(size_t K) { return ((K / QBLK) * 2 + 15) / 16 * 16; }
// bytes of one weight row of K elements in device layout, any weight type
VSL_HD size_t weight_row_bytes(int dt, size_t K) {
    return is_quant(dt) ? quant_bytes(dt, K) + scale_bytes(K) * (has_min(dt) ? 2 : 1) : K * (dt == VSL_F32 ? 4 : 2);
}
// bytes of one GGUF block
VSL_HD size_t gguf_block_bytes(int dt) { return dt == VSL_Q8_0 ? 34 : dt == VSL_Q4_1 ? 20 : 18; }

}  // namespace vsl
