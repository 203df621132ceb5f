// GGUF block-quantized rows -> the device row layout of kernels/quant_layout.h (host side,
// once per tensor at upload). GGUF block: fp16 scale d, then (Q4_1 only) fp16 minimum m, then
// 32 int8 quants (Q8_0) or 16 bytes of nibbles (Q4_0 / Q4_1); the reference reads the same
// blocks in GGUFLoader.cpp:1150-1207.
#include <cstring>

#include "kernels.h"
#include "status.h"
#include "vsl.h"

namespace vsl {

int repack_gguf_rows(int dtype, const void* blocks, size_t cols, size_t row0, size_t nrows, size_t col0, size_t ncols,
                     void* out, size_t out_ld, int legacy_q4) {
    if (!is_quant(dtype)) return set_error(VSL_ERR_UNSUPPORTED, "repack: dtype %d is not block-quantized", dtype);
    if (!blocks || !out || cols % QBLK || col0 % QBLK || ncols % QBLK || col0 + ncols > cols ||
        out_ld < weight_row_bytes(dtype, ncols))
        return set_error(VSL_ERR_INVALID, "repack: bad slice (cols %zu, col0 %zu, ncols %zu, pitch %zu)", cols, col0,
                         ncols, out_ld);
    const size_t bb = gguf_block_bytes(dtype), bpr = cols / QBLK, nblk = ncols / QBLK;
    const size_t qb = quant_bytes(dtype, ncols), sb = scale_bytes(ncols);
    const size_t hb = has_min(dtype) ? 4 : 2;  // block header: d (and m)
    for (size_t r = 0; r < nrows; r++) {
        const unsigned char* src = static_cast<const unsigned char*>(blocks) + ((row0 + r) * bpr + col0 / QBLK) * bb;
        unsigned char* dst = static_cast<unsigned char*>(out) + r * out_ld;
        unsigned char* scales = dst + qb;
        unsigned char* mins = scales + sb;
        memset(scales, 0, has_min(dtype) ? 2 * sb : sb);
        for (size_t k = 0; k < nblk; k++) {
            const unsigned char* blk = src + k * bb;
            memcpy(scales + 2 * k, blk, 2);                   // fp16 d, little-endian
            if (has_min(dtype)) memcpy(mins + 2 * k, blk + 2, 2);  // fp16 m
            const unsigned char* qs = blk + hb;
            if (dtype == VSL_Q8_0) {
                memcpy(dst + k * QBLK, qs, QBLK);
            } else if (!legacy_q4) {
                memcpy(dst + k * 16, qs, 16);  // ggml order is the device order
            } else {
                // reference order: element 2i = low nibble, 2i + 1 = high nibble of byte i
                unsigned char n[QBLK];
                for (int i = 0; i < 16; i++) {
                    n[2 * i] = qs[i] & 15;
                    n[2 * i + 1] = qs[i] >> 4;
                }
                for (int i = 0; i < 16; i++) dst[k * 16 + i] = (unsigned char)(n[i] | (n[i + 16] << 4));
            }
        }
    }
    return VSL_OK;
}

}  // namespace vsl

extern "C" int vsl_weight_row_bytes(int dtype, int K, size_t* bytes) {
    using namespace vsl;
    if (!bytes || K <= 0) return set_error(VSL_ERR_INVALID, "weight_row_bytes: bad arguments");
    if (dtype != VSL_F32 && dtype != VSL_F16 && dtype != VSL_BF16 && !is_quant(dtype))
        return set_error(VSL_ERR_UNSUPPORTED, "weight_row_bytes: dtype %d", dtype);
    if (is_quant(dtype) && K % QBLK) return set_error(VSL_ERR_INVALID, "weight_row_bytes: K %% 32 != 0");
    *bytes = weight_row_bytes(dtype, (size_t)K);
    return VSL_OK;
}

extern "C" int vsl_repack_gguf_rows(int dtype, const void* blocks, size_t cols, size_t row0, size_t nrows, size_t col0,
                                    size_t ncols, void* out, size_t out_ld, int legacy_q4) {
    return vsl::repack_gguf_rows(dtype, blocks, cols, row0, nrows, col0, ncols, out, out_ld, legacy_q4);
}
