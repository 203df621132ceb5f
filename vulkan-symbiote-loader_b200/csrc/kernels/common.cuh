// Shared device helpers for the sm_100a decode kernels.
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../../include/vsl.h"

namespace vsl {

// ---------------------------------------------------------------------------------------
// Programmatic dependent launch. A kernel launched with the programmatic-serialization
// attribute may start while its predecessor drains; it must call pdl_wait() before it
// reads anything the predecessor writes. Weights are never written by a predecessor, so
// weight streaming may begin before the wait.
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// 16-byte streaming load that bypasses L1 (weights are read exactly once per step).
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Weight element traits: how many elements one 16-byte vector holds and how to widen them.
template <typename T> struct WTraits;
template <> struct WTraits<float> {
    static constexpr int VEC = 4;
    __device__ __forceinline__ static void widen(const uint4& v, float* f) {
        f[0] = __uint_as_float(v.x); f[1] = __uint_as_float(v.y);
        f[2] = __uint_as_float(v.z); f[3] = __uint_as_float(v.w);
    }
    __device__ __forceinline__ static float load(const float* p, size_t i) { return p[i]; }
};
template <> struct WTraits<__half> {
    static constexpr int VEC = 8;
    __device__ __forceinline__ static void widen(const uint4& v, float* f) {
        const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            float2 t = __half22float2(h[i]);
            f[2 * i] = t.x; f[2 * i + 1] = t.y;
        }
    }
    __device__ __forceinline__ static float load(const __half* p, size_t i) { return __half2float(p[i]); }
};
template <> struct WTraits<__nv_bfloat16> {
    static constexpr int VEC = 8;
    __device__ __forceinline__ static void widen(const uint4& v, float* f) {
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            f[2 * i] = __uint_as_float(w[i] << 16);
            f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
        }
    }
    __device__ __forceinline__ static float load(const __nv_bfloat16* p, size_t i) { return __bfloat162float(p[i]); }
};

// KV cache element store/load (fp32 or fp16 storage, fp32 arithmetic).
__device__ __forceinline__ void kv_put(void* base, size_t i, float v, int kvdtype) {
    if (kvdtype == VSL_F16) reinterpret_cast<__half*>(base)[i] = __float2half_rn(v);
    else if (kvdtype == VSL_BF16) reinterpret_cast<__nv_bfloat16*>(base)[i] = __float2bfloat16_rn(v);
    else reinterpret_cast<float*>(base)[i] = v;
}

// Order-preserving map of a float to uint32 (larger float -> larger key; NaN excluded
// by the caller). Packed with the complement of the index so that a 64-bit max picks
// the largest value and, among equal values, the lowest index.
__device__ __forceinline__ uint32_t float_key(float f) {
    uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ unsigned long long pack_argmax(float v, uint32_t idx) {
    return ((unsigned long long)float_key(v) << 32) | (unsigned long long)(0xffffffffu - idx);
}
__device__ __forceinline__ uint32_t unpack_argmax_idx(unsigned long long p) {
    return 0xffffffffu - (uint32_t)(p & 0xffffffffu);
}

}  // namespace vsl
