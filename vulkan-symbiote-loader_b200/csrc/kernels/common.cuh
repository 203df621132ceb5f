// Shared device helpers for the sm_100a decode kernels.
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../../include/vsl.h"
#include "sparse_mask.h"

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

// ---------------------------------------------------------------------------------------
// Bulk asynchronous copies (TMA, non-tensor form) and mbarriers.
// Every wait is bounded by wall time (%globaltimer): on expiry the caller records
// VSL_ERR_TIMEOUT in a status word and stops, instead of spinning forever.
// ---------------------------------------------------------------------------------------
constexpr unsigned long long WAIT_LIMIT_NS = 1000000000ull;  // one second

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
// System-scope acquire load / release store (flags exchanged with peer GPUs over NVLink)
__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                     smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// try_wait that may suspend the thread up to `hint_ns` while the phase is incomplete
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}
// Wait for the phase with the given parity to complete; false after WAIT_LIMIT_NS.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = globaltimer_ns();
    while (true) {
        for (int i = 0; i < 64; i++)
            if (mbar_try_wait(bar, parity)) return true;
        if (globaltimer_ns() - t0 > WAIT_LIMIT_NS) return false;
    }
}
// global -> shared bulk copy completing on `bar` (bytes % 16 == 0, both addresses 16-aligned)
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst_smem)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
// bring [src, src+bytes) into L2 without waiting (bytes % 16 == 0)
__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
// Request share `part` of `nparts` of [base, base+bytes) into L2, split among `nlanes`
// callers (caller `lane_id` issues every nlanes-th 16 KB piece).
__device__ __forceinline__ void prefetch_share(const void* base, size_t bytes, int part, int nparts, int lane_id,
                                               int nlanes) {
    const size_t lo = (bytes * (size_t)part / (size_t)nparts) & ~(size_t)15;
    const size_t hi = (bytes * (size_t)(part + 1) / (size_t)nparts) & ~(size_t)15;
    const char* b = reinterpret_cast<const char*>(base);
    for (size_t off = lo + (size_t)lane_id * 16384; off < hi; off += (size_t)nlanes * 16384)
        prefetch_l2(b + off, (uint32_t)(hi - off < 16384 ? hi - off : 16384));
}

__device__ __forceinline__ void named_barrier_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
// Named barrier that also ORs a predicate over the participating threads: every thread gets
// true if any of them passed true. Threads that must leave a loop together (for example after
// a timed-out wait) decide with this, so none is left waiting at a later bar.sync.
__device__ __forceinline__ bool named_barrier_or(int id, int threads, bool pred) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbarrier.red.or.pred q, %2, %3, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)pred), "r"(id), "r"(threads)
        : "memory");
    return r != 0;
}
__device__ __forceinline__ void set_status(int* status, int code) {
    if (status) atomicCAS(status, 0, code);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Maximum over the 32 lanes of a warp in one instruction (sm_100a's redux.sync on f32; like
// fmaxf, a NaN lane does not win over a number).
__device__ __forceinline__ float warp_max_redux(float v) {
    float r;
    asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(v));
    return r;
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
