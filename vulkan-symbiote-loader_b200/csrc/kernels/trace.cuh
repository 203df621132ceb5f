// Per-CTA timeline of the decode step's kernels: entry, release from griddepcontrol.wait and exit
// of every CTA, stamped with %globaltimer. Compiled in only by the trace build (`make trace`,
// -DVSL_TRACE, lib/libvsl_trace.so); in libvsl.so every macro below expands to nothing.
//
// Each translation unit that includes this header keeps its own device record array (device
// symbols are per translation unit without relocatable device code) and exports a reader,
// vsl_trace_read_<unit>(out, cap, reset) -> records copied. A launch is identified by the id its
// host launcher draws from vsl_trace_next_id() (one counter for the whole library), so records
// of different units order into one timeline.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#ifdef VSL_TRACE

namespace vsl {

struct TraceRec {
    uint32_t id;    // launch id (host counter)
    uint32_t blk;   // blockIdx.x | blockIdx.y << 12 | blockIdx.z << 22
    uint32_t tag;   // kernel kind (see the launchers)
    uint32_t smid;
    uint64_t t0, t1, t2;  // entry, release from griddepcontrol.wait, exit (ns)
    uint64_t pad;
};
constexpr uint32_t TRACE_CAP = 1u << 20;

__device__ __forceinline__ uint64_t trace_now() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ uint32_t trace_smid() {
    uint32_t s;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(s));
    return s;
}

uint32_t trace_next_id();  // host: next launch id (trace build only)

}  // namespace vsl

// One record array per translation unit, plus its reader.
#define VSL_TRACE_UNIT(NAME)                                                                               \
    static __device__ vsl::TraceRec g_trace_rec[vsl::TRACE_CAP];                                           \
    static __device__ unsigned int g_trace_n;                                                              \
    static __device__ __forceinline__ void vsl_trace_record(uint32_t id, uint32_t tag, uint64_t t0, uint64_t t1) { \
        const uint64_t t2 = vsl::trace_now();                                                              \
        const unsigned i = atomicAdd(&g_trace_n, 1u);                                                      \
        if (i < vsl::TRACE_CAP) {                                                                          \
            vsl::TraceRec r;                                                                               \
            r.id = id;                                                                                     \
            r.blk = blockIdx.x | (blockIdx.y << 12) | (blockIdx.z << 22);                                 \
            r.tag = tag;                                                                                   \
            r.smid = vsl::trace_smid();                                                                    \
            r.t0 = t0;                                                                                     \
            r.t1 = t1;                                                                                     \
            r.t2 = t2;                                                                                     \
            r.pad = 0;                                                                                     \
            g_trace_rec[i] = r;                                                                            \
        }                                                                                                  \
    }                                                                                                      \
    extern "C" __attribute__((visibility("default"))) int vsl_trace_read_##NAME(void* out, unsigned cap,  \
                                                                               int reset) {              \
        unsigned n = 0;                                                                                    \
        if (cudaMemcpyFromSymbol(&n, g_trace_n, sizeof(n)) != cudaSuccess) return -1;                     \
        if (n > vsl::TRACE_CAP) n = vsl::TRACE_CAP;                                                        \
        if (n > cap) n = cap;                                                                              \
        if (out && n && cudaMemcpyFromSymbol(out, g_trace_rec, n * sizeof(vsl::TraceRec)) != cudaSuccess) \
            return -2;                                                                                     \
        if (reset) {                                                                                       \
            const unsigned z = 0;                                                                          \
            if (cudaMemcpyToSymbol(g_trace_n, &z, sizeof(z)) != cudaSuccess) return -3;                    \
        }                                                                                                  \
        return (int)n;                                                                                     \
    }
#define VSL_TRACE_ENTRY() const uint64_t vsl_tr0 = vsl::trace_now(); uint64_t vsl_tr1 = vsl_tr0
#define VSL_TRACE_RELEASED() vsl_tr1 = vsl::trace_now()
#define VSL_TRACE_EXIT(ID, TAG)                                      \
    do {                                                             \
        __syncthreads();                                             \
        if (threadIdx.x == 0) vsl_trace_record((ID), (TAG), vsl_tr0, vsl_tr1); \
    } while (0)
#define VSL_TRACE_ID() vsl::trace_next_id()

#else

#define VSL_TRACE_UNIT(NAME)
#define VSL_TRACE_ENTRY() \
    do {                  \
    } while (0)
#define VSL_TRACE_RELEASED() \
    do {                     \
    } while (0)
#define VSL_TRACE_EXIT(ID, TAG) \
    do {                        \
    } while (0)
#define VSL_TRACE_ID() 0u

#endif
