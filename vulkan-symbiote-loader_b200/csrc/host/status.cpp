#include "status.h"

#include <atomic>
#include <cstdarg>
#include <cstdint>
#include <cstdio>

namespace vsl {

static thread_local char g_msg[512] = "";

int set_error(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_msg, sizeof g_msg, fmt, ap);
    va_end(ap);
    return code;
}

void clear_error() { g_msg[0] = 0; }

#ifdef VSL_TRACE
// Launch ids of the trace build's per-CTA timeline (csrc/kernels/trace.cuh).
uint32_t trace_next_id() {
    static std::atomic<uint32_t> n{0};
    return ++n;
}
#endif

}  // namespace vsl

extern "C" const char* vsl_last_error_string(void) { return vsl::g_msg; }

extern "C" int vsl_version(void) { return 1; }
