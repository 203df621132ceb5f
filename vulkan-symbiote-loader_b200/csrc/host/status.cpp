#include "status.h"

#include <cstdarg>
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

}  // namespace vsl

extern "C" const char* vsl_last_error_string(void) { return vsl::g_msg; }

extern "C" int vsl_version(void) { return 1; }
