// Error reporting shared by every C-ABI entry point: a thread-local message plus the
// negative status code the call returns.
#pragma once
#include "../../../include/vsl.h"

namespace vsl {

// Record `code` with a printf-style message for vsl_last_error_string(); returns code.
int set_error(int code, const char* fmt, ...)
#if defined(__GNUC__)
    __attribute__((format(printf, 2, 3)))
#endif
    ;

void clear_error();

}  // namespace vsl
