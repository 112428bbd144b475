// Version and error reporting of the C ABI (pure host code).
#include <stdarg.h>
#include <stdio.h>

#include "ps_common.cuh"

namespace ps {

static thread_local char g_message[1024];

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_message, sizeof(g_message), fmt, ap);
  va_end(ap);
  return code;
}

void clear_error() { g_message[0] = '\0'; }

}  // namespace ps

extern "C" int32_t ps_abi_version(void) { return PS_ABI_VERSION; }

extern "C" const char* ps_error_message(void) { return ps::g_message; }
