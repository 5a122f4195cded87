// Status reporting of the C ABI.
#include "common.cuh"

namespace decik {

static thread_local char g_last_error[512] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

}  // namespace decik

extern "C" const char* decik_last_error(void) { return decik::g_last_error; }

extern "C" int decik_abi_version(void) { return 1; }
