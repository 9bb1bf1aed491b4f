// Error reporting for the C ABI: each entry point returns a status code and leaves a
// message for ssla_last_error() on the calling host thread.
#include "common.cuh"

namespace ssla {

static thread_local char g_last_error[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

const char* get_error() { return g_last_error; }

}  // namespace ssla

extern "C" int ssla_abi_version(void) { return 2; }
extern "C" const char* ssla_last_error(void) { return ssla::get_error(); }
