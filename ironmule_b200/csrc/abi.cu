// ABI bookkeeping: version and thread-local error messages.
#include <stdarg.h>
#include <string.h>

#include "common.cuh"
#include "../../include/imspec.h"

namespace im {

static thread_local char g_error[512];

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_error, sizeof(g_error), fmt, ap);
  va_end(ap);
}

void clear_error() { g_error[0] = '\0'; }

}  // namespace im

extern "C" int im_abi_version(void) { return IM_ABI_VERSION; }

extern "C" int im_set_launch_overlap(int on) {
  const int was = im::launch_overlap() ? 1 : 0;
  im::launch_overlap() = on != 0;
  return was;
}

extern "C" const char* im_last_error(void) { return im::g_error; }
