// C-ABI plumbing shared by every entry point: the thread-local error message and the
// library version.
#include "common.cuh"

namespace mzb {

static thread_local char g_err[512] = {0};

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

}  // namespace mzb

extern "C" const char* mzb_last_error(void) { return mzb::g_err; }

extern "C" int mzb_version(void) { return MZB_VERSION; }
