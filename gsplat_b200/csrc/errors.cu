// Error reporting for the C ABI (see include/gsplat_b200.h).
#include <cstring>

#include "common.cuh"
#include "gsb_internal.h"

namespace gsb {

static thread_local char g_last_error[512] = {0};

int set_error(int code, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return code;
}

int check_launch(const char *what) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(kErrLaunch, "%s: %s", what, cudaGetErrorString(e));
    return kOk;
}

} // namespace gsb

extern "C" const char *gsb_last_error(void) { return gsb::g_last_error; }

extern "C" int gsb_version(void) { return 1; }
