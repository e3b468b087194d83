// Host-side helpers shared by the C-ABI entry points: error reporting and
// launch checking. Errors are returned as negative status codes; the message of
// the most recent error on the calling thread is kept for gsb_last_error().
#pragma once

#include <cstdarg>
#include <cstdio>
#include <cuda_runtime.h>

#include "gsplat_b200.h"

namespace gsb {

int set_error(int code, const char *fmt, ...);

// Returns kOk, or kErrLaunch with the CUDA error string of the last launch.
int check_launch(const char *what);

} // namespace gsb
