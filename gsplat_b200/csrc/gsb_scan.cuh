// Device prefix-sum entry used by several host pipelines (see scan.cu).
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace gsb {

size_t scan_scratch_bytes(size_t n);

// out[i] = in[0] + ... + in[i] (int64). `scratch` must hold scan_scratch_bytes(n).
int inclusive_scan_i32_i64(const int32_t *in, int64_t *out, size_t n, void *scratch,
                           size_t scratch_bytes, cudaStream_t stream);

} // namespace gsb
