// FP32 FMA throughput probe: the denominator of the FP32-issue roofline reported
// for the rasterizer kernels (bench.py). Every thread runs 8 independent FMA
// chains of `iters` steps; FLOPs = blocks * threads * iters * 8 * 2.
#include "common.cuh"
#include "gsb_internal.h"

namespace gsb {

__global__ void fma_probe_kernel(float *out, int iters) {
    float a[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) a[j] = (float)(threadIdx.x + j) * 1e-3f;
    for (int i = 0; i < iters; ++i) {
#pragma unroll
        for (int j = 0; j < 8; ++j) a[j] = fmaf(a[j], 0.999999f, 1e-7f);
    }
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) s += a[j];
    out[(size_t)blockIdx.x * blockDim.x + threadIdx.x] = s;
}

} // namespace gsb

extern "C" int gsb_fp32_fma_probe(float *out, int blocks, int threads, int iters,
                                  cudaStream_t stream) {
    if (blocks <= 0 || threads <= 0 || threads > 1024 || iters <= 0)
        return gsb::set_error(gsb::kErrInvalidArgument, "bad probe launch shape");
    gsb::fma_probe_kernel<<<blocks, threads, 0, stream>>>(out, iters);
    return gsb::check_launch("fma_probe_kernel");
}
