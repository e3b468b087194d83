// Running screen-space statistics of the densification strategy: per Gaussian,
// the sum of its normalised 2D mean-gradient norms, the number of views it was
// visible in, and (optionally) its largest normalised screen radius. One pass
// over the visible (camera, Gaussian) pairs; reference
// gsplat/strategy/default.py:218-276 (DefaultStrategy._update_state), which
// does the same with clone, scale, norm, index_add_ x2 and an indexed
// maximum.
//
// grads: [n, 2] (packed pairs, or all C*N dense pairs), scaled by
// (width / 2 * n_cameras, height / 2 * n_cameras) before the norm. A dense pair
// counts when both radii are positive. Sums are float atomics (index_add_ is
// too); the radius maximum is an integer atomic on the non-negative float's
// bits, a true scatter maximum where the reference's indexed assignment keeps
// one of the duplicates of a Gaussian seen by several cameras.
#include "common.cuh"
#include "gsb_internal.h"

namespace gsb {

__global__ void __launch_bounds__(256) densify_accumulate_kernel(long long n, int N, const int64_t *__restrict__ gids,
                                                                 const float *__restrict__ grads,
                                                                 const int32_t *__restrict__ radii, float sx, float sy,
                                                                 float inv_max_wh, float *__restrict__ grad2d,
                                                                 float *__restrict__ count, float *__restrict__ max_radii) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int32_t rx = radii[i * 2], ry = radii[i * 2 + 1];
    long long g;
    if (gids != nullptr) {
        g = gids[i];
    } else {
        if (rx <= 0 || ry <= 0) return;
        g = i % N;
    }
    const float gx = grads[i * 2] * sx, gy = grads[i * 2 + 1] * sy;
    atomicAdd(grad2d + g, sqrtf(gx * gx + gy * gy));
    atomicAdd(count + g, 1.f);
    if (max_radii != nullptr) {
        const float r = (float)max(rx, ry) * inv_max_wh;
        atomicMax(reinterpret_cast<int *>(max_radii) + g, __float_as_int(fmaxf(r, 0.f)));
    }
}

} // namespace gsb

using namespace gsb;

extern "C" int gsb_densify_accumulate(long long n, int N, const int64_t *gaussian_ids, const float *grads,
                                      const int32_t *radii, int width, int height, int n_cameras, float *grad2d,
                                      float *count, float *max_radii, cudaStream_t stream) {
    if (n < 0 || N <= 0 || width <= 0 || height <= 0 || n_cameras <= 0)
        return set_error(kErrInvalidArgument, "bad sizes");
    if (n == 0) return kOk;
    const float sx = (float)width / 2.0f * (float)n_cameras;
    const float sy = (float)height / 2.0f * (float)n_cameras;
    const float inv = 1.f / (float)(width > height ? width : height);
    densify_accumulate_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(n, N, gaussian_ids, grads, radii, sx,
                                                                              sy, inv, grad2d, count, max_radii);
    return check_launch("densify_accumulate_kernel");
}
