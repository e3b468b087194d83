// Spherical-harmonic colour evaluation, forward and backward.
//
// Reference behaviour: gsplat/cuda/csrc/SphericalHarmonicsCUDA.cu:391-502 (one
// thread per element and channel there). Here one thread owns one element (all
// three channels share the basis evaluation) and the block stages its slice of
// the [n, K, 3] coefficient array through shared memory so that HBM is read and
// written with unit-stride, fully coalesced accesses.
#include "common.cuh"
#include "gsb_internal.h"
#include "sh_basis.cuh"

namespace gsb {

constexpr int kShThreads = 128;

// Copies `count` floats between global and shared memory cooperatively.
__device__ __forceinline__ void block_copy_in(float *dst, const float *src, size_t count) {
    for (size_t i = threadIdx.x; i < count; i += blockDim.x) dst[i] = src[i];
}
__device__ __forceinline__ void block_copy_out(float *dst, const float *src, size_t count) {
    for (size_t i = threadIdx.x; i < count; i += blockDim.x) dst[i] = src[i];
}

template <int D>
__global__ void __launch_bounds__(kShThreads)
    sh_fwd_kernel(uint32_t n, uint32_t K, const float *__restrict__ dirs,
                  const float *__restrict__ coeffs, const bool *__restrict__ masks,
                  float *__restrict__ colors) {
    extern __shared__ float smem[];
    const size_t first = (size_t)blockIdx.x * kShThreads;
    const uint32_t count = (uint32_t)min((size_t)kShThreads, n - first);
    constexpr int NB = (D + 1) * (D + 1);
    // Only the first NB basis rows of each element are needed.
    float *sc = smem; // [count, K, 3]
    block_copy_in(sc, coeffs + first * K * 3, (size_t)count * K * 3);
    __syncthreads();
    const uint32_t t = threadIdx.x;
    if (t >= count) return;
    const size_t e = first + t;
    float out[3] = {0.f, 0.f, 0.f};
    if (masks == nullptr || masks[e]) {
        float x = dirs[e * 3], y = dirs[e * 3 + 1], z = dirs[e * 3 + 2];
        const float inv = rsqrtf(x * x + y * y + z * z);
        x *= inv;
        y *= inv;
        z *= inv;
        float Y[NB];
        sh_eval<D>(x, y, z, Y);
        const float *cf = sc + (size_t)t * K * 3;
#pragma unroll
        for (int k = 0; k < NB; ++k) {
            out[0] += Y[k] * cf[k * 3 + 0];
            out[1] += Y[k] * cf[k * 3 + 1];
            out[2] += Y[k] * cf[k * 3 + 2];
        }
    }
    colors[e * 3 + 0] = out[0];
    colors[e * 3 + 1] = out[1];
    colors[e * 3 + 2] = out[2];
}

template <int D>
__global__ void __launch_bounds__(kShThreads)
    sh_bwd_kernel(uint32_t n, uint32_t K, const float *__restrict__ dirs,
                  const float *__restrict__ coeffs, const bool *__restrict__ masks,
                  const float *__restrict__ v_colors, float *__restrict__ v_coeffs,
                  float *__restrict__ v_dirs) {
    extern __shared__ float smem[];
    const size_t first = (size_t)blockIdx.x * kShThreads;
    const uint32_t count = (uint32_t)min((size_t)kShThreads, n - first);
    constexpr int NB = (D + 1) * (D + 1);
    float *sc = smem; // [count, K, 3]: coefficients in, then coefficient gradients out
    if (v_dirs != nullptr) block_copy_in(sc, coeffs + first * K * 3, (size_t)count * K * 3);
    __syncthreads();
    const uint32_t t = threadIdx.x;
    float vd[3] = {0.f, 0.f, 0.f};
    float Y[NB];
    float vc[3] = {0.f, 0.f, 0.f};
    bool active = false;
    float x = 0.f, y = 0.f, z = 0.f, inv = 0.f;
    if (t < count) {
        const size_t e = first + t;
        active = masks == nullptr || masks[e];
        if (active) {
            x = dirs[e * 3];
            y = dirs[e * 3 + 1];
            z = dirs[e * 3 + 2];
            inv = rsqrtf(x * x + y * y + z * z);
            x *= inv;
            y *= inv;
            z *= inv;
            sh_eval<D>(x, y, z, Y);
            vc[0] = v_colors[e * 3];
            vc[1] = v_colors[e * 3 + 1];
            vc[2] = v_colors[e * 3 + 2];
            if (v_dirs != nullptr && D > 0) {
                float w[NB];
                const float *cf = sc + (size_t)t * K * 3;
#pragma unroll
                for (int k = 0; k < NB; ++k)
                    w[k] = cf[k * 3] * vc[0] + cf[k * 3 + 1] * vc[1] + cf[k * 3 + 2] * vc[2];
                float gn[3];
                sh_grad_dot<D>(x, y, z, w, gn);
                const float d = gn[0] * x + gn[1] * y + gn[2] * z;
                vd[0] = (gn[0] - d * x) * inv;
                vd[1] = (gn[1] - d * y) * inv;
                vd[2] = (gn[2] - d * z) * inv;
            }
        }
    }
    __syncthreads();
    if (t < count) {
        float *vcf = sc + (size_t)t * K * 3;
#pragma unroll
        for (int k = 0; k < NB; ++k) {
            const float yk = active ? Y[k] : 0.f;
            vcf[k * 3 + 0] = yk * vc[0];
            vcf[k * 3 + 1] = yk * vc[1];
            vcf[k * 3 + 2] = yk * vc[2];
        }
        for (uint32_t k = NB; k < K; ++k) {
            vcf[k * 3 + 0] = 0.f;
            vcf[k * 3 + 1] = 0.f;
            vcf[k * 3 + 2] = 0.f;
        }
        if (v_dirs != nullptr) {
            const size_t e = first + t;
            v_dirs[e * 3 + 0] = vd[0];
            v_dirs[e * 3 + 1] = vd[1];
            v_dirs[e * 3 + 2] = vd[2];
        }
    }
    __syncthreads();
    block_copy_out(v_coeffs + first * K * 3, sc, (size_t)count * K * 3);
}

template <int D>
static void launch_sh_fwd(uint32_t n, uint32_t K, const float *dirs, const float *coeffs,
                          const bool *masks, float *colors, cudaStream_t s) {
    const size_t smem = (size_t)kShThreads * K * 3 * sizeof(float);
    if (smem > 48 * 1024)
        cudaFuncSetAttribute(sh_fwd_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    sh_fwd_kernel<D><<<(n + kShThreads - 1) / kShThreads, kShThreads, smem, s>>>(n, K, dirs, coeffs,
                                                                               masks, colors);
}

template <int D>
static void launch_sh_bwd(uint32_t n, uint32_t K, const float *dirs, const float *coeffs,
                          const bool *masks, const float *v_colors, float *v_coeffs,
                          float *v_dirs, cudaStream_t s) {
    const size_t smem = (size_t)kShThreads * K * 3 * sizeof(float);
    if (smem > 48 * 1024)
        cudaFuncSetAttribute(sh_bwd_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    sh_bwd_kernel<D><<<(n + kShThreads - 1) / kShThreads, kShThreads, smem, s>>>(
        n, K, dirs, coeffs, masks, v_colors, v_coeffs, v_dirs);
}

} // namespace gsb

using namespace gsb;

extern "C" int gsb_spherical_harmonics_fwd(int degree, long long n, int K, const float *dirs,
                                           const float *coeffs, const bool *masks, float *colors,
                                           cudaStream_t stream) {
    if (degree < 0 || degree > 4)
        return set_error(kErrUnsupported, "spherical harmonics degree %d not in [0, 4]", degree);
    if ((degree + 1) * (degree + 1) > K)
        return set_error(kErrInvalidArgument, "K=%d coefficients is too few for degree %d", K, degree);
    if (K > 64) return set_error(kErrUnsupported, "K=%d coefficients per element exceeds 64", K);
    if (n <= 0) return kOk;
    switch (degree) {
    case 0: launch_sh_fwd<0>(n, K, dirs, coeffs, masks, colors, stream); break;
    case 1: launch_sh_fwd<1>(n, K, dirs, coeffs, masks, colors, stream); break;
    case 2: launch_sh_fwd<2>(n, K, dirs, coeffs, masks, colors, stream); break;
    case 3: launch_sh_fwd<3>(n, K, dirs, coeffs, masks, colors, stream); break;
    default: launch_sh_fwd<4>(n, K, dirs, coeffs, masks, colors, stream); break;
    }
    return check_launch("sh_fwd_kernel");
}

extern "C" int gsb_spherical_harmonics_bwd(int degree, long long n, int K, const float *dirs,
                                           const float *coeffs, const bool *masks,
                                           const float *v_colors, float *v_coeffs, float *v_dirs,
                                           cudaStream_t stream) {
    if (degree < 0 || degree > 4)
        return set_error(kErrUnsupported, "spherical harmonics degree %d not in [0, 4]", degree);
    if ((degree + 1) * (degree + 1) > K)
        return set_error(kErrInvalidArgument, "K=%d coefficients is too few for degree %d", K, degree);
    if (K > 64) return set_error(kErrUnsupported, "K=%d coefficients per element exceeds 64", K);
    if (n <= 0) return kOk;
    switch (degree) {
    case 0: launch_sh_bwd<0>(n, K, dirs, coeffs, masks, v_colors, v_coeffs, v_dirs, stream); break;
    case 1: launch_sh_bwd<1>(n, K, dirs, coeffs, masks, v_colors, v_coeffs, v_dirs, stream); break;
    case 2: launch_sh_bwd<2>(n, K, dirs, coeffs, masks, v_colors, v_coeffs, v_dirs, stream); break;
    case 3: launch_sh_bwd<3>(n, K, dirs, coeffs, masks, v_colors, v_coeffs, v_dirs, stream); break;
    default: launch_sh_bwd<4>(n, K, dirs, coeffs, masks, v_colors, v_coeffs, v_dirs, stream); break;
    }
    return check_launch("sh_bwd_kernel");
}
