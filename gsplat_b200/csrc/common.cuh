// Shared device-side definitions for the gsplat_b200 kernels (sm_100a).
//
// Constants follow the reference fork's values (gsplat/cuda/include/Common.h:73-93,
// gsplat/cuda/_constants.py:16-29); the small linear-algebra helpers below replace
// glm and use plain row-major float arrays: M[r][c] is row r, column c.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "detmath.h"

namespace gsb {

constexpr float kAlphaThreshold = 1.f / 255.f;   // Common.h:74
constexpr float kGaussianExtend = 3.33f;         // Common.h:76
constexpr float kMaxAlpha = 0.99f;               // Common.h:82
constexpr float kTransmittanceThreshold = 1e-4f; // Common.h:83
constexpr float kMinCompensation = 0.005f;       // Common.h:89
constexpr float kMinOneMinusAlpha = 1e-6f;       // Common.h:93

enum CameraModel : int { kPinhole = 0, kOrtho = 1, kFisheye = 2 };

// Error codes returned through the C ABI (0 = success).
enum Status : int {
    kOk = 0,
    kErrInvalidArgument = -1,
    kErrUnsupported = -2,
    kErrLaunch = -3,
};

struct M3 {
    float m[3][3];
};
struct M2 {
    float m[2][2];
};

__host__ __device__ inline M3 m3_zero() {
    M3 r;
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j) r.m[i][j] = 0.f;
    return r;
}

__host__ __device__ inline M3 m3_mul(const M3 &a, const M3 &b) {
    M3 r;
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j)
            r.m[i][j] = a.m[i][0] * b.m[0][j] + a.m[i][1] * b.m[1][j] + a.m[i][2] * b.m[2][j];
    return r;
}

// a * b^T
__host__ __device__ inline M3 m3_mul_bt(const M3 &a, const M3 &b) {
    M3 r;
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j)
            r.m[i][j] = a.m[i][0] * b.m[j][0] + a.m[i][1] * b.m[j][1] + a.m[i][2] * b.m[j][2];
    return r;
}

// a^T * b
__host__ __device__ inline M3 m3_mul_at(const M3 &a, const M3 &b) {
    M3 r;
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j)
            r.m[i][j] = a.m[0][i] * b.m[0][j] + a.m[1][i] * b.m[1][j] + a.m[2][i] * b.m[2][j];
    return r;
}

__host__ __device__ inline M3 m3_add(const M3 &a, const M3 &b) {
    M3 r;
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j) r.m[i][j] = a.m[i][j] + b.m[i][j];
    return r;
}

__host__ __device__ inline M3 m3_transpose(const M3 &a) {
    M3 r;
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j) r.m[i][j] = a.m[j][i];
    return r;
}

// Rotation matrix of the normalised quaternion (w, x, y, z); follows
// gsplat/cuda/include/Utils.cuh:174-196 (written here in row-major form).
__device__ inline M3 quat_to_rotmat(float w, float x, float y, float z) {
    const float inv = 1.f / sqrtf(w * w + x * x + y * y + z * z);
    w *= inv;
    x *= inv;
    y *= inv;
    z *= inv;
    M3 R;
    R.m[0][0] = 1.f - 2.f * (y * y + z * z);
    R.m[0][1] = 2.f * (x * y - w * z);
    R.m[0][2] = 2.f * (x * z + w * y);
    R.m[1][0] = 2.f * (x * y + w * z);
    R.m[1][1] = 1.f - 2.f * (x * x + z * z);
    R.m[1][2] = 2.f * (y * z - w * x);
    R.m[2][0] = 2.f * (x * z - w * y);
    R.m[2][1] = 2.f * (y * z + w * x);
    R.m[2][2] = 1.f - 2.f * (x * x + y * y);
    return R;
}

// Gradient of quat_to_rotmat with respect to the unnormalised quaternion,
// given G = dL/dR (row-major). Same result as Utils.cuh:198-221.
__device__ inline void quat_to_rotmat_vjp(const float q[4], const M3 &G, float v_q[4]) {
    const float inv = 1.f / sqrtf(q[0] * q[0] + q[1] * q[1] + q[2] * q[2] + q[3] * q[3]);
    const float w = q[0] * inv, x = q[1] * inv, y = q[2] * inv, z = q[3] * inv;
    const float g[3][3] = {{G.m[0][0], G.m[0][1], G.m[0][2]},
                           {G.m[1][0], G.m[1][1], G.m[1][2]},
                           {G.m[2][0], G.m[2][1], G.m[2][2]}};
    float vn[4];
    vn[0] = 2.f * (x * (g[2][1] - g[1][2]) + y * (g[0][2] - g[2][0]) + z * (g[1][0] - g[0][1]));
    vn[1] = 2.f * (-2.f * x * (g[1][1] + g[2][2]) + y * (g[0][1] + g[1][0]) +
                   z * (g[0][2] + g[2][0]) + w * (g[2][1] - g[1][2]));
    vn[2] = 2.f * (x * (g[0][1] + g[1][0]) - 2.f * y * (g[0][0] + g[2][2]) +
                   z * (g[1][2] + g[2][1]) + w * (g[0][2] - g[2][0]));
    vn[3] = 2.f * (x * (g[0][2] + g[2][0]) + y * (g[1][2] + g[2][1]) -
                   2.f * z * (g[0][0] + g[1][1]) + w * (g[1][0] - g[0][1]));
    const float d = vn[0] * w + vn[1] * x + vn[2] * y + vn[3] * z;
    v_q[0] += (vn[0] - d * w) * inv;
    v_q[1] += (vn[1] - d * x) * inv;
    v_q[2] += (vn[2] - d * y) * inv;
    v_q[3] += (vn[3] - d * z) * inv;
}

// Sigma = (R S)(R S)^T with S = diag(scale); Utils.cuh:223-237.
__device__ inline M3 covar_from_quat_scale(const float q[4], const float s[3], M3 *rot_out) {
    M3 R = quat_to_rotmat(q[0], q[1], q[2], q[3]);
    if (rot_out) *rot_out = R;
    M3 M;
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j) M.m[i][j] = R.m[i][j] * s[j];
    return m3_mul_bt(M, M);
}

// Back-propagates dL/dSigma into the quaternion and scale; Utils.cuh:259-296.
__device__ inline void covar_from_quat_scale_vjp(const float q[4], const float s[3], const M3 &R,
                                                 const M3 &v_sigma, float v_q[4], float v_s[3]) {
    M3 M;
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j) M.m[i][j] = R.m[i][j] * s[j];
    // d(M M^T): v_M = (G + G^T) M
    M3 vsym = m3_add(v_sigma, m3_transpose(v_sigma));
    M3 vM = m3_mul(vsym, M);
    M3 vR;
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j) vR.m[i][j] = vM.m[i][j] * s[j];
    quat_to_rotmat_vjp(q, vR, v_q);
#pragma unroll
    for (int j = 0; j < 3; ++j)
        v_s[j] += R.m[0][j] * vM.m[0][j] + R.m[1][j] * vM.m[1][j] + R.m[2][j] * vM.m[2][j];
}

// Pinhole EWA projection of a camera-space Gaussian with the 1.3x FOV clamp on the
// Jacobian; Utils.cuh:542-581.
struct PinholeJ {
    float j00, j02, j11, j12; // J = [[j00, 0, j02], [0, j11, j12]]
};

__device__ inline void persp_limits(float fx, float fy, float cx, float cy, uint32_t W, uint32_t H,
                                    float &lxp, float &lxn, float &lyp, float &lyn) {
    const float tfx = 0.5f * (float)W / fx;
    const float tfy = 0.5f * (float)H / fy;
    lxp = ((float)W - cx) / fx + 0.3f * tfx;
    lxn = cx / fx + 0.3f * tfx;
    lyp = ((float)H - cy) / fy + 0.3f * tfy;
    lyn = cy / fy + 0.3f * tfy;
}

// Symmetric 2x2 from J Sigma J^T where J = [[a, 0, b], [0, c, d]].
__device__ inline void jsjt(const M3 &S, float a, float b, float c, float d, float &s00, float &s01,
                            float &s11) {
    // rows of J Sigma
    const float r00 = a * S.m[0][0] + b * S.m[2][0];
    const float r01 = a * S.m[0][1] + b * S.m[2][1];
    const float r02 = a * S.m[0][2] + b * S.m[2][2];
    const float r10 = c * S.m[1][0] + d * S.m[2][0];
    const float r11 = c * S.m[1][1] + d * S.m[2][1];
    const float r12 = c * S.m[1][2] + d * S.m[2][2];
    s00 = r00 * a + r02 * b;
    s01 = r01 * c + r02 * d;
    s11 = r11 * c + r12 * d;
    (void)r10;
}

// Warp sum over all 32 lanes (butterfly, result in every lane).
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

} // namespace gsb
