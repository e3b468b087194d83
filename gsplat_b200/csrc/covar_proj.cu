// Stand-alone covariance and projection ops of the reference's _wrapper API:
// quat_scale_to_covar_preci (QuatScaleToCovarCUDA.cu:36-292) and proj
// (ProjectionEWASimple.cu:36-317), forward and backward, for the three camera
// models (Utils.cuh:473-801). One thread per element; every output row is
// written by its own thread (no atomics).
//
// Matrices are row-major in memory. proj computes cov2d = J Sigma J^T and
// returns dL/dSigma = J^T G J (G = dL/dcov2d) and the gradient of the point
// through J with dL/dJ = G J Sigma^T + G^T J Sigma, the derivatives of the
// reference's PyTorch form (_torch_impl.py:42-211); for the symmetric
// covariances the ops are used with this equals the reference kernels' result.
#include "common.cuh"
#include "gsb_internal.h"
#include "projection_common.cuh"

namespace gsb {

// --------------------------------------------------------------------------
// quat_scale_to_covar_preci
// --------------------------------------------------------------------------

// Precision P = (R S^-1)(R S^-1)^T; Utils.cuh:238-256.
__device__ inline M3 preci_from_quat_scale(const M3 &R, const float s[3]) {
    M3 M;
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j) M.m[i][j] = R.m[i][j] * (1.f / s[j]);
    return m3_mul_bt(M, M);
}

__device__ inline void store_sym(float *out, const M3 &A, bool triu) {
    if (triu) {
        out[0] = A.m[0][0];
        out[1] = A.m[0][1];
        out[2] = A.m[0][2];
        out[3] = A.m[1][1];
        out[4] = A.m[1][2];
        out[5] = A.m[2][2];
    } else {
#pragma unroll
        for (int i = 0; i < 3; ++i)
#pragma unroll
            for (int j = 0; j < 3; ++j) out[i * 3 + j] = A.m[i][j];
    }
}

// Upstream gradient of a [.., 6] (upper triangle, off-diagonals shared by two
// entries: halved) or [.., 3, 3] output; QuatScaleToCovarCUDA.cu:205-243.
__device__ inline M3 load_grad(const float *g, bool triu) {
    M3 G;
    if (triu) {
        G.m[0][0] = g[0];
        G.m[0][1] = G.m[1][0] = 0.5f * g[1];
        G.m[0][2] = G.m[2][0] = 0.5f * g[2];
        G.m[1][1] = g[3];
        G.m[1][2] = G.m[2][1] = 0.5f * g[4];
        G.m[2][2] = g[5];
    } else {
#pragma unroll
        for (int i = 0; i < 3; ++i)
#pragma unroll
            for (int j = 0; j < 3; ++j) G.m[i][j] = g[i * 3 + j];
    }
    return G;
}

__global__ void __launch_bounds__(256) covar_preci_fwd_kernel(long long n, const float *__restrict__ quats,
                                                              const float *__restrict__ scales, bool triu,
                                                              float *__restrict__ covars,
                                                              float *__restrict__ precis) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float q[4] = {quats[i * 4], quats[i * 4 + 1], quats[i * 4 + 2], quats[i * 4 + 3]};
    const float s[3] = {scales[i * 3], scales[i * 3 + 1], scales[i * 3 + 2]};
    M3 R;
    const M3 C = covar_from_quat_scale(q, s, &R);
    const int w = triu ? 6 : 9;
    if (covars != nullptr) store_sym(covars + i * w, C, triu);
    if (precis != nullptr) store_sym(precis + i * w, preci_from_quat_scale(R, s), triu);
}

__global__ void __launch_bounds__(256) covar_preci_bwd_kernel(long long n, const float *__restrict__ quats,
                                                              const float *__restrict__ scales, bool triu,
                                                              const float *__restrict__ v_covars,
                                                              const float *__restrict__ v_precis,
                                                              float *__restrict__ v_quats,
                                                              float *__restrict__ v_scales) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float q[4] = {quats[i * 4], quats[i * 4 + 1], quats[i * 4 + 2], quats[i * 4 + 3]};
    const float s[3] = {scales[i * 3], scales[i * 3 + 1], scales[i * 3 + 2]};
    const M3 R = quat_to_rotmat(q[0], q[1], q[2], q[3]);
    float vq[4] = {0.f, 0.f, 0.f, 0.f}, vs[3] = {0.f, 0.f, 0.f};
    const int w = triu ? 6 : 9;
    if (v_covars != nullptr) covar_from_quat_scale_vjp(q, s, R, load_grad(v_covars + i * w, triu), vq, vs);
    if (v_precis != nullptr) {
        // Utils.cuh:298-341: M = R S^-1, v_M = (G + G^T) M, v_R = v_M S^-1,
        // dL/ds_j = -s_j^-2 sum_k R[k][j] v_M[k][j]
        const M3 G = load_grad(v_precis + i * w, triu);
        const float si[3] = {1.f / s[0], 1.f / s[1], 1.f / s[2]};
        M3 M;
#pragma unroll
        for (int a = 0; a < 3; ++a)
#pragma unroll
            for (int b = 0; b < 3; ++b) M.m[a][b] = R.m[a][b] * si[b];
        const M3 vM = m3_mul(m3_add(G, m3_transpose(G)), M);
        M3 vR;
#pragma unroll
        for (int a = 0; a < 3; ++a)
#pragma unroll
            for (int b = 0; b < 3; ++b) vR.m[a][b] = vM.m[a][b] * si[b];
        quat_to_rotmat_vjp(q, vR, vq);
#pragma unroll
        for (int j = 0; j < 3; ++j)
            vs[j] += -si[j] * si[j] * (R.m[0][j] * vM.m[0][j] + R.m[1][j] * vM.m[1][j] + R.m[2][j] * vM.m[2][j]);
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) v_quats[i * 4 + k] = vq[k];
#pragma unroll
    for (int k = 0; k < 3; ++k) v_scales[i * 3 + k] = vs[k];
}

// --------------------------------------------------------------------------
// proj: camera-space means [B, C, N, 3] and covariances [B, C, N, 3, 3]
// --------------------------------------------------------------------------

// Pixel position and Jacobian of one camera-space point (Utils.cuh:473-500,
// 542-581, 662-700). Pinhole clamps the Jacobian's x / z and y / z to 1.3x the
// field of view.
__device__ inline void point_jacobian(int model, float x, float y, float z, float fx, float fy, float cx,
                                      float cy, uint32_t W, uint32_t H, float &mx, float &my, float J[2][3]) {
    if (model == kOrtho) {
        J[0][0] = fx;
        J[0][1] = 0.f;
        J[0][2] = 0.f;
        J[1][0] = 0.f;
        J[1][1] = fy;
        J[1][2] = 0.f;
        mx = fx * x + cx;
        my = fy * y + cy;
    } else if (model == kFisheye) {
        fisheye_mean_jacobian(x, y, z, fx, fy, cx, cy, mx, my, J);
    } else {
        float lxp, lxn, lyp, lyn;
        persp_limits(fx, fy, cx, cy, W, H, lxp, lxn, lyp, lyn);
        const float rz = 1.f / z;
        const float rz2 = rz * rz;
        const float tx = z * fminf(lxp, fmaxf(-lxn, x * rz));
        const float ty = z * fminf(lyp, fmaxf(-lyn, y * rz));
        J[0][0] = fx * rz;
        J[0][1] = 0.f;
        J[0][2] = -fx * tx * rz2;
        J[1][0] = 0.f;
        J[1][1] = fy * rz;
        J[1][2] = -fy * ty * rz2;
        mx = fx * x * rz + cx;
        my = fy * y * rz + cy;
    }
}

__global__ void __launch_bounds__(256) proj_fwd_kernel(uint32_t B, uint32_t C, uint32_t N,
                                                       const float *__restrict__ means,
                                                       const float *__restrict__ covars,
                                                       const float *__restrict__ Ks, uint32_t W, uint32_t H,
                                                       int model, float *__restrict__ means2d,
                                                       float *__restrict__ covars2d) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)B * C * N) return;
    const long long bc = i / N;
    const float *K = Ks + bc * 9;
    const float x = means[i * 3], y = means[i * 3 + 1], z = means[i * 3 + 2];
    float mx, my, J[2][3];
    point_jacobian(model, x, y, z, K[0], K[4], K[2], K[5], W, H, mx, my, J);
    const float *S = covars + i * 9;
    float JS[2][3];
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int j = 0; j < 3; ++j) JS[r][j] = J[r][0] * S[j] + J[r][1] * S[3 + j] + J[r][2] * S[6 + j];
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int c = 0; c < 2; ++c)
            covars2d[i * 4 + r * 2 + c] = JS[r][0] * J[c][0] + JS[r][1] * J[c][1] + JS[r][2] * J[c][2];
    means2d[i * 2] = mx;
    means2d[i * 2 + 1] = my;
}

__global__ void __launch_bounds__(256) proj_bwd_kernel(uint32_t B, uint32_t C, uint32_t N,
                                                       const float *__restrict__ means,
                                                       const float *__restrict__ covars,
                                                       const float *__restrict__ Ks, uint32_t W, uint32_t H,
                                                       int model, const float *__restrict__ v_means2d,
                                                       const float *__restrict__ v_covars2d,
                                                       float *__restrict__ v_means, float *__restrict__ v_covars) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)B * C * N) return;
    const long long bc = i / N;
    const float *K = Ks + bc * 9;
    const float fx = K[0], fy = K[4], cx = K[2], cy = K[5];
    const float x = means[i * 3], y = means[i * 3 + 1], z = means[i * 3 + 2];
    float mx, my, J[2][3];
    point_jacobian(model, x, y, z, fx, fy, cx, cy, W, H, mx, my, J);
    const float *S = covars + i * 9;
    const float g00 = v_covars2d[i * 4], g01 = v_covars2d[i * 4 + 1];
    const float g10 = v_covars2d[i * 4 + 2], g11 = v_covars2d[i * 4 + 3];
    const float v_m2d[2] = {v_means2d[i * 2], v_means2d[i * 2 + 1]};
    // dL/dSigma = J^T G J
    float GJ[2][3];
#pragma unroll
    for (int j = 0; j < 3; ++j) {
        GJ[0][j] = g00 * J[0][j] + g01 * J[1][j];
        GJ[1][j] = g10 * J[0][j] + g11 * J[1][j];
    }
#pragma unroll
    for (int a = 0; a < 3; ++a)
#pragma unroll
        for (int b = 0; b < 3; ++b) v_covars[i * 9 + a * 3 + b] = J[0][a] * GJ[0][b] + J[1][a] * GJ[1][b];
    // dL/dJ = G J S^T + G^T J S
    float JSt[2][3], JS[2][3], vJ[2][3];
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int j = 0; j < 3; ++j) {
            JSt[r][j] = J[r][0] * S[j * 3] + J[r][1] * S[j * 3 + 1] + J[r][2] * S[j * 3 + 2];
            JS[r][j] = J[r][0] * S[j] + J[r][1] * S[3 + j] + J[r][2] * S[6 + j];
        }
#pragma unroll
    for (int j = 0; j < 3; ++j) {
        vJ[0][j] = g00 * JSt[0][j] + g01 * JSt[1][j] + g00 * JS[0][j] + g10 * JS[1][j];
        vJ[1][j] = g10 * JSt[0][j] + g11 * JSt[1][j] + g01 * JS[0][j] + g11 * JS[1][j];
    }
    float vm[3] = {0.f, 0.f, 0.f};
    if (model == kOrtho) {
        vm[0] = fx * v_m2d[0];
        vm[1] = fy * v_m2d[1];
    } else if (model == kFisheye) {
        fisheye_point_vjp(x, y, z, fx, fy, v_m2d, vJ, vm);
    } else {
        // Utils.cuh:583-660
        float lxp, lxn, lyp, lyn;
        persp_limits(fx, fy, cx, cy, W, H, lxp, lxn, lyp, lyn);
        const float rz = 1.f / z;
        const float rz2 = rz * rz;
        const float rz3 = rz2 * rz;
        const float tx = z * fminf(lxp, fmaxf(-lxn, x * rz));
        const float ty = z * fminf(lyp, fmaxf(-lyn, y * rz));
        vm[0] = fx * rz * v_m2d[0];
        vm[1] = fy * rz * v_m2d[1];
        vm[2] = -(fx * x * v_m2d[0] + fy * y * v_m2d[1]) * rz2;
        if (x * rz <= lxp && x * rz >= -lxn) {
            vm[0] += -fx * rz2 * vJ[0][2];
        } else {
            vm[2] += -fx * rz3 * vJ[0][2] * tx;
        }
        if (y * rz <= lyp && y * rz >= -lyn) {
            vm[1] += -fy * rz2 * vJ[1][2];
        } else {
            vm[2] += -fy * rz3 * vJ[1][2] * ty;
        }
        vm[2] += -fx * rz2 * vJ[0][0] - fy * rz2 * vJ[1][1] + 2.f * fx * tx * rz3 * vJ[0][2] +
                 2.f * fy * ty * rz3 * vJ[1][2];
    }
#pragma unroll
    for (int k = 0; k < 3; ++k) v_means[i * 3 + k] = vm[k];
}

static unsigned blocks_for(long long n) { return (unsigned)((n + 255) / 256); }

static int check_model(int m) {
    if (m == kPinhole || m == kOrtho || m == kFisheye) return kOk;
    return set_error(kErrUnsupported, "camera_model %d is not supported (pinhole=0, ortho=1, fisheye=2)", m);
}

} // namespace gsb

using namespace gsb;

extern "C" int gsb_quat_scale_to_covar_preci_fwd(long long n, const float *quats, const float *scales, int triu,
                                                 float *covars, float *precis, cudaStream_t stream) {
    if (n < 0) return set_error(kErrInvalidArgument, "negative element count");
    if (n == 0 || (covars == nullptr && precis == nullptr)) return kOk;
    covar_preci_fwd_kernel<<<blocks_for(n), 256, 0, stream>>>(n, quats, scales, triu != 0, covars, precis);
    return check_launch("covar_preci_fwd_kernel");
}

extern "C" int gsb_quat_scale_to_covar_preci_bwd(long long n, const float *quats, const float *scales, int triu,
                                                 const float *v_covars, const float *v_precis, float *v_quats,
                                                 float *v_scales, cudaStream_t stream) {
    if (n < 0) return set_error(kErrInvalidArgument, "negative element count");
    if (n == 0) return kOk;
    covar_preci_bwd_kernel<<<blocks_for(n), 256, 0, stream>>>(n, quats, scales, triu != 0, v_covars, v_precis,
                                                              v_quats, v_scales);
    return check_launch("covar_preci_bwd_kernel");
}

extern "C" int gsb_proj_fwd(int B, int C, int N, const float *means, const float *covars, const float *Ks,
                            int width, int height, int camera_model, float *means2d, float *covars2d,
                            cudaStream_t stream) {
    if (int e = check_model(camera_model)) return e;
    if (B < 0 || C < 0 || N < 0) return set_error(kErrInvalidArgument, "negative shape");
    const long long n = (long long)B * C * N;
    if (n == 0) return kOk;
    proj_fwd_kernel<<<blocks_for(n), 256, 0, stream>>>((uint32_t)B, (uint32_t)C, (uint32_t)N, means, covars, Ks,
                                                       (uint32_t)width, (uint32_t)height, camera_model, means2d,
                                                       covars2d);
    return check_launch("proj_fwd_kernel");
}

extern "C" int gsb_proj_bwd(int B, int C, int N, const float *means, const float *covars, const float *Ks,
                            int width, int height, int camera_model, const float *v_means2d,
                            const float *v_covars2d, float *v_means, float *v_covars, cudaStream_t stream) {
    if (int e = check_model(camera_model)) return e;
    if (B < 0 || C < 0 || N < 0) return set_error(kErrInvalidArgument, "negative shape");
    const long long n = (long long)B * C * N;
    if (n == 0) return kOk;
    proj_bwd_kernel<<<blocks_for(n), 256, 0, stream>>>((uint32_t)B, (uint32_t)C, (uint32_t)N, means, covars, Ks,
                                                       (uint32_t)width, (uint32_t)height, camera_model, v_means2d,
                                                       v_covars2d, v_means, v_covars);
    return check_launch("proj_bwd_kernel");
}
