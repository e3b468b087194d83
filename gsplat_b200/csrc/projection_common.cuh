// Per-(camera, Gaussian) EWA projection and its vector-Jacobian product, shared
// by the projection kernels (projection.cu) and the fused projection + SH
// kernels (projection_sh.cu).
//
// Reference behaviour: gsplat/cuda/csrc/ProjectionEWA3DGSFused.cu:72-233 (forward)
// and :347-552 (backward), with the math of gsplat/cuda/include/Utils.cuh.
#pragma once

#include "common.cuh"

namespace gsb {

// Fisheye (equidistant) projection of a camera-space point: pixel position and
// the 2x3 Jacobian J; Utils.cuh:662-700 (the eps terms of the reference kept).
__device__ inline void fisheye_mean_jacobian(float x, float y, float z, float fx, float fy, float cx, float cy,
                                             float &mx, float &my, float J[2][3]) {
    const float eps = 0.0000001f;
    const float xy_len = sqrtf(x * x + y * y) + eps;
    const float theta = atan2f(xy_len, z + eps);
    mx = x * fx * theta / xy_len + cx;
    my = y * fy * theta / xy_len + cy;
    const float x2 = x * x + eps;
    const float y2 = y * y;
    const float xy = x * y;
    const float x2y2 = x2 + y2;
    const float x2y2z2_inv = 1.f / (x2y2 + z * z);
    const float b = atan2f(xy_len, z) / xy_len / x2y2;
    const float a = z * x2y2z2_inv / x2y2;
    J[0][0] = fx * (x2 * a + y2 * b);
    J[0][1] = fx * xy * (a - b);
    J[0][2] = -fx * x * x2y2z2_inv;
    J[1][0] = fy * xy * (a - b);
    J[1][1] = fy * (y2 * a + x2 * b);
    J[1][2] = -fy * y * x2y2z2_inv;
}

// Gradient of the fisheye projection with respect to the camera-space point p =
// (x, y, z) given dL/dmean2d and dL/dJ (row-major 2x3), for the J of
// fisheye_mean_jacobian (the reference's Utils.cuh:662-700, eps terms included).
//
// Derivation. With s = x^2 + eps + y^2, rho = |(x, y)| + eps, theta =
// atan2(rho, z), q = 1 / (s + z^2), a = z q / s and b = theta / (rho s), J is
//   J00 = fx ((x^2 + eps) a + y^2 b)   J01 = fx x y (a - b)   J02 = -fx x q
//   J10 = fy x y (a - b)               J11 = fy (y^2 a + (x^2 + eps) b)
//   J12 = -fy y q,
// i.e. polynomial coefficients in x, y times the three scalar functions a, b, q.
// By the product rule, sum_rk vJ_rk dJ_rk/dp = (derivative of the coefficients
// with a, b, q held) + G_a grad(a) + G_b grad(b) + G_q grad(q), where G_f is the
// sum of vJ_rk times the coefficient of f in J_rk. The scalar gradients:
//   grad(q) = -2 q^2 (x, y, z)
//   grad(a) = (-2 x a (q + 1/s), -2 y a (q + 1/s), (q / s)(1 - 2 z^2 q))
//   grad(b) = (x beta, y beta, -t / s),  t = 1 / (rho^2 + z^2),
//             beta = z t / (r rho s) - b (1 / (r rho) + 2 / s),  r = |(x, y)|
// (d theta / d rho = z t, d theta / dz = -rho t, d rho / d(x, y) = (x, y) / r).
__device__ inline void fisheye_point_vjp(float x, float y, float z, float fx, float fy, const float v_m2d[2],
                                         const float vJ[2][3], float vmc[3]) {
    const float eps = 0.0000001f;
    const float xe = x * x + eps, yy = y * y, xy = x * y;
    const float s = xe + yy;
    const float inv_s = 1.f / s;
    const float r = sqrtf(x * x + yy);
    const float rho = r + eps;
    const float inv_rho = 1.f / rho;
    const float inv_r = r > 0.f ? 1.f / r : 0.f; // d rho / d(x, y) = (x, y) / r
    const float theta = atan2f(rho, z);
    const float q = 1.f / (s + z * z);
    const float a = z * q * inv_s;
    const float b = theta * inv_rho * inv_s;
    const float d = a - b;
    // dL/dmean2d through J (J^T v)
    const float J00 = fx * (xe * a + yy * b), J01 = fx * xy * d, J02 = -fx * x * q;
    const float J10 = fy * xy * d, J11 = fy * (yy * a + xe * b), J12 = -fy * y * q;
    vmc[0] += J00 * v_m2d[0] + J10 * v_m2d[1];
    vmc[1] += J01 * v_m2d[0] + J11 * v_m2d[1];
    vmc[2] += J02 * v_m2d[0] + J12 * v_m2d[1];
    // dL/dJ through dJ/dp
    const float w00 = fx * vJ[0][0], w01 = fx * vJ[0][1], w02 = fx * vJ[0][2];
    const float w10 = fy * vJ[1][0], w11 = fy * vJ[1][1], w12 = fy * vJ[1][2];
    const float wxy = w01 + w10;
    const float Ga = w00 * xe + wxy * xy + w11 * yy;
    const float Gb = w00 * yy - wxy * xy + w11 * xe;
    const float Gq = -(w02 * x + w12 * y);
    const float ex = 2.f * x * (w00 * a + w11 * b) + y * wxy * d - w02 * q;
    const float ey = 2.f * y * (w00 * b + w11 * a) + x * wxy * d - w12 * q;
    const float t = 1.f / (rho * rho + z * z);
    const float ra = -2.f * a * (q + inv_s);
    const float beta = z * t * inv_r * inv_rho * inv_s - b * (inv_r * inv_rho + 2.f * inv_s);
    const float qq = -2.f * q * q;
    vmc[0] += ex + x * (Ga * ra + Gb * beta + Gq * qq);
    vmc[1] += ey + y * (Ga * ra + Gb * beta + Gq * qq);
    vmc[2] += Ga * q * inv_s * (1.f - 2.f * z * z * q) - Gb * t * inv_s + Gq * qq * z;
}

// Symmetric 2x2 J S J^T for a full 2x3 J and a symmetric S.
__device__ inline void jsjt_full(const M3 &S, const float J[2][3], float &s00, float &s01, float &s11) {
    float JS[2][3];
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int j = 0; j < 3; ++j) JS[r][j] = J[r][0] * S.m[0][j] + J[r][1] * S.m[1][j] + J[r][2] * S.m[2][j];
    s00 = JS[0][0] * J[0][0] + JS[0][1] * J[0][1] + JS[0][2] * J[0][2];
    s01 = JS[0][0] * J[1][0] + JS[0][1] * J[1][1] + JS[0][2] * J[1][2];
    s11 = JS[1][0] * J[1][0] + JS[1][1] * J[1][1] + JS[1][2] * J[1][2];
}

struct ProjParams {
    uint32_t B, C, N;
    const float *means, *covars, *quats, *scales, *opacities, *viewmats, *Ks;
    uint32_t W, H;
    float eps2d, near_plane, far_plane, radius_clip;
    bool calc_comp;
    int camera_model;
};

struct ProjOut {
    bool valid;
    int32_t rx, ry;
    float mx, my, depth, conic[3], comp;
};

__device__ inline void load_gaussian(const ProjParams &p, uint32_t b, uint32_t g, float mean[3],
                                     M3 &covar) {
    const float *mp = p.means + ((size_t)b * p.N + g) * 3;
    mean[0] = mp[0];
    mean[1] = mp[1];
    mean[2] = mp[2];
    if (p.covars != nullptr) {
        const float *cp = p.covars + ((size_t)b * p.N + g) * 6;
        covar.m[0][0] = cp[0];
        covar.m[0][1] = cp[1];
        covar.m[0][2] = cp[2];
        covar.m[1][0] = cp[1];
        covar.m[1][1] = cp[3];
        covar.m[1][2] = cp[4];
        covar.m[2][0] = cp[2];
        covar.m[2][1] = cp[4];
        covar.m[2][2] = cp[5];
    } else {
        const float *qp = p.quats + ((size_t)b * p.N + g) * 4;
        const float *sp = p.scales + ((size_t)b * p.N + g) * 3;
        const float qa[4] = {qp[0], qp[1], qp[2], qp[3]};
        const float sa[3] = {sp[0], sp[1], sp[2]};
        covar = covar_from_quat_scale(qa, sa, nullptr);
    }
}

// Projects one Gaussian into one camera; follows ProjectionEWA3DGSFused.cu:72-233.
// With `known_visible` the culling tests are skipped: the caller already decided
// visibility (pass 1 of the packed layout) and only wants the outputs.
__device__ inline ProjOut project_one(const ProjParams &p, uint32_t b, uint32_t c, uint32_t g,
                                      const float mean[3], const M3 &covar,
                                      bool known_visible = false) {
    ProjOut o;
    o.valid = false;
    const float *vm = p.viewmats + ((size_t)b * p.C + c) * 16;
    const float *K = p.Ks + ((size_t)b * p.C + c) * 9;
    M3 R;
    R.m[0][0] = vm[0];
    R.m[0][1] = vm[1];
    R.m[0][2] = vm[2];
    R.m[1][0] = vm[4];
    R.m[1][1] = vm[5];
    R.m[1][2] = vm[6];
    R.m[2][0] = vm[8];
    R.m[2][1] = vm[9];
    R.m[2][2] = vm[10];
    const float x = R.m[0][0] * mean[0] + R.m[0][1] * mean[1] + R.m[0][2] * mean[2] + vm[3];
    const float y = R.m[1][0] * mean[0] + R.m[1][1] * mean[1] + R.m[1][2] * mean[2] + vm[7];
    const float z = R.m[2][0] * mean[0] + R.m[2][1] * mean[1] + R.m[2][2] * mean[2] + vm[11];
    if (!known_visible && (z < p.near_plane || z > p.far_plane)) return o;

    const M3 cov_c = m3_mul_bt(m3_mul(R, covar), R);
    const float fx = K[0], cx = K[2], fy = K[4], cy = K[5];
    float s00, s01, s11, mx, my;
    if (p.camera_model == kOrtho) {
        jsjt(cov_c, fx, 0.f, fy, 0.f, s00, s01, s11);
        mx = fx * x + cx;
        my = fy * y + cy;
    } else if (p.camera_model == kFisheye) {
        float J[2][3];
        fisheye_mean_jacobian(x, y, z, fx, fy, cx, cy, mx, my, J);
        jsjt_full(cov_c, J, s00, s01, s11);
    } else {
        float lxp, lxn, lyp, lyn;
        persp_limits(fx, fy, cx, cy, p.W, p.H, lxp, lxn, lyp, lyn);
        const float rz = 1.f / z;
        const float rz2 = rz * rz;
        const float tx = z * fminf(lxp, fmaxf(-lxn, x * rz));
        const float ty = z * fminf(lyp, fmaxf(-lyn, y * rz));
        jsjt(cov_c, fx * rz, -fx * tx * rz2, fy * rz, -fy * ty * rz2, s00, s01, s11);
        mx = fx * x * rz + cx;
        my = fy * y * rz + cy;
    }
    // add_blur (Utils.cuh:424-432)
    const float det_orig = s00 * s11 - s01 * s01;
    s00 += p.eps2d;
    s11 += p.eps2d;
    const float det = s00 * s11 - s01 * s01;
    const float comp = sqrtf(fmaxf(kMinCompensation * kMinCompensation, det_orig / det));
    if (!known_visible && det <= 0.f) return o;
    const float inv_det = 1.f / det;

    float extend = kGaussianExtend;
    if (p.opacities != nullptr) {
        float op = p.opacities[(size_t)b * p.N + g];
        if (p.calc_comp) op *= comp;
        if (!known_visible && op < kAlphaThreshold) return o;
        extend = fminf(kGaussianExtend, sqrtf(2.f * det_logf(fmaxf(op, kAlphaThreshold) / kAlphaThreshold)));
    }
    const float rx = ceilf(extend * sqrtf(s00));
    const float ry = ceilf(extend * sqrtf(s11));
    if (!known_visible) {
        if (rx <= p.radius_clip && ry <= p.radius_clip) return o;
        if (mx + rx <= 0.f || mx - rx >= (float)p.W || my + ry <= 0.f || my - ry >= (float)p.H) return o;
    }

    o.valid = true;
    o.rx = (int32_t)rx;
    o.ry = (int32_t)ry;
    o.mx = mx;
    o.my = my;
    o.depth = z;
    o.conic[0] = s11 * inv_det;
    o.conic[1] = -s01 * inv_det;
    o.conic[2] = s00 * inv_det;
    o.comp = comp;
    return o;
}

// ---------------------------------------------------------------------------
// Backward
// ---------------------------------------------------------------------------

struct ProjGrads {
    float v_mean[3];
    M3 v_cov;     // dL/dSigma (world)
    M3 v_R;       // dL/dR of this camera
    float v_t[3]; // dL/dt of this camera
};

// VJP of project_one for one (camera, Gaussian) pair: Utils.cuh:417-467 (inverse,
// blur), 583-660 (pinhole), 502-540 (ortho), 702-801 (fisheye), 62-112
// (world-to-camera).
__device__ inline void project_one_vjp(const ProjParams &p, uint32_t b, uint32_t c,
                                       const float mean[3], const M3 &covar, const float conic[3],
                                       float comp, const float v_m2d[2], float v_depth,
                                       const float v_conic[3], float v_comp, bool has_vcomp,
                                       ProjGrads &gr) {
    // inverse VJP: v_S = -Inv V Inv, V = [[va, vb/2], [vb/2, vc]]
    const float i00 = conic[0], i01 = conic[1], i11 = conic[2];
    const float va = v_conic[0], vb = 0.5f * v_conic[1], vc = v_conic[2];
    // Inv V
    const float t00 = i00 * va + i01 * vb, t01 = i00 * vb + i01 * vc;
    const float t10 = i01 * va + i11 * vb, t11 = i01 * vb + i11 * vc;
    float g00 = -(t00 * i00 + t01 * i01);
    float g01 = -(t00 * i01 + t01 * i11);
    float g10 = -(t10 * i00 + t11 * i01);
    float g11 = -(t10 * i01 + t11 * i11);
    if (has_vcomp) {
        const float det_conic = i00 * i11 - i01 * i01;
        const float v_sqr = v_comp * 0.5f / (comp + 1e-6f);
        const float omc = 1.f - comp * comp;
        g00 += v_sqr * (omc * i00 - p.eps2d * det_conic);
        g01 += v_sqr * (omc * i01);
        g10 += v_sqr * (omc * i01);
        g11 += v_sqr * (omc * i11 - p.eps2d * det_conic);
    }

    const float *vm = p.viewmats + ((size_t)b * p.C + c) * 16;
    const float *K = p.Ks + ((size_t)b * p.C + c) * 9;
    M3 R;
    R.m[0][0] = vm[0];
    R.m[0][1] = vm[1];
    R.m[0][2] = vm[2];
    R.m[1][0] = vm[4];
    R.m[1][1] = vm[5];
    R.m[1][2] = vm[6];
    R.m[2][0] = vm[8];
    R.m[2][1] = vm[9];
    R.m[2][2] = vm[10];
    const float x = R.m[0][0] * mean[0] + R.m[0][1] * mean[1] + R.m[0][2] * mean[2] + vm[3];
    const float y = R.m[1][0] * mean[0] + R.m[1][1] * mean[1] + R.m[1][2] * mean[2] + vm[7];
    const float z = R.m[2][0] * mean[0] + R.m[2][1] * mean[1] + R.m[2][2] * mean[2] + vm[11];
    const M3 RS = m3_mul(R, covar);
    const M3 cov_c = m3_mul_bt(RS, R);
    const float fx = K[0], cx = K[2], fy = K[4], cy = K[5];

    float vmc[3] = {0.f, 0.f, 0.f};
    M3 vcov_c;
    // J (2x3), v_cov3 += J^T G J
    float J[2][3];
    if (p.camera_model == kOrtho) {
        J[0][0] = fx;
        J[0][1] = 0.f;
        J[0][2] = 0.f;
        J[1][0] = 0.f;
        J[1][1] = fy;
        J[1][2] = 0.f;
    } else if (p.camera_model == kFisheye) {
        float mx_unused, my_unused;
        fisheye_mean_jacobian(x, y, z, fx, fy, cx, cy, mx_unused, my_unused, J);
    } else {
        const float rz = 1.f / z;
        float lxp, lxn, lyp, lyn;
        persp_limits(fx, fy, cx, cy, p.W, p.H, lxp, lxn, lyp, lyn);
        const float rz2 = rz * rz;
        const float tx = z * fminf(lxp, fmaxf(-lxn, x * rz));
        const float ty = z * fminf(lyp, fmaxf(-lyn, y * rz));
        J[0][0] = fx * rz;
        J[0][1] = 0.f;
        J[0][2] = -fx * tx * rz2;
        J[1][0] = 0.f;
        J[1][1] = fy * rz;
        J[1][2] = -fy * ty * rz2;
    }
    // G J (2x3)
    float GJ[2][3];
#pragma unroll
    for (int j = 0; j < 3; ++j) {
        GJ[0][j] = g00 * J[0][j] + g01 * J[1][j];
        GJ[1][j] = g10 * J[0][j] + g11 * J[1][j];
    }
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j) vcov_c.m[i][j] = J[0][i] * GJ[0][j] + J[1][i] * GJ[1][j];

    if (p.camera_model == kOrtho) {
        vmc[0] += fx * v_m2d[0];
        vmc[1] += fy * v_m2d[1];
    } else if (p.camera_model == kFisheye) {
        // v_J = G J S^T + G^T J S with S = cov_c symmetric: (G + G^T) J S
        float JS[2][3], vJ[2][3];
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
            for (int j = 0; j < 3; ++j)
                JS[r][j] = J[r][0] * cov_c.m[0][j] + J[r][1] * cov_c.m[1][j] + J[r][2] * cov_c.m[2][j];
#pragma unroll
        for (int j = 0; j < 3; ++j) {
            vJ[0][j] = 2.f * g00 * JS[0][j] + (g01 + g10) * JS[1][j];
            vJ[1][j] = (g10 + g01) * JS[0][j] + 2.f * g11 * JS[1][j];
        }
        fisheye_point_vjp(x, y, z, fx, fy, v_m2d, vJ, vmc);
    } else {
        const float rz = 1.f / z;
        const float rz2 = rz * rz;
        const float rz3 = rz2 * rz;
        float lxp, lxn, lyp, lyn;
        persp_limits(fx, fy, cx, cy, p.W, p.H, lxp, lxn, lyp, lyn);
        const float tx = z * fminf(lxp, fmaxf(-lxn, x * rz));
        const float ty = z * fminf(lyp, fmaxf(-lyn, y * rz));
        vmc[0] += fx * rz * v_m2d[0];
        vmc[1] += fy * rz * v_m2d[1];
        vmc[2] += -(fx * x * v_m2d[0] + fy * y * v_m2d[1]) * rz2;
        // v_J = G J S^T + G^T J S; S = cov_c is symmetric so both products use J S
        float vJ[2][3];
        // (J S) and (J S^T) rows; S symmetric so both equal
        float JS[2][3];
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
            for (int j = 0; j < 3; ++j)
                JS[r][j] = J[r][0] * cov_c.m[0][j] + J[r][1] * cov_c.m[1][j] + J[r][2] * cov_c.m[2][j];
#pragma unroll
        for (int j = 0; j < 3; ++j) {
            vJ[0][j] = g00 * JS[0][j] + g01 * JS[1][j] + g00 * JS[0][j] + g10 * JS[1][j];
            vJ[1][j] = g10 * JS[0][j] + g11 * JS[1][j] + g01 * JS[0][j] + g11 * JS[1][j];
        }
        if (x * rz <= lxp && x * rz >= -lxn) {
            vmc[0] += -fx * rz2 * vJ[0][2];
        } else {
            vmc[2] += -fx * rz3 * vJ[0][2] * tx;
        }
        if (y * rz <= lyp && y * rz >= -lyn) {
            vmc[1] += -fy * rz2 * vJ[1][2];
        } else {
            vmc[2] += -fy * rz3 * vJ[1][2] * ty;
        }
        vmc[2] += -fx * rz2 * vJ[0][0] - fy * rz2 * vJ[1][1] + 2.f * fx * tx * rz3 * vJ[0][2] +
                  2.f * fy * ty * rz3 * vJ[1][2];
    }
    vmc[2] += v_depth;

    // world-to-camera VJPs
#pragma unroll
    for (int i = 0; i < 3; ++i) {
        gr.v_t[i] = vmc[i];
        gr.v_mean[i] = R.m[0][i] * vmc[0] + R.m[1][i] * vmc[1] + R.m[2][i] * vmc[2];
#pragma unroll
        for (int j = 0; j < 3; ++j) gr.v_R.m[i][j] = vmc[i] * mean[j];
    }
    // v_R += G R S^T + G^T R S ; v_S = R^T G R   (G = vcov_c)
    const M3 GRS = m3_mul(vcov_c, RS);                 // G (R S)
    const M3 GtRS = m3_mul(m3_transpose(vcov_c), RS);  // G^T (R S)
    // S symmetric: R S^T = R S
    gr.v_R = m3_add(gr.v_R, m3_add(GRS, GtRS));
    gr.v_cov = m3_mul(m3_mul_at(R, vcov_c), R);
}

} // namespace gsb
