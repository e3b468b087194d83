/*
 * CPU ORACLE -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference gsplat (mc8max/gsplat v1.5.3) CUDA
 * semantics for the training hot path. It exists to check the gsplat_b200 kernels
 * (tests/, __graft_entry__.smoke, bench.py's CPU baseline) and is never part of
 * the product path. Every function cites the reference code it restates:
 *
 *   ora_projection_fwd   ProjectionEWA3DGSFused.cu:63-233 (+ Utils.cuh:174-257, 424-432, 473-581)
 *   ora_projection_bwd   ProjectionEWA3DGSFused.cu:347-552 (+ Utils.cuh:59-112, 198-296, 417-467, 502-660)
 *   ora_sh_fwd / _bwd    SphericalHarmonicsCUDA.cu:38-388 (Sloan's polynomial form)
 *   ora_isect_count/emit IntersectTile.cu:40-126, 132-288
 *   ora_sort_pairs       cub::DeviceRadixSort::SortPairs (stable) of IntersectTile.cu:478-521
 *   ora_isect_offsets    IntersectTile.cu:391-439
 *   ora_raster_fwd       RasterizeToPixels3DGSFwd.cu:64-212
 *   ora_raster_bwd       RasterizeToPixels3DGSBwd.cu:74-299
 *   ora_adam             AdamCUDA.cu:48-68
 *   ora_covar_preci_fwd / _bwd   QuatScaleToCovarCUDA.cu:36-292 (+ Utils.cuh:223-341)
 *   ora_proj_fwd / _bwd  ProjectionEWASimple.cu:36-317 (+ Utils.cuh:473-801)
 *   ora_raster_indices   RasterizeToIndices3DGS.cu:36-200, Rasterization.cpp:216-300
 *
 * Forward math is single precision in the reference's operation order (compiled
 * with -ffp-contract=off, libm expf/sqrtf). Gradient sums over pixels / cameras
 * are accumulated in double, which makes this the reference answer for the
 * order-dependent float atomics of the GPU. Tile intersection uses the shared
 * deterministic primitives of detmath.h so that it is bit-exact with the GPU.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "detmath.h"

#define ORA_ALPHA_THRESHOLD (1.f / 255.f)
#define ORA_EXTEND 3.33f
#define ORA_MAX_ALPHA 0.99f
#define ORA_T_THRESHOLD 1e-4f
#define ORA_MIN_COMP 0.005f
#define ORA_MIN_1MA 1e-6f

typedef struct {
    float m[3][3];
} ora_m3;

static ora_m3 m3mul(ora_m3 a, ora_m3 b) {
    ora_m3 r;
    for (int i = 0; i < 3; ++i)
        for (int j = 0; j < 3; ++j) r.m[i][j] = a.m[i][0] * b.m[0][j] + a.m[i][1] * b.m[1][j] + a.m[i][2] * b.m[2][j];
    return r;
}
static ora_m3 m3t(ora_m3 a) {
    ora_m3 r;
    for (int i = 0; i < 3; ++i)
        for (int j = 0; j < 3; ++j) r.m[i][j] = a.m[j][i];
    return r;
}

/* Utils.cuh:174-196 (row-major form) */
static ora_m3 quat_rot(const float *q) {
    float w = q[0], x = q[1], y = q[2], z = q[3];
    float inv = 1.f / sqrtf(x * x + y * y + z * z + w * w);
    x *= inv; y *= inv; z *= inv; w *= inv;
    ora_m3 R;
    R.m[0][0] = 1.f - 2.f * (y * y + z * z); R.m[0][1] = 2.f * (x * y - w * z); R.m[0][2] = 2.f * (x * z + w * y);
    R.m[1][0] = 2.f * (x * y + w * z); R.m[1][1] = 1.f - 2.f * (x * x + z * z); R.m[1][2] = 2.f * (y * z - w * x);
    R.m[2][0] = 2.f * (x * z - w * y); R.m[2][1] = 2.f * (y * z + w * x); R.m[2][2] = 1.f - 2.f * (x * x + y * y);
    return R;
}

static ora_m3 covar_of(const float *covars, const float *quats, const float *scales, size_t gi) {
    ora_m3 S;
    if (covars) {
        const float *c = covars + gi * 6;
        S.m[0][0] = c[0]; S.m[0][1] = c[1]; S.m[0][2] = c[2];
        S.m[1][0] = c[1]; S.m[1][1] = c[3]; S.m[1][2] = c[4];
        S.m[2][0] = c[2]; S.m[2][1] = c[4]; S.m[2][2] = c[5];
        return S;
    }
    ora_m3 R = quat_rot(quats + gi * 4);
    const float *s = scales + gi * 3;
    ora_m3 M;
    for (int i = 0; i < 3; ++i)
        for (int j = 0; j < 3; ++j) M.m[i][j] = R.m[i][j] * s[j];
    return m3mul(M, m3t(M));
}

typedef struct {
    ora_m3 R;
    float t[3];
    float fx, fy, cx, cy;
} ora_cam;

static ora_cam cam_of(const float *viewmats, const float *Ks, size_t ci) {
    ora_cam c;
    const float *v = viewmats + ci * 16;
    for (int i = 0; i < 3; ++i) {
        for (int j = 0; j < 3; ++j) c.R.m[i][j] = v[i * 4 + j];
        c.t[i] = v[i * 4 + 3];
    }
    const float *K = Ks + ci * 9;
    c.fx = K[0]; c.cx = K[2]; c.fy = K[4]; c.cy = K[5];
    return c;
}

/* fisheye mean and J; Utils.cuh:662-700 (eps terms kept) */
static void fisheye_jacobian(float fx, float fy, float cx, float cy, float x, float y, float z,
                             float J[2][3], float *mx, float *my) {
    const float eps = 0.0000001f;
    float xy_len = sqrtf(x * x + y * y) + eps;
    float theta = atan2f(xy_len, z + eps);
    *mx = x * fx * theta / xy_len + cx;
    *my = y * fy * theta / xy_len + cy;
    float x2 = x * x + eps, y2 = y * y, xy = x * y, x2y2 = x2 + y2;
    float inv = 1.f / (x2y2 + z * z);
    float b = atan2f(xy_len, z) / xy_len / x2y2;
    float a = z * inv / x2y2;
    J[0][0] = fx * (x2 * a + y2 * b); J[0][1] = fx * xy * (a - b); J[0][2] = -fx * x * inv;
    J[1][0] = fy * xy * (a - b); J[1][1] = fy * (y2 * a + x2 * b); J[1][2] = -fy * y * inv;
}

/* J for pinhole (with the 1.3x fov clamp), ortho or fisheye; Utils.cuh:473-700 */
static void proj_jacobian(int model, const ora_cam *c, int W, int H, float x, float y, float z,
                          float J[2][3], float *mx, float *my) {
    if (model == 2) {
        fisheye_jacobian(c->fx, c->fy, c->cx, c->cy, x, y, z, J, mx, my);
        return;
    }
    if (model == 1) {
        J[0][0] = c->fx; J[0][1] = 0.f; J[0][2] = 0.f;
        J[1][0] = 0.f; J[1][1] = c->fy; J[1][2] = 0.f;
        *mx = c->fx * x + c->cx;
        *my = c->fy * y + c->cy;
        return;
    }
    float tan_fovx = 0.5f * (float)W / c->fx, tan_fovy = 0.5f * (float)H / c->fy;
    float lxp = ((float)W - c->cx) / c->fx + 0.3f * tan_fovx;
    float lxn = c->cx / c->fx + 0.3f * tan_fovx;
    float lyp = ((float)H - c->cy) / c->fy + 0.3f * tan_fovy;
    float lyn = c->cy / c->fy + 0.3f * tan_fovy;
    float rz = 1.f / z, rz2 = rz * rz;
    float tx = z * fminf(lxp, fmaxf(-lxn, x * rz));
    float ty = z * fminf(lyp, fmaxf(-lyn, y * rz));
    J[0][0] = c->fx * rz; J[0][1] = 0.f; J[0][2] = -c->fx * tx * rz2;
    J[1][0] = 0.f; J[1][1] = c->fy * rz; J[1][2] = -c->fy * ty * rz2;
    *mx = c->fx * x * rz + c->cx;
    *my = c->fy * y * rz + c->cy;
}

void ora_projection_fwd(int B, int C, int N, const float *means, const float *covars,
                        const float *quats, const float *scales, const float *opacities,
                        const float *viewmats, const float *Ks, int W, int H, float eps2d,
                        float near_plane, float far_plane, float radius_clip, int calc_comp,
                        int camera_model, int32_t *radii, float *means2d, float *depths,
                        float *conics, float *comps) {
#pragma omp parallel for schedule(static)
    for (long long idx = 0; idx < (long long)B * C * N; ++idx) {
        const size_t b = idx / ((size_t)C * N), c = (idx / N) % C, g = idx % N;
        const size_t gi = b * N + g;
        radii[idx * 2] = 0; radii[idx * 2 + 1] = 0;
        means2d[idx * 2] = 0.f; means2d[idx * 2 + 1] = 0.f;
        depths[idx] = 0.f;
        conics[idx * 3] = conics[idx * 3 + 1] = conics[idx * 3 + 2] = 0.f;
        if (comps) comps[idx] = 0.f;
        ora_cam cam = cam_of(viewmats, Ks, b * C + c);
        const float *m = means + gi * 3;
        float p[3];
        for (int i = 0; i < 3; ++i) p[i] = cam.R.m[i][0] * m[0] + cam.R.m[i][1] * m[1] + cam.R.m[i][2] * m[2] + cam.t[i];
        if (p[2] < near_plane || p[2] > far_plane) continue;
        ora_m3 S = covar_of(covars, quats, scales, gi);
        ora_m3 Sc = m3mul(m3mul(cam.R, S), m3t(cam.R));
        float J[2][3], mx, my;
        proj_jacobian(camera_model, &cam, W, H, p[0], p[1], p[2], J, &mx, &my);
        float JS[2][3];
        for (int r = 0; r < 2; ++r)
            for (int j = 0; j < 3; ++j) JS[r][j] = J[r][0] * Sc.m[0][j] + J[r][1] * Sc.m[1][j] + J[r][2] * Sc.m[2][j];
        float c00 = JS[0][0] * J[0][0] + JS[0][1] * J[0][1] + JS[0][2] * J[0][2];
        float c01 = JS[0][0] * J[1][0] + JS[0][1] * J[1][1] + JS[0][2] * J[1][2];
        float c11 = JS[1][0] * J[1][0] + JS[1][1] * J[1][1] + JS[1][2] * J[1][2];
        float det_orig = c00 * c11 - c01 * c01;
        c00 += eps2d; c11 += eps2d;
        float det = c00 * c11 - c01 * c01;
        float comp = sqrtf(fmaxf(ORA_MIN_COMP * ORA_MIN_COMP, det_orig / det));
        if (det <= 0.f) continue;
        float extend = ORA_EXTEND;
        if (opacities) {
            float op = opacities[gi];
            if (calc_comp) op *= comp;
            if (op < ORA_ALPHA_THRESHOLD) continue;
            extend = fminf(ORA_EXTEND, sqrtf(2.f * det_logf(op / ORA_ALPHA_THRESHOLD)));
        }
        float rx = ceilf(extend * sqrtf(c00)), ry = ceilf(extend * sqrtf(c11));
        if (rx <= radius_clip && ry <= radius_clip) continue;
        if (mx + rx <= 0 || mx - rx >= (float)W || my + ry <= 0 || my - ry >= (float)H) continue;
        float inv = 1.f / det;
        radii[idx * 2] = (int32_t)rx; radii[idx * 2 + 1] = (int32_t)ry;
        means2d[idx * 2] = mx; means2d[idx * 2 + 1] = my;
        depths[idx] = p[2];
        conics[idx * 3] = c11 * inv; conics[idx * 3 + 1] = -c01 * inv; conics[idx * 3 + 2] = c00 * inv;
        if (comps) comps[idx] = comp;
    }
}

/* quat_to_rotmat_vjp, Utils.cuh:198-221 (G = dL/dR, row-major) */
static void quat_vjp(const float *q, const double G[3][3], double vq[4]) {
    double w = q[0], x = q[1], y = q[2], z = q[3];
    double inv = 1.0 / sqrt(w * w + x * x + y * y + z * z);
    w *= inv; x *= inv; y *= inv; z *= inv;
    double vn[4];
    vn[0] = 2 * (x * (G[2][1] - G[1][2]) + y * (G[0][2] - G[2][0]) + z * (G[1][0] - G[0][1]));
    vn[1] = 2 * (-2 * x * (G[1][1] + G[2][2]) + y * (G[0][1] + G[1][0]) + z * (G[0][2] + G[2][0]) + w * (G[2][1] - G[1][2]));
    vn[2] = 2 * (x * (G[0][1] + G[1][0]) - 2 * y * (G[0][0] + G[2][2]) + z * (G[1][2] + G[2][1]) + w * (G[0][2] - G[2][0]));
    vn[3] = 2 * (x * (G[0][2] + G[2][0]) + y * (G[1][2] + G[2][1]) - 2 * z * (G[0][0] + G[1][1]) + w * (G[1][0] - G[0][1]));
    double d = vn[0] * w + vn[1] * x + vn[2] * y + vn[3] * z;
    vq[0] += (vn[0] - d * w) * inv; vq[1] += (vn[1] - d * x) * inv;
    vq[2] += (vn[2] - d * y) * inv; vq[3] += (vn[3] - d * z) * inv;
}

/* Forward-mode dual numbers: a value and its derivatives with respect to three
 * inputs (the fisheye Jacobian below and the SH bases). */
typedef struct {
    double v, d[3];
} dual3;

static dual3 dc(double v) { dual3 r = {v, {0, 0, 0}}; return r; }
static dual3 dadd(dual3 a, dual3 b) { dual3 r; r.v = a.v + b.v; for (int i = 0; i < 3; ++i) r.d[i] = a.d[i] + b.d[i]; return r; }
static dual3 dsub(dual3 a, dual3 b) { dual3 r; r.v = a.v - b.v; for (int i = 0; i < 3; ++i) r.d[i] = a.d[i] - b.d[i]; return r; }
static dual3 dmul(dual3 a, dual3 b) { dual3 r; r.v = a.v * b.v; for (int i = 0; i < 3; ++i) r.d[i] = a.d[i] * b.v + a.v * b.d[i]; return r; }
static dual3 dscale(double s, dual3 a) { dual3 r; r.v = s * a.v; for (int i = 0; i < 3; ++i) r.d[i] = s * a.d[i]; return r; }

static dual3 ddiv(dual3 a, dual3 b) {
    dual3 r; r.v = a.v / b.v;
    for (int i = 0; i < 3; ++i) r.d[i] = (a.d[i] * b.v - a.v * b.d[i]) / (b.v * b.v);
    return r;
}
static dual3 dsqrt(dual3 a) { dual3 r; r.v = sqrt(a.v); for (int i = 0; i < 3; ++i) r.d[i] = a.d[i] / (2.0 * r.v); return r; }
static dual3 datan2(dual3 y, dual3 x) {
    dual3 r; r.v = atan2(y.v, x.v);
    double n = x.v * x.v + y.v * y.v;
    for (int i = 0; i < 3; ++i) r.d[i] = (x.v * y.d[i] - y.v * x.d[i]) / n;
    return r;
}

/* Fisheye (equidistant) J of Utils.cuh:662-700 as dual numbers over the
 * camera-space point: J's values and, in .d, dJ/d(x, y, z) by forward-mode
 * differentiation of the same formula (eps terms kept as the reference has them). */
static void fisheye_jacobian_dual(double fx, double fy, double x, double y, double z, dual3 J[2][3]) {
    const double eps = 0.0000001;
    dual3 X = {x, {1, 0, 0}}, Y = {y, {0, 1, 0}}, Z = {z, {0, 0, 1}};
    dual3 x2 = dadd(dmul(X, X), dc(eps)), y2 = dmul(Y, Y), xy = dmul(X, Y), x2y2 = dadd(x2, y2);
    dual3 len_xy = dadd(dsqrt(dadd(dmul(X, X), y2)), dc(eps));
    dual3 inv = ddiv(dc(1.0), dadd(x2y2, dmul(Z, Z)));
    dual3 b = ddiv(ddiv(datan2(len_xy, Z), len_xy), x2y2);
    dual3 a = ddiv(dmul(Z, inv), x2y2);
    J[0][0] = dscale(fx, dadd(dmul(x2, a), dmul(y2, b)));
    J[0][1] = dscale(fx, dmul(xy, dsub(a, b)));
    J[0][2] = dscale(-fx, dmul(X, inv));
    J[1][0] = dscale(fy, dmul(xy, dsub(a, b)));
    J[1][1] = dscale(fy, dadd(dmul(y2, a), dmul(x2, b)));
    J[1][2] = dscale(-fy, dmul(Y, inv));
}

static void fisheye_jacobian_d(double fx, double fy, double x, double y, double z, double J[2][3]) {
    dual3 Jd[2][3];
    fisheye_jacobian_dual(fx, fy, x, y, z, Jd);
    for (int r = 0; r < 2; ++r)
        for (int k = 0; k < 3; ++k) J[r][k] = Jd[r][k].v;
}

/* dL/dpoint = J^T dL/dmean2d + sum_rk dL/dJ_rk dJ_rk/dpoint (Utils.cuh:702-801). */
static void fisheye_point_vjp_d(double fx, double fy, double x, double y, double z, const double vm2[2],
                                const double vJ[2][3], double vmc[3]) {
    dual3 J[2][3];
    fisheye_jacobian_dual(fx, fy, x, y, z, J);
    for (int i = 0; i < 3; ++i) {
        vmc[i] += J[0][i].v * vm2[0] + J[1][i].v * vm2[1];
        for (int r = 0; r < 2; ++r)
            for (int k = 0; k < 3; ++k) vmc[i] += vJ[r][k] * J[r][k].d[i];
    }
}

/* Dense backward, double precision throughout; one Gaussian per iteration
 * summing over cameras, like the per-(c,n) atomics of the reference. */
void ora_projection_bwd(int B, int C, int N, const float *means, const float *covars,
                        const float *quats, const float *scales, const float *viewmats,
                        const float *Ks, int W, int H, float eps2d, int camera_model,
                        const int32_t *radii, const float *conics, const float *comps,
                        const float *v_means2d, const float *v_depths, const float *v_conics,
                        const float *v_comps, float *v_means, float *v_covars, float *v_quats,
                        float *v_scales, float *v_viewmats) {
    double *vview = NULL;
    if (v_viewmats) vview = (double *)calloc((size_t)B * C * 16, sizeof(double));
#pragma omp parallel
    {
        double *vview_local = v_viewmats ? (double *)calloc((size_t)B * C * 16, sizeof(double)) : NULL;
#pragma omp for schedule(static)
        for (long long bg = 0; bg < (long long)B * N; ++bg) {
            const size_t b = bg / N, g = bg % N, gi = bg;
            double vm[3] = {0, 0, 0}, vS[3][3] = {{0}};
            ora_m3 Sf = covar_of(covars, quats, scales, gi);
            double S[3][3];
            for (int i = 0; i < 3; ++i)
                for (int j = 0; j < 3; ++j) S[i][j] = Sf.m[i][j];
            const float *m = means + gi * 3;
            for (int c = 0; c < C; ++c) {
                const size_t idx = (b * C + c) * (size_t)N + g;
                if (radii[idx * 2] <= 0 || radii[idx * 2 + 1] <= 0) continue;
                ora_cam cam = cam_of(viewmats, Ks, b * C + c);
                double R[3][3], t[3], p[3];
                for (int i = 0; i < 3; ++i) {
                    for (int j = 0; j < 3; ++j) R[i][j] = cam.R.m[i][j];
                    t[i] = cam.t[i];
                }
                for (int i = 0; i < 3; ++i) p[i] = R[i][0] * m[0] + R[i][1] * m[1] + R[i][2] * m[2] + t[i];
                double RS[3][3], Sc[3][3];
                for (int i = 0; i < 3; ++i)
                    for (int j = 0; j < 3; ++j) RS[i][j] = R[i][0] * S[0][j] + R[i][1] * S[1][j] + R[i][2] * S[2][j];
                for (int i = 0; i < 3; ++i)
                    for (int j = 0; j < 3; ++j) Sc[i][j] = RS[i][0] * R[j][0] + RS[i][1] * R[j][1] + RS[i][2] * R[j][2];
                /* inverse VJP (Utils.cuh:417-422) */
                double i00 = conics[idx * 3], i01 = conics[idx * 3 + 1], i11 = conics[idx * 3 + 2];
                double Vm[2][2] = {{v_conics[idx * 3], 0.5 * v_conics[idx * 3 + 1]},
                                   {0.5 * v_conics[idx * 3 + 1], v_conics[idx * 3 + 2]}};
                double Inv[2][2] = {{i00, i01}, {i01, i11}}, T2[2][2], G[2][2];
                for (int i = 0; i < 2; ++i)
                    for (int j = 0; j < 2; ++j) T2[i][j] = Inv[i][0] * Vm[0][j] + Inv[i][1] * Vm[1][j];
                for (int i = 0; i < 2; ++i)
                    for (int j = 0; j < 2; ++j) G[i][j] = -(T2[i][0] * Inv[0][j] + T2[i][1] * Inv[1][j]);
                if (v_comps) { /* add_blur_vjp, Utils.cuh:434-467 */
                    double comp = comps[idx], vc = v_comps[idx];
                    double detc = i00 * i11 - i01 * i01;
                    double vsq = vc * 0.5 / (comp + 1e-6), omc = 1 - comp * comp;
                    G[0][0] += vsq * (omc * i00 - eps2d * detc);
                    G[0][1] += vsq * (omc * i01);
                    G[1][0] += vsq * (omc * i01);
                    G[1][1] += vsq * (omc * i11 - eps2d * detc);
                }
                double x = p[0], y = p[1], z = p[2];
                double J[2][3], vmc[3] = {0, 0, 0};
                double fx = cam.fx, fy = cam.fy, cx = cam.cx, cy = cam.cy;
                double tx = 0, ty = 0, rz = 0, rz2 = 0, rz3 = 0, lxp = 0, lxn = 0, lyp = 0, lyn = 0;
                if (camera_model == 2) {
                    fisheye_jacobian_d(fx, fy, x, y, z, J);
                } else if (camera_model == 1) {
                    J[0][0] = fx; J[0][1] = 0; J[0][2] = 0; J[1][0] = 0; J[1][1] = fy; J[1][2] = 0;
                    vmc[0] += fx * v_means2d[idx * 2];
                    vmc[1] += fy * v_means2d[idx * 2 + 1];
                } else {
                    double tfx = 0.5 * W / fx, tfy = 0.5 * H / fy;
                    lxp = (W - cx) / fx + 0.3 * tfx; lxn = cx / fx + 0.3 * tfx;
                    lyp = (H - cy) / fy + 0.3 * tfy; lyn = cy / fy + 0.3 * tfy;
                    rz = 1.0 / z; rz2 = rz * rz; rz3 = rz2 * rz;
                    tx = z * fmin(lxp, fmax(-lxn, x * rz));
                    ty = z * fmin(lyp, fmax(-lyn, y * rz));
                    J[0][0] = fx * rz; J[0][1] = 0; J[0][2] = -fx * tx * rz2;
                    J[1][0] = 0; J[1][1] = fy * rz; J[1][2] = -fy * ty * rz2;
                    double vx = v_means2d[idx * 2], vy = v_means2d[idx * 2 + 1];
                    vmc[0] += fx * rz * vx;
                    vmc[1] += fy * rz * vy;
                    vmc[2] += -(fx * x * vx + fy * y * vy) * rz2;
                }
                double vSc[3][3], GJ[2][3];
                for (int r = 0; r < 2; ++r)
                    for (int j = 0; j < 3; ++j) GJ[r][j] = G[r][0] * J[0][j] + G[r][1] * J[1][j];
                for (int i = 0; i < 3; ++i)
                    for (int j = 0; j < 3; ++j) vSc[i][j] = J[0][i] * GJ[0][j] + J[1][i] * GJ[1][j];
                if (camera_model == 2) {
                    double JS[2][3], vJ[2][3], vm2[2] = {v_means2d[idx * 2], v_means2d[idx * 2 + 1]};
                    for (int r = 0; r < 2; ++r)
                        for (int j = 0; j < 3; ++j) JS[r][j] = J[r][0] * Sc[0][j] + J[r][1] * Sc[1][j] + J[r][2] * Sc[2][j];
                    for (int r = 0; r < 2; ++r)
                        for (int j = 0; j < 3; ++j) vJ[r][j] = (G[r][0] + G[0][r]) * JS[0][j] + (G[r][1] + G[1][r]) * JS[1][j];
                    fisheye_point_vjp_d(fx, fy, x, y, z, vm2, vJ, vmc);
                } else if (camera_model != 1) {
                    double JS[2][3], vJ[2][3];
                    for (int r = 0; r < 2; ++r)
                        for (int j = 0; j < 3; ++j) JS[r][j] = J[r][0] * Sc[0][j] + J[r][1] * Sc[1][j] + J[r][2] * Sc[2][j];
                    for (int r = 0; r < 2; ++r)
                        for (int j = 0; j < 3; ++j) vJ[r][j] = (G[r][0] + G[0][r]) * JS[0][j] + (G[r][1] + G[1][r]) * JS[1][j];
                    if (x * rz <= lxp && x * rz >= -lxn) vmc[0] += -fx * rz2 * vJ[0][2];
                    else vmc[2] += -fx * rz3 * vJ[0][2] * tx;
                    if (y * rz <= lyp && y * rz >= -lyn) vmc[1] += -fy * rz2 * vJ[1][2];
                    else vmc[2] += -fy * rz3 * vJ[1][2] * ty;
                    vmc[2] += -fx * rz2 * vJ[0][0] - fy * rz2 * vJ[1][1] + 2 * fx * tx * rz3 * vJ[0][2] +
                              2 * fy * ty * rz3 * vJ[1][2];
                }
                vmc[2] += v_depths[idx];
                for (int i = 0; i < 3; ++i) vm[i] += R[0][i] * vmc[0] + R[1][i] * vmc[1] + R[2][i] * vmc[2];
                /* v_S += R^T vSc R */
                double RtG[3][3];
                for (int i = 0; i < 3; ++i)
                    for (int j = 0; j < 3; ++j) RtG[i][j] = R[0][i] * vSc[0][j] + R[1][i] * vSc[1][j] + R[2][i] * vSc[2][j];
                for (int i = 0; i < 3; ++i)
                    for (int j = 0; j < 3; ++j) vS[i][j] += RtG[i][0] * R[0][j] + RtG[i][1] * R[1][j] + RtG[i][2] * R[2][j];
                if (vview_local) {
                    double *vv = vview_local + (b * C + c) * 16;
                    for (int i = 0; i < 3; ++i) {
                        for (int j = 0; j < 3; ++j) {
                            double a = vmc[i] * m[j];
                            /* (G + G^T) R S  with G = vSc */
                            for (int k = 0; k < 3; ++k) a += (vSc[i][k] + vSc[k][i]) * RS[k][j];
                            vv[i * 4 + j] += a;
                        }
                        vv[i * 4 + 3] += vmc[i];
                    }
                }
            }
            if (v_means)
                for (int i = 0; i < 3; ++i) v_means[gi * 3 + i] = (float)vm[i];
            if (covars) {
                if (v_covars) {
                    float *o = v_covars + gi * 6;
                    o[0] = (float)vS[0][0]; o[1] = (float)(vS[0][1] + vS[1][0]); o[2] = (float)(vS[0][2] + vS[2][0]);
                    o[3] = (float)vS[1][1]; o[4] = (float)(vS[1][2] + vS[2][1]); o[5] = (float)vS[2][2];
                }
            } else {
                /* quat_scale_to_covar_vjp, Utils.cuh:259-296 */
                const float *q = quats + gi * 4, *s = scales + gi * 3;
                ora_m3 Rq = quat_rot(q);
                double M[3][3], vM[3][3], vR[3][3], vq[4] = {0, 0, 0, 0}, vs[3];
                for (int i = 0; i < 3; ++i)
                    for (int j = 0; j < 3; ++j) M[i][j] = (double)Rq.m[i][j] * s[j];
                for (int i = 0; i < 3; ++i)
                    for (int j = 0; j < 3; ++j) {
                        double a = 0;
                        for (int k = 0; k < 3; ++k) a += (vS[i][k] + vS[k][i]) * M[k][j];
                        vM[i][j] = a;
                        vR[i][j] = a * s[j];
                    }
                quat_vjp(q, vR, vq);
                for (int j = 0; j < 3; ++j) vs[j] = Rq.m[0][j] * vM[0][j] + Rq.m[1][j] * vM[1][j] + Rq.m[2][j] * vM[2][j];
                if (v_quats)
                    for (int i = 0; i < 4; ++i) v_quats[gi * 4 + i] = (float)vq[i];
                if (v_scales)
                    for (int i = 0; i < 3; ++i) v_scales[gi * 3 + i] = (float)vs[i];
            }
        }
        if (vview_local) {
#pragma omp critical
            for (size_t k = 0; k < (size_t)B * C * 16; ++k) vview[k] += vview_local[k];
            free(vview_local);
        }
    }
    if (v_viewmats) {
        for (size_t k = 0; k < (size_t)B * C * 16; ++k) v_viewmats[k] = (float)vview[k];
        free(vview);
    }
}

/* ------------------------------------------------------------------------ */
/* Spherical harmonics: SphericalHarmonicsCUDA.cu:38-388, bases of degree <= 4 */
static void sh_bases(int deg, double x, double y, double z, double *Y) {
    Y[0] = 0.2820947917738781;
    if (deg < 1) return;
    Y[1] = -0.48860251190292 * y; Y[2] = 0.48860251190292 * z; Y[3] = -0.48860251190292 * x;
    if (deg < 2) return;
    double z2 = z * z, fC1 = x * x - y * y, fS1 = 2 * x * y;
    Y[4] = 0.5462742152960395 * fS1; Y[5] = -1.092548430592079 * z * y;
    Y[6] = 0.9461746957575601 * z2 - 0.3153915652525201; Y[7] = -1.092548430592079 * z * x;
    Y[8] = 0.5462742152960395 * fC1;
    if (deg < 3) return;
    double fC2 = x * fC1 - y * fS1, fS2 = x * fS1 + y * fC1;
    double t0C = -2.285228997322329 * z2 + 0.4570457994644658, t1B = 1.445305721320277 * z;
    Y[9] = -0.5900435899266435 * fS2; Y[10] = t1B * fS1; Y[11] = t0C * y;
    Y[12] = z * (1.865881662950577 * z2 - 1.119528997770346); Y[13] = t0C * x; Y[14] = t1B * fC1;
    Y[15] = -0.5900435899266435 * fC2;
    if (deg < 4) return;
    double fC3 = x * fC2 - y * fS2, fS3 = x * fS2 + y * fC2;
    double t0D = z * (-4.683325804901025 * z2 + 2.007139630671868);
    double t1C = 3.31161143515146 * z2 - 0.47308734787878, t2B = -1.770130769779931 * z;
    Y[16] = 0.6258357354491763 * fS3; Y[17] = t2B * fS2; Y[18] = t1C * fS1; Y[19] = t0D * y;
    Y[20] = 1.984313483298443 * z * Y[12] - 1.006230589874905 * Y[6];
    Y[21] = t0D * x; Y[22] = t1C * fC1; Y[23] = t2B * fC2; Y[24] = 0.6258357354491763 * fC3;
}

static void unit_dir(const float *d, double *x, double *y, double *z, double *inv) {
    double l = (double)d[0] * d[0] + (double)d[1] * d[1] + (double)d[2] * d[2];
    *inv = 1.0 / sqrt(l);
    *x = d[0] * *inv; *y = d[1] * *inv; *z = d[2] * *inv;
}

void ora_sh_fwd(int deg, long long n, int K, const float *dirs, const float *coeffs,
                const uint8_t *masks, float *colors) {
#pragma omp parallel for schedule(static)
    for (long long e = 0; e < n; ++e) {
        colors[e * 3] = colors[e * 3 + 1] = colors[e * 3 + 2] = 0.f;
        if (masks && !masks[e]) continue;
        double x, y, z, inv, Y[25];
        unit_dir(dirs + e * 3, &x, &y, &z, &inv);
        sh_bases(deg, x, y, z, Y);
        int nb = (deg + 1) * (deg + 1);
        for (int c = 0; c < 3; ++c) {
            double acc = 0;
            for (int k = 0; k < nb; ++k) acc += Y[k] * coeffs[(e * K + k) * 3 + c];
            colors[e * 3 + c] = (float)acc;
        }
    }
}

/* Backward by central differences of the polynomial bases is not used: the
 * derivatives below are those of Y_k(x, y, z) treating the unit direction's
 * components as free variables, followed by the normalisation VJP, as in
 * SphericalHarmonicsCUDA.cu:130-388. They are evaluated by forward-mode dual
 * numbers over sh_bases to keep this restatement independent of the kernel's
 * hand-derived gradient formulas. */
static void sh_bases_dual(int deg, dual3 x, dual3 y, dual3 z, dual3 *Y) {
    Y[0] = dc(0.2820947917738781);
    if (deg < 1) return;
    Y[1] = dscale(-0.48860251190292, y); Y[2] = dscale(0.48860251190292, z); Y[3] = dscale(-0.48860251190292, x);
    if (deg < 2) return;
    dual3 z2 = dmul(z, z), fC1 = dsub(dmul(x, x), dmul(y, y)), fS1 = dscale(2, dmul(x, y));
    Y[4] = dscale(0.5462742152960395, fS1); Y[5] = dscale(-1.092548430592079, dmul(z, y));
    Y[6] = dsub(dscale(0.9461746957575601, z2), dc(0.3153915652525201));
    Y[7] = dscale(-1.092548430592079, dmul(z, x)); Y[8] = dscale(0.5462742152960395, fC1);
    if (deg < 3) return;
    dual3 fC2 = dsub(dmul(x, fC1), dmul(y, fS1)), fS2 = dadd(dmul(x, fS1), dmul(y, fC1));
    dual3 t0C = dadd(dscale(-2.285228997322329, z2), dc(0.4570457994644658));
    dual3 t1B = dscale(1.445305721320277, z);
    Y[9] = dscale(-0.5900435899266435, fS2); Y[10] = dmul(t1B, fS1); Y[11] = dmul(t0C, y);
    Y[12] = dmul(z, dsub(dscale(1.865881662950577, z2), dc(1.119528997770346)));
    Y[13] = dmul(t0C, x); Y[14] = dmul(t1B, fC1); Y[15] = dscale(-0.5900435899266435, fC2);
    if (deg < 4) return;
    dual3 fC3 = dsub(dmul(x, fC2), dmul(y, fS2)), fS3 = dadd(dmul(x, fS2), dmul(y, fC2));
    dual3 t0D = dmul(z, dadd(dscale(-4.683325804901025, z2), dc(2.007139630671868)));
    dual3 t1C = dsub(dscale(3.31161143515146, z2), dc(0.47308734787878));
    dual3 t2B = dscale(-1.770130769779931, z);
    Y[16] = dscale(0.6258357354491763, fS3); Y[17] = dmul(t2B, fS2); Y[18] = dmul(t1C, fS1);
    Y[19] = dmul(t0D, y);
    Y[20] = dsub(dscale(1.984313483298443, dmul(z, Y[12])), dscale(1.006230589874905, Y[6]));
    Y[21] = dmul(t0D, x); Y[22] = dmul(t1C, fC1); Y[23] = dmul(t2B, fC2);
    Y[24] = dscale(0.6258357354491763, fC3);
}

void ora_sh_bwd(int deg, long long n, int K, const float *dirs, const float *coeffs,
                const uint8_t *masks, const float *v_colors, float *v_coeffs, float *v_dirs) {
#pragma omp parallel for schedule(static)
    for (long long e = 0; e < n; ++e) {
        for (int k = 0; k < K * 3; ++k) v_coeffs[e * K * 3 + k] = 0.f;
        if (v_dirs) v_dirs[e * 3] = v_dirs[e * 3 + 1] = v_dirs[e * 3 + 2] = 0.f;
        if (masks && !masks[e]) continue;
        double x, y, z, inv;
        unit_dir(dirs + e * 3, &x, &y, &z, &inv);
        dual3 dx = {x, {1, 0, 0}}, dy = {y, {0, 1, 0}}, dz = {z, {0, 0, 1}};
        dual3 Y[25];
        sh_bases_dual(deg, dx, dy, dz, Y);
        int nb = (deg + 1) * (deg + 1);
        const float *vc = v_colors + e * 3;
        double g[3] = {0, 0, 0};
        for (int k = 0; k < nb; ++k) {
            double w = 0;
            for (int c = 0; c < 3; ++c) {
                v_coeffs[(e * K + k) * 3 + c] = (float)(Y[k].v * vc[c]);
                w += coeffs[(e * K + k) * 3 + c] * (double)vc[c];
            }
            for (int i = 0; i < 3; ++i) g[i] += w * Y[k].d[i];
        }
        if (v_dirs && deg > 0) {
            double d = g[0] * x + g[1] * y + g[2] * z;
            v_dirs[e * 3] = (float)((g[0] - d * x) * inv);
            v_dirs[e * 3 + 1] = (float)((g[1] - d * y) * inv);
            v_dirs[e * 3 + 2] = (float)((g[2] - d * z) * inv);
        }
    }
}

/* ------------------------------------------------------------------------ */
/* Tile intersection (IntersectTile.cu), bit-exact via detmath.h */
typedef struct {
    int64_t *keys;
    int32_t *ids;
    int64_t cur;
    int64_t hi;
    int64_t depth;
    int32_t fid;
} ora_sink;

static void sink_put(ora_sink *s, int64_t tile) {
    if (!s) return;
    s->keys[s->cur] = s->hi | (tile << 32) | s->depth;
    s->ids[s->cur] = s->fid;
    s->cur++;
}

static void ell_line(float A, float B, float C, float disc, float t, float px, float py, int isY,
                     float coord, float *lo, float *hi) {
    float pu = isY ? py : px, pv = isY ? px : py, co = isY ? A : C;
    float h = DET_SUB(coord, pu);
    float sq = DET_SQRT(DET_ADD(DET_MUL(DET_MUL(disc, h), h), DET_MUL(t, co)));
    float bh = DET_MUL(-B, h);
    *lo = DET_ADD(DET_DIV(DET_SUB(bh, sq), co), pv);
    *hi = DET_ADD(DET_DIV(DET_ADD(bh, sq), co), pv);
}

static int imin(int a, int b) { return a < b ? a : b; }
static int imax(int a, int b) { return a > b ? a : b; }

static uint32_t accutile(float mx, float my, float A, float B, float C, float op, int ts_i,
                         int tw, int th, ora_sink *s) {
    float disc = DET_SUB(DET_MUL(B, B), DET_MUL(A, C));
    float t = det_fmin(ORA_EXTEND * ORA_EXTEND, DET_MUL(2.0f, det_logf(DET_DIV(op, ORA_ALPHA_THRESHOLD))));
    float ntd = DET_DIV(-t, disc);
    float xe = DET_SQRT(DET_MUL(ntd, C)), ye = DET_SQRT(DET_MUL(ntd, A));
    float bminx = DET_SUB(mx, xe), bminy = DET_SUB(my, ye), bmaxx = DET_ADD(mx, xe), bmaxy = DET_ADD(my, ye);
    float bxc = DET_DIV(DET_MUL(B, xe), C), bya = DET_DIV(DET_MUL(B, ye), A);
    float aminx = DET_ADD(my, bxc), aminy = DET_ADD(mx, bya);
    float amaxx = DET_SUB(my, bxc), amaxy = DET_SUB(mx, bya);
    float ts = (float)ts_i;
    int rminx = imax(0, imin(tw, det_f2i_rz(DET_DIV(bminx, ts))));
    int rminy = imax(0, imin(th, det_f2i_rz(DET_DIV(bminy, ts))));
    int rmaxx = imax(0, imin(tw, det_f2i_rz(DET_ADD(DET_DIV(bmaxx, ts), 1.f))));
    int rmaxy = imax(0, imin(th, det_f2i_rz(DET_ADD(DET_DIV(bmaxy, ts), 1.f))));
    int ysp = rmaxy - rminy, xsp = rmaxx - rminx;
    if (ysp * xsp == 0) return 0;
    int isY = ysp < xsp;
    if (isY) {
        int ti; float tf;
        ti = rminx; rminx = rminy; rminy = ti;
        ti = rmaxx; rmaxx = rmaxy; rmaxy = ti;
        tf = bminx; bminx = bminy; bminy = tf;
        tf = bmaxx; bmaxx = bmaxy; bmaxy = tf;
        tf = aminx; aminx = aminy; aminy = tf;
        tf = amaxx; amaxx = amaxy; amaxy = tf;
    }
    uint32_t count = 0;
    float hi_lo = bmaxy, hi_hi = bminy, lo_lo, lo_hi;
    float min_line = DET_MUL((float)rminx, ts);
    if (bminx <= min_line) ell_line(A, B, C, disc, t, mx, my, isY, min_line, &lo_lo, &lo_hi);
    else { lo_lo = hi_lo; lo_hi = hi_hi; }
    for (int u = rminx; u < rmaxx; ++u) {
        float max_line = DET_ADD(min_line, ts);
        if (max_line <= bmaxx) ell_line(A, B, C, disc, t, mx, my, isY, max_line, &hi_lo, &hi_hi);
        float emin = (min_line <= aminy && aminy < max_line) ? bminy : det_fmin(lo_lo, hi_lo);
        float emax = (min_line <= amaxy && amaxy < max_line) ? bmaxy : det_fmax(lo_hi, hi_hi);
        int v0 = imax(rminy, imin(rmaxy, det_f2i_rz(DET_DIV(emin, ts))));
        int v1 = imin(rmaxy, imax(rminy, det_f2i_rz(DET_ADD(DET_DIV(emax, ts), 1.f))));
        if (v1 > v0) {
            count += (uint32_t)(v1 - v0);
            for (int v = v0; v < v1; ++v) sink_put(s, isY ? (int64_t)u * tw + v : (int64_t)v * tw + u);
        }
        lo_lo = hi_lo; lo_hi = hi_hi;
        min_line = max_line;
    }
    return count;
}

static uint32_t aabb(float mx, float my, int rx, int ry, int ts_i, int tw, int th, ora_sink *s) {
    float ts = (float)ts_i;
    float trx = DET_DIV((float)rx, ts), try_ = DET_DIV((float)ry, ts);
    float tx = DET_DIV(mx, ts), ty = DET_DIV(my, ts);
    int x0 = imin(imax(0, det_f2i_rz(floorf(DET_SUB(tx, trx)))), tw);
    int y0 = imin(imax(0, det_f2i_rz(floorf(DET_SUB(ty, try_)))), th);
    int x1 = imin(imax(0, det_f2i_rz(ceilf(DET_ADD(tx, trx)))), tw);
    int y1 = imin(imax(0, det_f2i_rz(ceilf(DET_ADD(ty, try_)))), th);
    for (int y = y0; y < y1; ++y)
        for (int x = x0; x < x1; ++x) sink_put(s, (int64_t)y * tw + x);
    return (uint32_t)((y1 - y0) * (x1 - x0));
}

static uint32_t bitlen(uint64_t v) { uint32_t b = 0; while (v) { ++b; v >>= 1; } return b; }

static uint32_t splat(long long idx, const float *means2d, const int32_t *radii,
                      const float *conics, const float *opac, int ts, int tw, int th, ora_sink *s) {
    int rx = radii[idx * 2], ry = radii[idx * 2 + 1];
    if (rx <= 0 || ry <= 0) return 0;
    float mx = means2d[idx * 2], my = means2d[idx * 2 + 1];
    if (conics && opac)
        return accutile(mx, my, conics[idx * 3], conics[idx * 3 + 1], conics[idx * 3 + 2], opac[idx], ts, tw, th, s);
    return aabb(mx, my, rx, ry, ts, tw, th, s);
}

void ora_isect_count(long long n, const float *means2d, const int32_t *radii, const float *conics,
                     const float *opac, int ts, int tw, int th, int32_t *tiles_per_gauss) {
#pragma omp parallel for schedule(dynamic, 1024)
    for (long long i = 0; i < n; ++i)
        tiles_per_gauss[i] = (int32_t)splat(i, means2d, radii, conics, opac, ts, tw, th, NULL);
}

/* image_ids: NULL for the dense layout (image = idx / N) */
void ora_isect_emit(long long n, int N, const int64_t *image_ids, int I, const float *means2d,
                    const int32_t *radii, const float *depths, const float *conics,
                    const float *opac, int ts, int tw, int th, const int64_t *cum,
                    int64_t *keys, int32_t *ids) {
    uint32_t tbits = bitlen((uint64_t)tw * th);
    (void)I;
#pragma omp parallel for schedule(dynamic, 1024)
    for (long long i = 0; i < n; ++i) {
        ora_sink s;
        s.keys = keys; s.ids = ids;
        s.cur = i == 0 ? 0 : cum[i - 1];
        int64_t iid = image_ids ? image_ids[i] : (int64_t)(i / N);
        s.hi = iid << (32 + tbits);
        s.depth = (int64_t)det_f2u(depths[i]);
        s.fid = (int32_t)i;
        splat(i, means2d, radii, conics, opac, ts, tw, th, &s);
    }
}

/* Stable sort of (key, value) pairs == sort by (key, original position). */
typedef struct { int64_t k; int64_t pos; int32_t v; } ora_kv;
static int kv_cmp(const void *a, const void *b) {
    const ora_kv *x = (const ora_kv *)a, *y = (const ora_kv *)b;
    if (x->k != y->k) return x->k < y->k ? -1 : 1;
    return x->pos < y->pos ? -1 : (x->pos > y->pos);
}
void ora_sort_pairs(long long n, int64_t *keys, int32_t *vals) {
    ora_kv *t = (ora_kv *)malloc(sizeof(ora_kv) * (size_t)(n > 0 ? n : 1));
    for (long long i = 0; i < n; ++i) { t[i].k = keys[i]; t[i].pos = i; t[i].v = vals[i]; }
    qsort(t, (size_t)n, sizeof(ora_kv), kv_cmp);
    for (long long i = 0; i < n; ++i) { keys[i] = t[i].k; vals[i] = t[i].v; }
    free(t);
}

void ora_isect_offsets(long long n, const int64_t *keys, int I, int tw, int th, int32_t *offsets) {
    uint32_t ntiles = (uint32_t)(tw * th), tbits = bitlen(ntiles);
    long long total = (long long)I * ntiles;
    if (n == 0) { for (long long i = 0; i < total; ++i) offsets[i] = 0; return; }
    for (long long i = 0; i < total; ++i) offsets[i] = (int32_t)n;
    long long prev = -1;
    for (long long k = 0; k < n; ++k) {
        int64_t hi = keys[k] >> 32;
        long long id = (hi >> tbits) * (long long)ntiles + (hi & ((1ll << tbits) - 1));
        for (long long i = prev + 1; i <= id; ++i) offsets[i] = (int32_t)k;
        prev = id;
    }
}

/* ------------------------------------------------------------------------ */
/* Rasterization */
typedef struct {
    int I, CH, W, H, ts, tw, th;
    const float *means2d, *conics, *colors, *opac, *bg;
    const uint8_t *masks;
    const int32_t *offsets, *fids;
    long long n_isects;
} ora_rp;

static void tile_range(const ora_rp *p, int img, int tile, int32_t *s, int32_t *e) {
    const int32_t *off = p->offsets + (size_t)img * p->tw * p->th;
    *s = off[tile];
    *e = (img == p->I - 1 && tile == p->tw * p->th - 1) ? (int32_t)p->n_isects : off[tile + 1];
}

void ora_raster_fwd(int I, int CH, const float *means2d, const float *conics, const float *colors,
                    const float *opac, const float *bg, const uint8_t *masks, int W, int H, int ts,
                    int tw, int th, const int32_t *offsets, const int32_t *fids, long long n_isects,
                    float *renders, float *alphas, int32_t *last_ids) {
    ora_rp p = {I, CH, W, H, ts, tw, th, means2d, conics, colors, opac, bg, masks, offsets, fids, n_isects};
#pragma omp parallel
    {
    float *pa = (float *)malloc(sizeof(float) * (size_t)CH);
#pragma omp for schedule(dynamic, 1)
    for (long long it = 0; it < (long long)I * tw * th; ++it) {
        int img = (int)(it / (tw * th)), tile = (int)(it % (tw * th));
        int ty = tile / tw, tx = tile % tw;
        int32_t s, e;
        tile_range(&p, img, tile, &s, &e);
        const float *bgi = bg ? bg + (size_t)img * CH : NULL;
        int masked = masks && !masks[(size_t)img * tw * th + tile];
        for (int py = ty * ts; py < imin((ty + 1) * ts, H); ++py)
            for (int px = tx * ts; px < imin((tx + 1) * ts, W); ++px) {
                size_t pix = ((size_t)img * H + py) * W + px;
                float *out = renders + pix * CH;
                if (masked) {
                    for (int c = 0; c < CH; ++c) out[c] = bgi ? bgi[c] : 0.f;
                    alphas[pix] = 0.f; last_ids[pix] = 0;
                    continue;
                }
                float fx = (float)px + 0.5f, fy = (float)py + 0.5f, T = 1.f;
                int32_t cur = 0;
                for (int c = 0; c < CH; ++c) pa[c] = 0.f;
                for (int32_t k = s; k < e; ++k) {
                    int32_t g = fids[k];
                    const float *cn = conics + (size_t)g * 3;
                    float dx = means2d[(size_t)g * 2] - fx, dy = means2d[(size_t)g * 2 + 1] - fy;
                    float sigma = 0.5f * (cn[0] * dx * dx + cn[2] * dy * dy) + cn[1] * dx * dy;
                    float alpha = fminf(ORA_MAX_ALPHA, opac[g] * expf(-sigma));
                    if (sigma < 0.f || alpha < ORA_ALPHA_THRESHOLD) continue;
                    float nT = T * (1.f - alpha);
                    if (nT <= ORA_T_THRESHOLD) break;
                    float vis = alpha * T;
                    for (int c = 0; c < CH; ++c) pa[c] += colors[(size_t)g * CH + c] * vis;
                    cur = k;
                    T = nT;
                }
                alphas[pix] = 1.f - T;
                for (int c = 0; c < CH; ++c) out[c] = bgi ? pa[c] + T * bgi[c] : pa[c];
                last_ids[pix] = cur;
            }
    }
    free(pa);
    }
}

void ora_raster_bwd(int I, int CH, const float *means2d, const float *conics, const float *colors,
                    const float *opac, const float *bg, const uint8_t *masks, int W, int H, int ts,
                    int tw, int th, const int32_t *offsets, const int32_t *fids, long long n_isects,
                    const float *render_alphas, int t_from_alphas, const int32_t *last_ids,
                    const float *v_renders, const float *v_alphas, long long n_splats,
                    float *v_means2d_abs, float *v_means2d, float *v_conics, float *v_colors,
                    float *v_opac) {
    ora_rp p = {I, CH, W, H, ts, tw, th, means2d, conics, colors, opac, bg, masks, offsets, fids, n_isects};
    /* per-splat gradient accumulators in double: 2 xy, 3 conic, 1 opacity, 2 abs, CH colour */
    const int G = 8 + CH;
    double *acc = (double *)calloc((size_t)n_splats * G, sizeof(double));
#pragma omp parallel
    {
        double *buf = (double *)malloc(sizeof(double) * (size_t)CH * 2);
#pragma omp for schedule(dynamic, 1)
        for (long long it = 0; it < (long long)I * tw * th; ++it) {
            int img = (int)(it / (tw * th)), tile = (int)(it % (tw * th));
            if (masks && !masks[(size_t)img * tw * th + tile]) continue;
            int ty = tile / tw, tx = tile % tw;
            int32_t s, e;
            tile_range(&p, img, tile, &s, &e);
            const float *bgi = bg ? bg + (size_t)img * CH : NULL;
            for (int py = ty * ts; py < imin((ty + 1) * ts, H); ++py)
                for (int px = tx * ts; px < imin((tx + 1) * ts, W); ++px) {
                    size_t pix = ((size_t)img * H + py) * W + px;
                    float fx = (float)px + 0.5f, fy = (float)py + 0.5f;
                    int32_t last = last_ids[pix];
                    /* Final transmittance: by default recomputed in double over the
                     * pairs the forward kept (the exact product the PyTorch path's
                     * autograd differentiates); with t_from_alphas, 1 - alpha as in
                     * RasterizeToPixels3DGSBwd.cu:130. */
                    double Tf = 1.0;
                    if (t_from_alphas) {
                        Tf = 1.0 - (double)render_alphas[pix];
                    } else {
                        for (int32_t k = s; k <= imin(e - 1, last); ++k) {
                            int32_t g = fids[k];
                            const float *cn = conics + (size_t)g * 3;
                            float dx = means2d[(size_t)g * 2] - fx, dy = means2d[(size_t)g * 2 + 1] - fy;
                            float sigma = 0.5f * (cn[0] * dx * dx + cn[2] * dy * dy) + cn[1] * dx * dy;
                            float alpha = fminf(ORA_MAX_ALPHA, opac[g] * expf(-sigma));
                            if (sigma < 0.f || alpha < ORA_ALPHA_THRESHOLD) continue;
                            Tf *= 1.0 - (double)alpha;
                        }
                    }
                    double T = Tf;
                    const float *vc = v_renders + pix * CH;
                    double va = v_alphas[pix], bgd = 0;
                    double *bb = buf;
                    for (int c = 0; c < CH; ++c) { bb[c] = 0; if (bgi) bgd += (double)bgi[c] * vc[c]; }
                    for (int32_t k = imin(e - 1, last); k >= s; --k) {
                        int32_t g = fids[k];
                        const float *cn = conics + (size_t)g * 3;
                        float dx = means2d[(size_t)g * 2] - fx, dy = means2d[(size_t)g * 2 + 1] - fy;
                        float sigma = 0.5f * (cn[0] * dx * dx + cn[2] * dy * dy) + cn[1] * dx * dy;
                        float visf = expf(-sigma);
                        float alpha = fminf(ORA_MAX_ALPHA, opac[g] * visf);
                        if (sigma < 0.f || alpha < ORA_ALPHA_THRESHOLD) continue;
                        double ra = 1.0 / fmax(ORA_MIN_1MA, 1.0 - (double)alpha);
                        T *= ra;
                        double fac = alpha * T, v_alpha = 0;
                        double *a = acc + (size_t)g * G;
                        const float *col = colors + (size_t)g * CH;
                        for (int c = 0; c < CH; ++c) {
                            double d = fac * vc[c];
#pragma omp atomic
                            a[8 + c] += d;
                            v_alpha += (col[c] * T - bb[c] * ra) * vc[c];
                        }
                        v_alpha += Tf * ra * va;
                        if (bgi) v_alpha += -Tf * ra * bgd;
                        if (opac[g] * visf <= ORA_MAX_ALPHA) {
                            double vs = -(double)opac[g] * visf * v_alpha;
                            double gx = vs * ((double)cn[0] * dx + (double)cn[1] * dy);
                            double gy = vs * ((double)cn[1] * dx + (double)cn[2] * dy);
#pragma omp atomic
                            a[0] += gx;
#pragma omp atomic
                            a[1] += gy;
#pragma omp atomic
                            a[2] += 0.5 * vs * dx * dx;
#pragma omp atomic
                            a[3] += vs * dx * dy;
#pragma omp atomic
                            a[4] += 0.5 * vs * dy * dy;
#pragma omp atomic
                            a[5] += visf * v_alpha;
#pragma omp atomic
                            a[6] += fabs(gx);
#pragma omp atomic
                            a[7] += fabs(gy);
                        }
                        for (int c = 0; c < CH; ++c) bb[c] += col[c] * fac;
                    }
                }
        }
        free(buf);
    }
    for (long long g = 0; g < n_splats; ++g) {
        const double *a = acc + (size_t)g * G;
        v_means2d[g * 2] = (float)a[0]; v_means2d[g * 2 + 1] = (float)a[1];
        v_conics[g * 3] = (float)a[2]; v_conics[g * 3 + 1] = (float)a[3]; v_conics[g * 3 + 2] = (float)a[4];
        v_opac[g] = (float)a[5];
        if (v_means2d_abs) { v_means2d_abs[g * 2] = (float)a[6]; v_means2d_abs[g * 2 + 1] = (float)a[7]; }
        for (int c = 0; c < CH; ++c) v_colors[g * CH + c] = (float)a[8 + c];
    }
    free(acc);
}

/* ------------------------------------------------------------------------ */
void ora_adam(long long N, long long D, float *param, const float *grad, float *m, float *v,
              const uint8_t *valid, float lr, float b1, float b2, float eps) {
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < N * D; ++i) {
        if (valid && !valid[i / D]) continue;
        float g = grad[i];
        float mm = b1 * m[i] + (1.0f - b1) * g;
        float vv = b2 * v[i] + (1.0f - b2) * g * g;
        param[i] += -lr * mm / (sqrtf(vv) + eps);
        m[i] = mm;
        v[i] = vv;
    }
}

/* ------------------------------------------------------------------------ */
/* quat_scale_to_covar_preci: QuatScaleToCovarCUDA.cu:36-292, Utils.cuh:223-341.
 * Forward in float in the reference's order; backward in double. */
static void store_sym3(float *o, const double A[3][3], int triu) {
    if (triu) {
        o[0] = (float)A[0][0]; o[1] = (float)A[0][1]; o[2] = (float)A[0][2];
        o[3] = (float)A[1][1]; o[4] = (float)A[1][2]; o[5] = (float)A[2][2];
    } else {
        for (int i = 0; i < 3; ++i)
            for (int j = 0; j < 3; ++j) o[i * 3 + j] = (float)A[i][j];
    }
}

void ora_covar_preci_fwd(long long n, const float *quats, const float *scales, int triu, float *covars,
                         float *precis) {
    int w = triu ? 6 : 9;
    for (long long i = 0; i < n; ++i) {
        ora_m3 R = quat_rot(quats + i * 4);
        const float *s = scales + i * 3;
        for (int which = 0; which < 2; ++which) {
            float *out = which == 0 ? covars : precis;
            if (!out) continue;
            ora_m3 M;
            for (int a = 0; a < 3; ++a)
                for (int b = 0; b < 3; ++b) M.m[a][b] = R.m[a][b] * (which == 0 ? s[b] : 1.f / s[b]);
            ora_m3 P = m3mul(M, m3t(M));
            double A[3][3];
            for (int a = 0; a < 3; ++a)
                for (int b = 0; b < 3; ++b) A[a][b] = P.m[a][b];
            store_sym3(out + i * w, A, triu);
        }
    }
}

static void load_grad3(const float *g, int triu, double G[3][3]) {
    if (triu) {
        G[0][0] = g[0]; G[0][1] = G[1][0] = 0.5 * g[1]; G[0][2] = G[2][0] = 0.5 * g[2];
        G[1][1] = g[3]; G[1][2] = G[2][1] = 0.5 * g[4]; G[2][2] = g[5];
    } else {
        for (int i = 0; i < 3; ++i)
            for (int j = 0; j < 3; ++j) G[i][j] = g[i * 3 + j];
    }
}

void ora_covar_preci_bwd(long long n, const float *quats, const float *scales, int triu, const float *v_covars,
                         const float *v_precis, float *v_quats, float *v_scales) {
    int w = triu ? 6 : 9;
    for (long long i = 0; i < n; ++i) {
        const float *q = quats + i * 4, *s = scales + i * 3;
        ora_m3 Rf = quat_rot(q);
        double vq[4] = {0, 0, 0, 0}, vs[3] = {0, 0, 0};
        for (int which = 0; which < 2; ++which) {
            const float *g = which == 0 ? v_covars : v_precis;
            if (!g) continue;
            double G[3][3], M[3][3], vM[3][3], vR[3][3], sc[3];
            load_grad3(g + i * w, triu, G);
            for (int b = 0; b < 3; ++b) sc[b] = which == 0 ? (double)s[b] : 1.0 / (double)s[b];
            for (int a = 0; a < 3; ++a)
                for (int b = 0; b < 3; ++b) M[a][b] = (double)Rf.m[a][b] * sc[b];
            for (int a = 0; a < 3; ++a)
                for (int b = 0; b < 3; ++b) {
                    double acc = 0;
                    for (int k = 0; k < 3; ++k) acc += (G[a][k] + G[k][a]) * M[k][b];
                    vM[a][b] = acc;
                    vR[a][b] = acc * sc[b];
                }
            quat_vjp(q, vR, vq);
            for (int b = 0; b < 3; ++b) {
                double d = Rf.m[0][b] * vM[0][b] + Rf.m[1][b] * vM[1][b] + Rf.m[2][b] * vM[2][b];
                vs[b] += which == 0 ? d : -sc[b] * sc[b] * d;
            }
        }
        for (int k = 0; k < 4; ++k) v_quats[i * 4 + k] = (float)vq[k];
        for (int k = 0; k < 3; ++k) v_scales[i * 3 + k] = (float)vs[k];
    }
}

/* ------------------------------------------------------------------------ */
/* proj: ProjectionEWASimple.cu:36-317 with Utils.cuh:473-801. cov2d = J S J^T,
 * dL/dS = J^T G J, dL/dJ = G J S^T + G^T J S (the PyTorch form of the reference,
 * _torch_impl.py:42-211). Forward float, backward double. */
void ora_proj_fwd(int B, int C, int N, const float *means, const float *covars, const float *Ks, int W, int H,
                  int model, float *means2d, float *covars2d) {
    for (long long i = 0; i < (long long)B * C * N; ++i) {
        long long bc = i / N;
        ora_cam cam;
        memset(&cam, 0, sizeof(cam));
        const float *K = Ks + bc * 9;
        cam.fx = K[0]; cam.cx = K[2]; cam.fy = K[4]; cam.cy = K[5];
        const float *m = means + i * 3, *S = covars + i * 9;
        float J[2][3], mx, my;
        proj_jacobian(model, &cam, W, H, m[0], m[1], m[2], J, &mx, &my);
        float JS[2][3];
        for (int r = 0; r < 2; ++r)
            for (int j = 0; j < 3; ++j) JS[r][j] = J[r][0] * S[j] + J[r][1] * S[3 + j] + J[r][2] * S[6 + j];
        for (int r = 0; r < 2; ++r)
            for (int c = 0; c < 2; ++c)
                covars2d[i * 4 + r * 2 + c] = JS[r][0] * J[c][0] + JS[r][1] * J[c][1] + JS[r][2] * J[c][2];
        means2d[i * 2] = mx;
        means2d[i * 2 + 1] = my;
    }
}

void ora_proj_bwd(int B, int C, int N, const float *means, const float *covars, const float *Ks, int W, int H,
                  int model, const float *v_means2d, const float *v_covars2d, float *v_means, float *v_covars) {
    for (long long i = 0; i < (long long)B * C * N; ++i) {
        long long bc = i / N;
        const float *K = Ks + bc * 9;
        double fx = K[0], cx = K[2], fy = K[4], cy = K[5];
        double x = means[i * 3], y = means[i * 3 + 1], z = means[i * 3 + 2];
        double S[3][3], G[2][2] = {{v_covars2d[i * 4], v_covars2d[i * 4 + 1]}, {v_covars2d[i * 4 + 2], v_covars2d[i * 4 + 3]}};
        double vm2[2] = {v_means2d[i * 2], v_means2d[i * 2 + 1]};
        for (int a = 0; a < 3; ++a)
            for (int b = 0; b < 3; ++b) S[a][b] = covars[i * 9 + a * 3 + b];
        double J[2][3], vmc[3] = {0, 0, 0};
        double tx = 0, ty = 0, rz = 0, rz2 = 0, rz3 = 0, lxp = 0, lxn = 0, lyp = 0, lyn = 0;
        if (model == 2) {
            fisheye_jacobian_d(fx, fy, x, y, z, J);
        } else if (model == 1) {
            J[0][0] = fx; J[0][1] = 0; J[0][2] = 0; J[1][0] = 0; J[1][1] = fy; J[1][2] = 0;
            vmc[0] = fx * vm2[0];
            vmc[1] = fy * vm2[1];
        } else {
            double tfx = 0.5 * W / fx, tfy = 0.5 * H / fy;
            lxp = (W - cx) / fx + 0.3 * tfx; lxn = cx / fx + 0.3 * tfx;
            lyp = (H - cy) / fy + 0.3 * tfy; lyn = cy / fy + 0.3 * tfy;
            rz = 1.0 / z; rz2 = rz * rz; rz3 = rz2 * rz;
            tx = z * fmin(lxp, fmax(-lxn, x * rz));
            ty = z * fmin(lyp, fmax(-lyn, y * rz));
            J[0][0] = fx * rz; J[0][1] = 0; J[0][2] = -fx * tx * rz2;
            J[1][0] = 0; J[1][1] = fy * rz; J[1][2] = -fy * ty * rz2;
            vmc[0] = fx * rz * vm2[0];
            vmc[1] = fy * rz * vm2[1];
            vmc[2] = -(fx * x * vm2[0] + fy * y * vm2[1]) * rz2;
        }
        double GJ[2][3];
        for (int r = 0; r < 2; ++r)
            for (int j = 0; j < 3; ++j) GJ[r][j] = G[r][0] * J[0][j] + G[r][1] * J[1][j];
        for (int a = 0; a < 3; ++a)
            for (int b = 0; b < 3; ++b) v_covars[i * 9 + a * 3 + b] = (float)(J[0][a] * GJ[0][b] + J[1][a] * GJ[1][b]);
        double JSt[2][3], JS[2][3], vJ[2][3];
        for (int r = 0; r < 2; ++r)
            for (int j = 0; j < 3; ++j) {
                JSt[r][j] = J[r][0] * S[j][0] + J[r][1] * S[j][1] + J[r][2] * S[j][2];
                JS[r][j] = J[r][0] * S[0][j] + J[r][1] * S[1][j] + J[r][2] * S[2][j];
            }
        for (int r = 0; r < 2; ++r)
            for (int j = 0; j < 3; ++j)
                vJ[r][j] = G[r][0] * JSt[0][j] + G[r][1] * JSt[1][j] + G[0][r] * JS[0][j] + G[1][r] * JS[1][j];
        if (model == 2) {
            fisheye_point_vjp_d(fx, fy, x, y, z, vm2, vJ, vmc);
        } else if (model == 0) {
            if (x * rz <= lxp && x * rz >= -lxn) vmc[0] += -fx * rz2 * vJ[0][2];
            else vmc[2] += -fx * rz3 * vJ[0][2] * tx;
            if (y * rz <= lyp && y * rz >= -lyn) vmc[1] += -fy * rz2 * vJ[1][2];
            else vmc[2] += -fy * rz3 * vJ[1][2] * ty;
            vmc[2] += -fx * rz2 * vJ[0][0] - fy * rz2 * vJ[1][1] + 2 * fx * tx * rz3 * vJ[0][2] +
                      2 * fy * ty * rz3 * vJ[1][2];
        }
        for (int k = 0; k < 3; ++k) v_means[i * 3 + k] = (float)vmc[k];
    }
}

/* ------------------------------------------------------------------------ */
/* rasterize_to_indices_in_range: RasterizeToIndices3DGS.cu:36-200. Pass
 * gids/pids NULL to count only (counts[I*H*W]); with them, the pairs are written
 * at the pixel's exclusive prefix of counts (which the caller passes in
 * `starts`), front to back. libm expf (the kernel uses __expf). */
void ora_raster_indices(int range_start, int range_end, int I, int N, long long n_isects, const float *means2d,
                        const float *conics, const float *opac, int W, int H, int ts, int tw, int th,
                        const int32_t *offsets, const int32_t *fids, const float *trans_in, int32_t *counts,
                        const int64_t *starts, int64_t *gids, int64_t *pids) {
    const int bs = ts * ts;
    for (int img = 0; img < I; ++img)
        for (int tile = 0; tile < tw * th; ++tile) {
            int s0 = offsets[(size_t)img * tw * th + tile];
            int s1 = (img == I - 1 && tile == tw * th - 1) ? (int)n_isects : offsets[(size_t)img * tw * th + tile + 1];
            int nb = (s1 - s0 + bs - 1) / bs;
            if (range_start >= nb) continue;
            int b_end = range_end < nb ? range_end : nb;
            for (int ly = 0; ly < ts; ++ly)
                for (int lx = 0; lx < ts; ++lx) {
                    int i = (tile / tw) * ts + ly, j = (tile % tw) * ts + lx;
                    if (i >= H || j >= W) continue;
                    size_t gp = (size_t)img * H * W + (size_t)i * W + j;
                    float px = (float)j + 0.5f, py = (float)i + 0.5f;
                    float T = trans_in[gp];
                    int cnt = 0, done = 0;
                    for (int k = s0 + range_start * bs; k < s0 + b_end * bs && k < s1 && !done; ++k) {
                        int g = fids[k];
                        float dx = means2d[(size_t)g * 2] - px, dy = means2d[(size_t)g * 2 + 1] - py;
                        const float *c = conics + (size_t)g * 3;
                        float sigma = 0.5f * (c[0] * dx * dx + c[2] * dy * dy) + c[1] * dx * dy;
                        float alpha = fminf(ORA_MAX_ALPHA, opac[g] * expf(-sigma));
                        if (sigma < 0.f || alpha < ORA_ALPHA_THRESHOLD) continue;
                        float next = T * (1.f - alpha);
                        if (next <= ORA_T_THRESHOLD) { done = 1; break; }
                        if (gids) {
                            gids[starts[gp] + cnt] = g % N;
                            pids[starts[gp] + cnt] = (int64_t)gp;
                        }
                        ++cnt;
                        T = next;
                    }
                    if (counts) counts[gp] = cnt;
                }
        }
}
