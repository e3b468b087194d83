// EWA projection of 3D Gaussians to image-space splats, forward and backward.
//
// Reference behaviour: gsplat/cuda/csrc/ProjectionEWA3DGSFused.cu:38-234 (forward),
// :316-553 (backward), ProjectionEWA3DGSPacked.cu:39-290 / 400-690 (packed COO
// layout), with the math of gsplat/cuda/include/Utils.cuh. Camera models: pinhole
// and orthographic.
//
// Layout: one thread owns one Gaussian of one batch element and loops over the C
// cameras, so the Gaussian's parameters are read from HBM once and its covariance
// is built once. Per-camera outputs are written as [B, C, N, ...] rows, which keeps
// the stores of a warp contiguous. The backward pass accumulates the per-camera
// gradients in registers and writes each Gaussian's gradient exactly once
// (no atomics, deterministic); only the view-matrix gradient is reduced across
// Gaussians (warp butterfly + one atomic per warp and camera).
#include "common.cuh"
#include "gsb_internal.h"

namespace gsb {

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
__device__ inline ProjOut project_one(const ProjParams &p, uint32_t b, uint32_t c, uint32_t g,
                                      const float mean[3], const M3 &covar) {
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
    if (z < p.near_plane || z > p.far_plane) return o;

    const M3 cov_c = m3_mul_bt(m3_mul(R, covar), R);
    const float fx = K[0], cx = K[2], fy = K[4], cy = K[5];
    float s00, s01, s11, mx, my;
    if (p.camera_model == kOrtho) {
        jsjt(cov_c, fx, 0.f, fy, 0.f, s00, s01, s11);
        mx = fx * x + cx;
        my = fy * y + cy;
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
    if (det <= 0.f) return o;
    const float inv_det = 1.f / det;

    float extend = kGaussianExtend;
    if (p.opacities != nullptr) {
        float op = p.opacities[(size_t)b * p.N + g];
        if (p.calc_comp) op *= comp;
        if (op < kAlphaThreshold) return o;
        extend = fminf(kGaussianExtend, sqrtf(2.f * det_logf(op / kAlphaThreshold)));
    }
    const float rx = ceilf(extend * sqrtf(s00));
    const float ry = ceilf(extend * sqrtf(s11));
    if (rx <= p.radius_clip && ry <= p.radius_clip) return o;
    if (mx + rx <= 0.f || mx - rx >= (float)p.W || my + ry <= 0.f || my - ry >= (float)p.H) return o;

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

__global__ void __launch_bounds__(256) projection_fwd_dense_kernel(ProjParams p, int32_t *radii,
                                                                   float *means2d, float *depths,
                                                                   float *conics, float *comps) {
    const uint32_t tid = blockIdx.x * blockDim.x + threadIdx.x;
    if (tid >= p.B * p.N) return;
    const uint32_t b = tid / p.N, g = tid % p.N;
    float mean[3];
    M3 covar;
    load_gaussian(p, b, g, mean, covar);
    for (uint32_t c = 0; c < p.C; ++c) {
        const ProjOut o = project_one(p, b, c, g, mean, covar);
        const size_t idx = ((size_t)b * p.C + c) * p.N + g;
        if (o.valid) {
            radii[idx * 2] = o.rx;
            radii[idx * 2 + 1] = o.ry;
            means2d[idx * 2] = o.mx;
            means2d[idx * 2 + 1] = o.my;
            depths[idx] = o.depth;
            conics[idx * 3 + 0] = o.conic[0];
            conics[idx * 3 + 1] = o.conic[1];
            conics[idx * 3 + 2] = o.conic[2];
            if (comps) comps[idx] = o.comp;
        } else {
            radii[idx * 2] = 0;
            radii[idx * 2 + 1] = 0;
            means2d[idx * 2] = 0.f;
            means2d[idx * 2 + 1] = 0.f;
            depths[idx] = 0.f;
            conics[idx * 3 + 0] = 0.f;
            conics[idx * 3 + 1] = 0.f;
            conics[idx * 3 + 2] = 0.f;
            if (comps) comps[idx] = 0.f;
        }
    }
}

// Packed layout, pass 1: number of visible (camera, Gaussian) pairs per block
// row. The grid is (ceil(N/256), B*C) like ProjectionEWA3DGSPacked.cu; a block's
// count goes to block_cnts[row * blocks_per_row + col].
__global__ void __launch_bounds__(256) projection_packed_count_kernel(ProjParams p,
                                                                      int32_t *block_cnts) {
    const uint32_t row = blockIdx.y;
    const uint32_t b = row / p.C, c = row % p.C;
    const uint32_t g = blockIdx.x * blockDim.x + threadIdx.x;
    bool valid = false;
    if (g < p.N) {
        float mean[3];
        M3 covar;
        load_gaussian(p, b, g, mean, covar);
        valid = project_one(p, b, c, g, mean, covar).valid;
    }
    const int n = __syncthreads_count(valid);
    if (threadIdx.x == 0) block_cnts[(size_t)row * gridDim.x + blockIdx.x] = n;
}

// Packed layout, pass 2: write the visible pairs at their compacted position.
// block_accum is the inclusive scan of block_cnts; output order is row-major in
// (b, c) and then by Gaussian id, matching the reference's BlockScan ordering.
__global__ void __launch_bounds__(256) projection_packed_write_kernel(
    ProjParams p, const int64_t *block_accum, int64_t nnz, int32_t *indptr, int64_t *batch_ids,
    int64_t *camera_ids, int64_t *gaussian_ids, int32_t *radii, float *means2d, float *depths,
    float *conics, float *comps) {
    __shared__ int32_t warp_tot[8];
    const uint32_t row = blockIdx.y;
    const uint32_t b = row / p.C, c = row % p.C;
    const uint32_t g = blockIdx.x * blockDim.x + threadIdx.x;
    const size_t block_idx = (size_t)row * gridDim.x + blockIdx.x;
    ProjOut o;
    o.valid = false;
    if (g < p.N) {
        float mean[3];
        M3 covar;
        load_gaussian(p, b, g, mean, covar);
        o = project_one(p, b, c, g, mean, covar);
    }
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t ballot = __ballot_sync(0xffffffffu, o.valid);
    if (lane == 0) warp_tot[warp] = __popc(ballot);
    __syncthreads();
    int32_t warp_off = 0;
    for (uint32_t w = 0; w < warp; ++w) warp_off += warp_tot[w];
    const int64_t base = block_idx == 0 ? 0 : block_accum[block_idx - 1];
    const int64_t pos = base + warp_off + __popc(ballot & ((1u << lane) - 1u));
    // Pass 1 evaluated the same visibility test; the bound only guards the
    // outputs should the two passes ever disagree.
    if (o.valid && pos < nnz) {
        batch_ids[pos] = b;
        camera_ids[pos] = c;
        gaussian_ids[pos] = g;
        radii[pos * 2] = o.rx;
        radii[pos * 2 + 1] = o.ry;
        means2d[pos * 2] = o.mx;
        means2d[pos * 2 + 1] = o.my;
        depths[pos] = o.depth;
        conics[pos * 3 + 0] = o.conic[0];
        conics[pos * 3 + 1] = o.conic[1];
        conics[pos * 3 + 2] = o.conic[2];
        if (comps) comps[pos] = o.comp;
    }
    if (threadIdx.x == 0 && blockIdx.x == 0) {
        indptr[row] = (int32_t)base;
        if (row == gridDim.y - 1) indptr[gridDim.y] = (int32_t)block_accum[(size_t)gridDim.y * gridDim.x - 1];
    }
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
// blur), 583-660 (pinhole), 502-540 (ortho), 62-112 (world-to-camera).
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

struct ProjBwdParams {
    ProjParams p;
    const int32_t *radii;
    const float *conics, *comps;
    const float *v_means2d, *v_depths, *v_conics, *v_comps;
    float *v_means, *v_covars, *v_quats, *v_scales, *v_viewmats;
};

__device__ inline void reduce_viewmat_grad(float *v_viewmats, size_t cam, const ProjGrads &gr,
                                           bool active) {
    // Sum the 12 view-matrix gradient entries over the warp, one atomic per entry.
    const uint32_t mask = __ballot_sync(0xffffffffu, active);
    if (mask == 0) return;
    float vals[12];
#pragma unroll
    for (int i = 0; i < 3; ++i) {
#pragma unroll
        for (int j = 0; j < 3; ++j) vals[i * 4 + j] = active ? gr.v_R.m[i][j] : 0.f;
        vals[i * 4 + 3] = active ? gr.v_t[i] : 0.f;
    }
#pragma unroll
    for (int k = 0; k < 12; ++k) vals[k] = warp_sum(vals[k]);
    if ((threadIdx.x & 31) == 0) {
#pragma unroll
        for (int k = 0; k < 12; ++k) atomicAdd(v_viewmats + cam * 16 + k, vals[k]);
    }
}

__global__ void __launch_bounds__(256) projection_bwd_dense_kernel(ProjBwdParams q) {
    const ProjParams &p = q.p;
    const uint32_t tid = blockIdx.x * blockDim.x + threadIdx.x;
    const bool in_range = tid < p.B * p.N;
    const uint32_t b = in_range ? tid / p.N : 0, g = in_range ? tid % p.N : 0;
    float mean[3] = {0.f, 0.f, 0.f};
    M3 covar = m3_zero();
    float quat[4] = {1.f, 0.f, 0.f, 0.f}, scale[3] = {1.f, 1.f, 1.f};
    if (in_range) {
        const float *mp = p.means + ((size_t)b * p.N + g) * 3;
        mean[0] = mp[0];
        mean[1] = mp[1];
        mean[2] = mp[2];
        if (p.covars != nullptr) {
            load_gaussian(p, b, g, mean, covar);
        } else {
            const float *qp = p.quats + ((size_t)b * p.N + g) * 4;
            quat[0] = qp[0];
            quat[1] = qp[1];
            quat[2] = qp[2];
            quat[3] = qp[3];
            const float *sp = p.scales + ((size_t)b * p.N + g) * 3;
            scale[0] = sp[0];
            scale[1] = sp[1];
            scale[2] = sp[2];
            covar = covar_from_quat_scale(quat, scale, nullptr);
        }
    }
    float v_mean[3] = {0.f, 0.f, 0.f};
    M3 v_cov = m3_zero();
    bool any = false;
    for (uint32_t c = 0; c < p.C; ++c) {
        const size_t idx = ((size_t)b * p.C + c) * p.N + g;
        bool active = false;
        ProjGrads gr;
        if (in_range) {
            active = q.radii[idx * 2] > 0 && q.radii[idx * 2 + 1] > 0;
        }
        if (active) {
            const float conic[3] = {q.conics[idx * 3], q.conics[idx * 3 + 1], q.conics[idx * 3 + 2]};
            const float v_m2d[2] = {q.v_means2d[idx * 2], q.v_means2d[idx * 2 + 1]};
            const float v_conic[3] = {q.v_conics[idx * 3], q.v_conics[idx * 3 + 1],
                                      q.v_conics[idx * 3 + 2]};
            const bool has_vcomp = q.v_comps != nullptr;
            const float comp = has_vcomp ? q.comps[idx] : 0.f;
            const float vcomp = has_vcomp ? q.v_comps[idx] : 0.f;
            project_one_vjp(p, b, c, mean, covar, conic, comp, v_m2d, q.v_depths[idx], v_conic,
                            vcomp, has_vcomp, gr);
            v_mean[0] += gr.v_mean[0];
            v_mean[1] += gr.v_mean[1];
            v_mean[2] += gr.v_mean[2];
            v_cov = m3_add(v_cov, gr.v_cov);
            any = true;
        }
        if (q.v_viewmats != nullptr) reduce_viewmat_grad(q.v_viewmats, (size_t)b * p.C + c, gr, active);
    }
    if (!in_range) return;
    const size_t gi = (size_t)b * p.N + g;
    if (q.v_means) {
        q.v_means[gi * 3 + 0] = v_mean[0];
        q.v_means[gi * 3 + 1] = v_mean[1];
        q.v_means[gi * 3 + 2] = v_mean[2];
    }
    if (p.covars != nullptr) {
        if (q.v_covars) {
            float *vc = q.v_covars + gi * 6;
            vc[0] = v_cov.m[0][0];
            vc[1] = v_cov.m[0][1] + v_cov.m[1][0];
            vc[2] = v_cov.m[0][2] + v_cov.m[2][0];
            vc[3] = v_cov.m[1][1];
            vc[4] = v_cov.m[1][2] + v_cov.m[2][1];
            vc[5] = v_cov.m[2][2];
        }
    } else {
        float v_q[4] = {0.f, 0.f, 0.f, 0.f}, v_s[3] = {0.f, 0.f, 0.f};
        if (any) {
            M3 Rq = quat_to_rotmat(quat[0], quat[1], quat[2], quat[3]);
            covar_from_quat_scale_vjp(quat, scale, Rq, v_cov, v_q, v_s);
        }
        if (q.v_quats) {
            q.v_quats[gi * 4 + 0] = v_q[0];
            q.v_quats[gi * 4 + 1] = v_q[1];
            q.v_quats[gi * 4 + 2] = v_q[2];
            q.v_quats[gi * 4 + 3] = v_q[3];
        }
        if (q.v_scales) {
            q.v_scales[gi * 3 + 0] = v_s[0];
            q.v_scales[gi * 3 + 1] = v_s[1];
            q.v_scales[gi * 3 + 2] = v_s[2];
        }
    }
}

struct ProjPackedBwdParams {
    ProjParams p;
    uint32_t nnz;
    const int64_t *batch_ids, *camera_ids, *gaussian_ids;
    const float *conics, *comps;
    const float *v_means2d, *v_depths, *v_conics, *v_comps;
    bool sparse_grad;
    float *v_means, *v_covars, *v_quats, *v_scales, *v_viewmats;
};

// Packed backward: one thread per visible pair. Dense gradients (sparse_grad
// false) are accumulated with atomics because a Gaussian may be visible in
// several cameras; sparse gradients are written per pair.
__global__ void __launch_bounds__(256) projection_bwd_packed_kernel(ProjPackedBwdParams q) {
    const ProjParams &p = q.p;
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    const bool active = i < q.nnz;
    const uint32_t b = active ? (uint32_t)q.batch_ids[i] : 0;
    const uint32_t c = active ? (uint32_t)q.camera_ids[i] : 0;
    const uint32_t g = active ? (uint32_t)q.gaussian_ids[i] : 0;
    ProjGrads gr;
    float quat[4] = {1.f, 0.f, 0.f, 0.f}, scale[3] = {1.f, 1.f, 1.f};
    if (active) {
        float mean[3];
        M3 covar;
        const float *mp = p.means + ((size_t)b * p.N + g) * 3;
        mean[0] = mp[0];
        mean[1] = mp[1];
        mean[2] = mp[2];
        if (p.covars != nullptr) {
            load_gaussian(p, b, g, mean, covar);
        } else {
            const float *qp = p.quats + ((size_t)b * p.N + g) * 4;
            quat[0] = qp[0];
            quat[1] = qp[1];
            quat[2] = qp[2];
            quat[3] = qp[3];
            const float *sp = p.scales + ((size_t)b * p.N + g) * 3;
            scale[0] = sp[0];
            scale[1] = sp[1];
            scale[2] = sp[2];
            covar = covar_from_quat_scale(quat, scale, nullptr);
        }
        const float conic[3] = {q.conics[(size_t)i * 3], q.conics[(size_t)i * 3 + 1], q.conics[(size_t)i * 3 + 2]};
        const float v_m2d[2] = {q.v_means2d[(size_t)i * 2], q.v_means2d[(size_t)i * 2 + 1]};
        const float v_conic[3] = {q.v_conics[(size_t)i * 3], q.v_conics[(size_t)i * 3 + 1],
                                  q.v_conics[(size_t)i * 3 + 2]};
        const bool has_vcomp = q.v_comps != nullptr;
        project_one_vjp(p, b, c, mean, covar, conic, has_vcomp ? q.comps[i] : 0.f, v_m2d,
                        q.v_depths[i], v_conic, has_vcomp ? q.v_comps[i] : 0.f, has_vcomp, gr);
        const size_t dst = q.sparse_grad ? (size_t)i : ((size_t)b * p.N + g);
        if (q.v_means) {
            float *vmp = q.v_means + dst * 3;
            if (q.sparse_grad) {
                vmp[0] = gr.v_mean[0];
                vmp[1] = gr.v_mean[1];
                vmp[2] = gr.v_mean[2];
            } else {
                atomicAdd(vmp + 0, gr.v_mean[0]);
                atomicAdd(vmp + 1, gr.v_mean[1]);
                atomicAdd(vmp + 2, gr.v_mean[2]);
            }
        }
        if (p.covars != nullptr) {
            if (q.v_covars) {
                float vals[6] = {gr.v_cov.m[0][0], gr.v_cov.m[0][1] + gr.v_cov.m[1][0],
                                 gr.v_cov.m[0][2] + gr.v_cov.m[2][0], gr.v_cov.m[1][1],
                                 gr.v_cov.m[1][2] + gr.v_cov.m[2][1], gr.v_cov.m[2][2]};
                float *vc = q.v_covars + dst * 6;
#pragma unroll
                for (int k = 0; k < 6; ++k) {
                    if (q.sparse_grad) vc[k] = vals[k];
                    else atomicAdd(vc + k, vals[k]);
                }
            }
        } else {
            float v_q[4] = {0.f, 0.f, 0.f, 0.f}, v_s[3] = {0.f, 0.f, 0.f};
            M3 Rq = quat_to_rotmat(quat[0], quat[1], quat[2], quat[3]);
            covar_from_quat_scale_vjp(quat, scale, Rq, gr.v_cov, v_q, v_s);
            if (q.v_quats) {
                float *vq = q.v_quats + dst * 4;
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    if (q.sparse_grad) vq[k] = v_q[k];
                    else atomicAdd(vq + k, v_q[k]);
                }
            }
            if (q.v_scales) {
                float *vs = q.v_scales + dst * 3;
#pragma unroll
                for (int k = 0; k < 3; ++k) {
                    if (q.sparse_grad) vs[k] = v_s[k];
                    else atomicAdd(vs + k, v_s[k]);
                }
            }
        }
    }
    if (q.v_viewmats != nullptr) {
        // Lanes of a warp almost always share one camera (pairs are sorted by
        // (b, c)); reduce per warp when they do, else fall back to per-lane atomics.
        const size_t cam = (size_t)b * p.C + c;
        const uint32_t amask = __ballot_sync(0xffffffffu, active);
        const uint32_t same = __match_any_sync(0xffffffffu, active ? (unsigned long long)cam : ~0ull);
        const bool uniform = (same & amask) == amask;
        if (__all_sync(0xffffffffu, uniform)) {
            reduce_viewmat_grad(q.v_viewmats, __shfl_sync(0xffffffffu, cam, __ffs(amask ? amask : 1u) - 1),
                                gr, active);
        } else if (active) {
#pragma unroll
            for (int r = 0; r < 3; ++r) {
#pragma unroll
                for (int j = 0; j < 3; ++j) atomicAdd(q.v_viewmats + cam * 16 + r * 4 + j, gr.v_R.m[r][j]);
                atomicAdd(q.v_viewmats + cam * 16 + r * 4 + 3, gr.v_t[r]);
            }
        }
    }
}

static ProjParams make_params(int B, int C, int N, const float *means, const float *covars,
                              const float *quats, const float *scales, const float *opacities,
                              const float *viewmats, const float *Ks, int W, int H, float eps2d,
                              float near_plane, float far_plane, float radius_clip, int calc_comp,
                              int camera_model) {
    ProjParams p;
    p.B = B;
    p.C = C;
    p.N = N;
    p.means = means;
    p.covars = covars;
    p.quats = quats;
    p.scales = scales;
    p.opacities = opacities;
    p.viewmats = viewmats;
    p.Ks = Ks;
    p.W = W;
    p.H = H;
    p.eps2d = eps2d;
    p.near_plane = near_plane;
    p.far_plane = far_plane;
    p.radius_clip = radius_clip;
    p.calc_comp = calc_comp != 0;
    p.camera_model = camera_model;
    return p;
}

static int check_camera_model(int m) {
    if (m == kPinhole || m == kOrtho) return kOk;
    return set_error(kErrUnsupported, "camera_model %d is not supported (pinhole=0, ortho=1)", m);
}

} // namespace gsb

using namespace gsb;

extern "C" int gsb_projection_fused_fwd(int B, int C, int N, const float *means,
                                        const float *covars, const float *quats,
                                        const float *scales, const float *opacities,
                                        const float *viewmats, const float *Ks, int width,
                                        int height, float eps2d, float near_plane,
                                        float far_plane, float radius_clip,
                                        int calc_compensations, int camera_model, int32_t *radii,
                                        float *means2d, float *depths, float *conics,
                                        float *compensations, cudaStream_t stream) {
    if (int e = check_camera_model(camera_model)) return e;
    if (covars == nullptr && (quats == nullptr || scales == nullptr))
        return set_error(kErrInvalidArgument, "covars or (quats, scales) is required");
    if ((size_t)B * N == 0 || C == 0) return kOk;
    ProjParams p = make_params(B, C, N, means, covars, quats, scales, opacities, viewmats, Ks, width,
                               height, eps2d, near_plane, far_plane, radius_clip,
                               calc_compensations, camera_model);
    const uint32_t n = (uint32_t)B * N;
    projection_fwd_dense_kernel<<<(n + 255) / 256, 256, 0, stream>>>(
        p, radii, means2d, depths, conics, calc_compensations ? compensations : nullptr);
    return check_launch("projection_fwd_dense_kernel");
}

extern "C" int gsb_projection_packed_blocks(int N) { return (N + 255) / 256; }

extern "C" int gsb_projection_packed_count(int B, int C, int N, const float *means,
                                           const float *covars, const float *quats,
                                           const float *scales, const float *opacities,
                                           const float *viewmats, const float *Ks, int width,
                                           int height, float eps2d, float near_plane,
                                           float far_plane, float radius_clip,
                                           int calc_compensations, int camera_model,
                                           int32_t *block_cnts, cudaStream_t stream) {
    if (int e = check_camera_model(camera_model)) return e;
    if ((size_t)B * C == 0 || N == 0) return kOk;
    ProjParams p = make_params(B, C, N, means, covars, quats, scales, opacities, viewmats, Ks, width,
                               height, eps2d, near_plane, far_plane, radius_clip,
                               calc_compensations, camera_model);
    dim3 grid((N + 255) / 256, B * C);
    projection_packed_count_kernel<<<grid, 256, 0, stream>>>(p, block_cnts);
    return check_launch("projection_packed_count_kernel");
}

extern "C" int gsb_projection_packed_write(
    int B, int C, int N, const float *means, const float *covars, const float *quats,
    const float *scales, const float *opacities, const float *viewmats, const float *Ks, int width,
    int height, float eps2d, float near_plane, float far_plane, float radius_clip,
    int calc_compensations, int camera_model, const int64_t *block_accum, long long nnz,
    int32_t *indptr, int64_t *batch_ids, int64_t *camera_ids, int64_t *gaussian_ids,
    int32_t *radii, float *means2d, float *depths, float *conics, float *compensations,
    cudaStream_t stream) {
    if (int e = check_camera_model(camera_model)) return e;
    if ((size_t)B * C == 0 || N == 0) return kOk;
    ProjParams p = make_params(B, C, N, means, covars, quats, scales, opacities, viewmats, Ks, width,
                               height, eps2d, near_plane, far_plane, radius_clip,
                               calc_compensations, camera_model);
    dim3 grid((N + 255) / 256, B * C);
    projection_packed_write_kernel<<<grid, 256, 0, stream>>>(
        p, block_accum, nnz, indptr, batch_ids, camera_ids, gaussian_ids, radii, means2d, depths, conics,
        calc_compensations ? compensations : nullptr);
    return check_launch("projection_packed_write_kernel");
}

extern "C" int gsb_projection_fused_bwd(int B, int C, int N, const float *means,
                                        const float *covars, const float *quats,
                                        const float *scales, const float *viewmats,
                                        const float *Ks, int width, int height, float eps2d,
                                        int camera_model, const int32_t *radii,
                                        const float *conics, const float *compensations,
                                        const float *v_means2d, const float *v_depths,
                                        const float *v_conics, const float *v_compensations,
                                        float *v_means, float *v_covars, float *v_quats,
                                        float *v_scales, float *v_viewmats, cudaStream_t stream) {
    if (int e = check_camera_model(camera_model)) return e;
    if (v_compensations != nullptr && compensations == nullptr)
        return set_error(kErrInvalidArgument, "v_compensations requires compensations");
    if ((size_t)B * N == 0 || C == 0) return kOk;
    ProjBwdParams q;
    q.p = make_params(B, C, N, means, covars, quats, scales, nullptr, viewmats, Ks, width, height,
                      eps2d, 0.f, 0.f, 0.f, 0, camera_model);
    q.radii = radii;
    q.conics = conics;
    q.comps = compensations;
    q.v_means2d = v_means2d;
    q.v_depths = v_depths;
    q.v_conics = v_conics;
    q.v_comps = v_compensations;
    q.v_means = v_means;
    q.v_covars = v_covars;
    q.v_quats = v_quats;
    q.v_scales = v_scales;
    q.v_viewmats = v_viewmats;
    const uint32_t n = (uint32_t)B * N;
    projection_bwd_dense_kernel<<<(n + 255) / 256, 256, 0, stream>>>(q);
    return check_launch("projection_bwd_dense_kernel");
}

extern "C" int gsb_projection_packed_bwd(
    int B, int C, int N, int nnz, const float *means, const float *covars, const float *quats,
    const float *scales, const float *viewmats, const float *Ks, int width, int height,
    float eps2d, int camera_model, const int64_t *batch_ids, const int64_t *camera_ids,
    const int64_t *gaussian_ids, const float *conics, const float *compensations,
    const float *v_means2d, const float *v_depths, const float *v_conics,
    const float *v_compensations, int sparse_grad, float *v_means, float *v_covars,
    float *v_quats, float *v_scales, float *v_viewmats, cudaStream_t stream) {
    if (int e = check_camera_model(camera_model)) return e;
    if (v_compensations != nullptr && compensations == nullptr)
        return set_error(kErrInvalidArgument, "v_compensations requires compensations");
    if (nnz == 0) return kOk;
    ProjPackedBwdParams q;
    q.p = make_params(B, C, N, means, covars, quats, scales, nullptr, viewmats, Ks, width, height,
                      eps2d, 0.f, 0.f, 0.f, 0, camera_model);
    q.nnz = nnz;
    q.batch_ids = batch_ids;
    q.camera_ids = camera_ids;
    q.gaussian_ids = gaussian_ids;
    q.conics = conics;
    q.comps = compensations;
    q.v_means2d = v_means2d;
    q.v_depths = v_depths;
    q.v_conics = v_conics;
    q.v_comps = v_compensations;
    q.sparse_grad = sparse_grad != 0;
    q.v_means = v_means;
    q.v_covars = v_covars;
    q.v_quats = v_quats;
    q.v_scales = v_scales;
    q.v_viewmats = v_viewmats;
    projection_bwd_packed_kernel<<<(nnz + 255) / 256, 256, 0, stream>>>(q);
    return check_launch("projection_bwd_packed_kernel");
}
