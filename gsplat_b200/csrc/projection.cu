// EWA projection of 3D Gaussians to image-space splats, forward and backward.
//
// Reference behaviour: gsplat/cuda/csrc/ProjectionEWA3DGSFused.cu:38-234 (forward),
// :316-553 (backward), ProjectionEWA3DGSPacked.cu:39-290 / 400-690 (packed COO
// layout), with the math of gsplat/cuda/include/Utils.cuh. Camera models: pinhole,
// orthographic and fisheye (the reference's packed kernels have no fisheye branch;
// here both layouts share the projection math, so packed fisheye works too).
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
#include "projection_common.cuh"

namespace gsb {

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

// Packed layout, pass 1: visibility of every (camera, Gaussian) pair. The grid is
// (ceil(N/256), B*C) like ProjectionEWA3DGSPacked.cu; each warp stores its ballot
// in vis_bits[(row * gridDim.x + blockIdx.x) * 8 + warp] and each block its count
// in block_cnts[row * gridDim.x + blockIdx.x]. Pass 2 reuses the stored ballots,
// so both passes agree on the compacted positions by construction.
__global__ void __launch_bounds__(256) projection_packed_count_kernel(ProjParams p,
                                                                      int32_t *block_cnts,
                                                                      uint32_t *vis_bits) {
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
    const size_t block_idx = (size_t)row * gridDim.x + blockIdx.x;
    const uint32_t ballot = __ballot_sync(0xffffffffu, valid);
    if ((threadIdx.x & 31) == 0) vis_bits[block_idx * 8 + (threadIdx.x >> 5)] = ballot;
    const int n = __syncthreads_count(valid);
    if (threadIdx.x == 0) block_cnts[block_idx] = n;
}

// Position of this lane's pair in the packed arrays (valid lanes only), from the
// pass-1 ballots and the inclusive scan of the block counts.
__device__ inline int64_t packed_position(const uint32_t *vis_bits, const int64_t *block_accum,
                                          size_t block_idx, uint32_t &ballot) {
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t *words = vis_bits + block_idx * 8;
    ballot = words[warp];
    int64_t off = block_idx == 0 ? 0 : block_accum[block_idx - 1];
    for (uint32_t w = 0; w < warp; ++w) off += __popc(words[w]);
    return off + __popc(ballot & ((1u << lane) - 1u));
}

// Packed layout, pass 2: write the visible pairs at their compacted position.
// Output order is row-major in (b, c) and then by Gaussian id, matching the
// reference's BlockScan ordering.
__global__ void __launch_bounds__(256) projection_packed_write_kernel(
    ProjParams p, const uint32_t *vis_bits, const int64_t *block_accum, int64_t nnz,
    int32_t *indptr, int64_t *batch_ids, int64_t *camera_ids, int64_t *gaussian_ids,
    int32_t *radii, float *means2d, float *depths, float *conics, float *comps) {
    const uint32_t row = blockIdx.y;
    const uint32_t b = row / p.C, c = row % p.C;
    const uint32_t g = blockIdx.x * blockDim.x + threadIdx.x;
    const size_t block_idx = (size_t)row * gridDim.x + blockIdx.x;
    uint32_t ballot;
    const int64_t pos = packed_position(vis_bits, block_accum, block_idx, ballot);
    if (threadIdx.x == 0 && blockIdx.x == 0) {
        indptr[row] = (int32_t)(block_idx == 0 ? 0 : block_accum[block_idx - 1]);
        if (row == gridDim.y - 1) indptr[gridDim.y] = (int32_t)block_accum[(size_t)gridDim.y * gridDim.x - 1];
    }
    if (!((ballot >> (threadIdx.x & 31)) & 1u) || g >= p.N || pos >= nnz) return;
    float mean[3];
    M3 covar;
    load_gaussian(p, b, g, mean, covar);
    const ProjOut o = project_one(p, b, c, g, mean, covar, true);
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
    if (m == kPinhole || m == kOrtho || m == kFisheye) return kOk;
    return set_error(kErrUnsupported, "camera_model %d is not supported (pinhole=0, ortho=1, fisheye=2)", m);
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
    if ((size_t)B * N == 0 || C == 0) return kOk;
    if (covars == nullptr && (quats == nullptr || scales == nullptr))
        return set_error(kErrInvalidArgument, "covars or (quats, scales) is required");
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
                                           int32_t *block_cnts, uint32_t *vis_bits,
                                           cudaStream_t stream) {
    if (int e = check_camera_model(camera_model)) return e;
    if ((size_t)B * C == 0 || N == 0) return kOk;
    ProjParams p = make_params(B, C, N, means, covars, quats, scales, opacities, viewmats, Ks, width,
                               height, eps2d, near_plane, far_plane, radius_clip,
                               calc_compensations, camera_model);
    dim3 grid((N + 255) / 256, B * C);
    projection_packed_count_kernel<<<grid, 256, 0, stream>>>(p, block_cnts, vis_bits);
    return check_launch("projection_packed_count_kernel");
}

extern "C" int gsb_projection_packed_write(
    int B, int C, int N, const float *means, const float *covars, const float *quats,
    const float *scales, const float *opacities, const float *viewmats, const float *Ks, int width,
    int height, float eps2d, float near_plane, float far_plane, float radius_clip,
    int calc_compensations, int camera_model, const uint32_t *vis_bits,
    const int64_t *block_accum, long long nnz, int32_t *indptr, int64_t *batch_ids, int64_t *camera_ids, int64_t *gaussian_ids,
    int32_t *radii, float *means2d, float *depths, float *conics, float *compensations,
    cudaStream_t stream) {
    if (int e = check_camera_model(camera_model)) return e;
    if ((size_t)B * C == 0 || N == 0) return kOk;
    ProjParams p = make_params(B, C, N, means, covars, quats, scales, opacities, viewmats, Ks, width,
                               height, eps2d, near_plane, far_plane, radius_clip,
                               calc_compensations, camera_model);
    dim3 grid((N + 255) / 256, B * C);
    projection_packed_write_kernel<<<grid, 256, 0, stream>>>(
        p, vis_bits, block_accum, nnz, indptr, batch_ids, camera_ids, gaussian_ids, radii, means2d, depths, conics,
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
