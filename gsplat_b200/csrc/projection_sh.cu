// Fused projection + spherical-harmonic colour evaluation, forward and backward.
//
// One kernel covers what the reference's rasterization() does in separate
// launches and torch ops (gsplat/rendering.py:749-872): EWA projection
// (ProjectionEWA3DGSFused.cu / ProjectionEWA3DGSPacked.cu), the view direction
// normalize(mean - campos) (rendering.py:227-253), SH evaluation
// (SphericalHarmonicsCUDA.cu:38-128), colors = clamp_min(sh + 0.5, 0)
// (rendering.py:872) and opacities * compensations (rendering.py:793-794).
// Coefficients are read straight from the per-Gaussian [N, K, 3] tensor for the
// visible pairs only, instead of gathering or broadcasting them first.
//
// The backward kernel runs one thread per Gaussian, loops over the cameras and
// writes every gradient row exactly once (zeros for Gaussians seen by no camera):
// v_means (projection + view-direction terms), v_quats, v_scales, v_opacities and
// v_sh [N, K, 3] -- no atomics, no zero-fill pass, no scatter of per-pair
// coefficient gradients.
#include "common.cuh"
#include "gsb_internal.h"
#include "projection_common.cuh"
#include "sh_basis.cuh"

namespace gsb {

struct FusedParams {
    ProjParams p;
    const float *sh; // [B, N, K, 3]
    uint32_t K;
    bool sh_vec; // rows of sh are 16-byte aligned (K*3 % 4 == 0, aligned base)
};

__device__ __forceinline__ void campos_of(const float *vm, float cp[3]) {
    // -R^T t
#pragma unroll
    for (int j = 0; j < 3; ++j) cp[j] = -(vm[0 * 4 + j] * vm[3] + vm[1 * 4 + j] * vm[7] + vm[2 * 4 + j] * vm[11]);
}

// Loads the first (D+1)^2 coefficient rows of one Gaussian; with `vec` the row
// starts 16-byte aligned and is read with 128-bit loads (all issued up front).
template <int D>
__device__ __forceinline__ void load_coefs(const float *coef, bool vec, float *c) {
    constexpr int NC = (D + 1) * (D + 1) * 3;
    if (vec && NC % 4 == 0) {
        const float4 *c4 = reinterpret_cast<const float4 *>(coef);
#pragma unroll
        for (int i = 0; i < NC / 4; ++i) {
            const float4 v = __ldg(c4 + i);
            c[4 * i + 0] = v.x;
            c[4 * i + 1] = v.y;
            c[4 * i + 2] = v.z;
            c[4 * i + 3] = v.w;
        }
    } else {
#pragma unroll
        for (int i = 0; i < NC; ++i) c[i] = __ldg(coef + i);
    }
}

// Calls fn(f, coef[f]) for the (D + 1)^2 * 3 coefficients of one Gaussian in
// order, reading them with 128-bit loads when the row is 16-byte aligned; the
// loop is fully unrolled, so f is a compile-time index in fn.
template <int D, class Fn>
__device__ __forceinline__ void for_each_coef(const float *coef, bool vec, Fn fn) {
    constexpr int NC = (D + 1) * (D + 1) * 3;
    if (vec && NC % 4 == 0) {
        const float4 *c4 = reinterpret_cast<const float4 *>(coef);
#pragma unroll
        for (int i = 0; i < NC / 4; ++i) {
            const float4 v = __ldg(c4 + i);
            fn(4 * i + 0, v.x);
            fn(4 * i + 1, v.y);
            fn(4 * i + 2, v.z);
            fn(4 * i + 3, v.w);
        }
    } else {
#pragma unroll
        for (int i = 0; i < NC; ++i) fn(i, __ldg(coef + i));
    }
}

// SH colour of one (camera, Gaussian) pair; returns the pre-clamp value in raw[].
template <int D>
__device__ __forceinline__ void sh_color(const float *coef, bool vec, const float dir[3], float raw[3]) {
    constexpr int NB = (D + 1) * (D + 1);
    float c[NB * 3];
    load_coefs<D>(coef, vec, c);
    const float inv = rsqrtf(dir[0] * dir[0] + dir[1] * dir[1] + dir[2] * dir[2]);
    float Y[NB];
    sh_eval<D>(dir[0] * inv, dir[1] * inv, dir[2] * inv, Y);
    raw[0] = raw[1] = raw[2] = 0.f;
#pragma unroll
    for (int k = 0; k < NB; ++k) {
        raw[0] += Y[k] * c[k * 3 + 0];
        raw[1] += Y[k] * c[k * 3 + 1];
        raw[2] += Y[k] * c[k * 3 + 2];
    }
}

// ---------------------------------------------------------------------------
// Forward, packed layout (pass 2; pass 1 is projection_packed_count_kernel)
// ---------------------------------------------------------------------------
template <int D>
#ifndef GSB_PACKED_WRITE_MINB
#define GSB_PACKED_WRITE_MINB 4 // measured fastest (latency-bound loads; a few bytes spill at degree 3)
#endif
__global__ void __launch_bounds__(256, GSB_PACKED_WRITE_MINB) fused_packed_write_kernel(
    FusedParams f, const uint32_t *vis_bits, const int64_t *block_accum, int64_t nnz,
    int32_t *indptr, int64_t *batch_ids, int64_t *camera_ids, int64_t *gaussian_ids,
    int32_t *radii, float *means2d, float *depths, float *conics, float *comps, float *colors,
    float *opac_out, int32_t *pair_index) {
    const ProjParams &p = f.p;
    const uint32_t row = blockIdx.y;
    const uint32_t b = row / p.C, c = row % p.C;
    const uint32_t g = blockIdx.x * blockDim.x + threadIdx.x;
    const size_t block_idx = (size_t)row * gridDim.x + blockIdx.x;
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t *words = vis_bits + block_idx * 8;
    const uint32_t ballot = words[warp];
    int64_t pos = block_idx == 0 ? 0 : block_accum[block_idx - 1];
    for (uint32_t w = 0; w < warp; ++w) pos += __popc(words[w]);
    pos += __popc(ballot & ((1u << lane) - 1u));
    if (threadIdx.x == 0 && blockIdx.x == 0) {
        indptr[row] = (int32_t)(block_idx == 0 ? 0 : block_accum[block_idx - 1]);
        if (row == gridDim.y - 1) indptr[gridDim.y] = (int32_t)block_accum[(size_t)gridDim.y * gridDim.x - 1];
    }
    if (g >= p.N) return;
    const bool vis = ((ballot >> lane) & 1u) && pos < nnz;
    if (pair_index) pair_index[(size_t)row * p.N + g] = vis ? (int32_t)pos : -1;
    if (!vis) return;
    float mean[3];
    M3 covar;
    load_gaussian(p, b, g, mean, covar);
    const ProjOut o = project_one(p, b, c, g, mean, covar, true);
    const float *vm = p.viewmats + ((size_t)b * p.C + c) * 16;
    float cp[3];
    campos_of(vm, cp);
    const float dir[3] = {mean[0] - cp[0], mean[1] - cp[1], mean[2] - cp[2]};
    float raw[3];
    sh_color<D>(f.sh + ((size_t)b * p.N + g) * f.K * 3, f.sh_vec, dir, raw);
    const float op = p.opacities[(size_t)b * p.N + g];
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
    colors[pos * 3 + 0] = fmaxf(raw[0] + 0.5f, 0.f);
    colors[pos * 3 + 1] = fmaxf(raw[1] + 0.5f, 0.f);
    colors[pos * 3 + 2] = fmaxf(raw[2] + 0.5f, 0.f);
    opac_out[pos] = p.calc_comp ? op * o.comp : op;
}

// ---------------------------------------------------------------------------
// Forward, dense [B, C, N] layout
// ---------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(256) fused_dense_fwd_kernel(FusedParams f, int32_t *radii,
                                                              float *means2d, float *depths,
                                                              float *conics, float *comps,
                                                              float *colors, float *opac_out) {
    const ProjParams &p = f.p;
    const uint32_t tid = blockIdx.x * blockDim.x + threadIdx.x;
    if (tid >= p.B * p.N) return;
    const uint32_t b = tid / p.N, g = tid % p.N;
    float mean[3];
    M3 covar;
    load_gaussian(p, b, g, mean, covar);
    const float op = p.opacities[(size_t)b * p.N + g];
    const float *coef = f.sh + ((size_t)b * p.N + g) * f.K * 3;
    for (uint32_t c = 0; c < p.C; ++c) {
        const ProjOut o = project_one(p, b, c, g, mean, covar);
        const size_t idx = ((size_t)b * p.C + c) * p.N + g;
        float raw[3] = {-0.5f, -0.5f, -0.5f};
        if (o.valid) {
            const float *vm = p.viewmats + ((size_t)b * p.C + c) * 16;
            float cp[3];
            campos_of(vm, cp);
            const float dir[3] = {mean[0] - cp[0], mean[1] - cp[1], mean[2] - cp[2]};
            sh_color<D>(coef, f.sh_vec, dir, raw);
        }
        radii[idx * 2] = o.valid ? o.rx : 0;
        radii[idx * 2 + 1] = o.valid ? o.ry : 0;
        means2d[idx * 2] = o.valid ? o.mx : 0.f;
        means2d[idx * 2 + 1] = o.valid ? o.my : 0.f;
        depths[idx] = o.valid ? o.depth : 0.f;
        conics[idx * 3 + 0] = o.valid ? o.conic[0] : 0.f;
        conics[idx * 3 + 1] = o.valid ? o.conic[1] : 0.f;
        conics[idx * 3 + 2] = o.valid ? o.conic[2] : 0.f;
        if (comps) comps[idx] = o.valid ? o.comp : 0.f;
        colors[idx * 3 + 0] = fmaxf(raw[0] + 0.5f, 0.f);
        colors[idx * 3 + 1] = fmaxf(raw[1] + 0.5f, 0.f);
        colors[idx * 3 + 2] = fmaxf(raw[2] + 0.5f, 0.f);
        opac_out[idx] = p.calc_comp ? (o.valid ? op * o.comp : 0.f) : op;
    }
}

// ---------------------------------------------------------------------------
// Backward (both layouts): thread per (batch, Gaussian), loop over cameras.
// ---------------------------------------------------------------------------
struct FusedBwdParams {
    FusedParams f;
    bool packed;
    const int32_t *pair_index; // packed: [B*C*N] position or -1
    const int32_t *radii;      // dense: [B,C,N,2]
    const float *conics, *comps;
    const float *v_means2d, *v_depths, *v_conics, *v_comps, *v_colors, *v_opac;
    float *v_means, *v_quats, *v_scales, *v_opacities, *v_sh;
};

constexpr int kFusedBwdThreads = 128;

template <int D>
#ifndef GSB_FUSED_BWD_MINB
#define GSB_FUSED_BWD_MINB 5
#endif
__global__ void __launch_bounds__(kFusedBwdThreads, (D >= 4 ? 3 : (D == 1 ? 4 : GSB_FUSED_BWD_MINB)))
    fused_bwd_kernel(FusedBwdParams q) {
    constexpr int NB = (D + 1) * (D + 1);
    // v_sh rows are accumulated in shared memory (row stride K*3 rounded up to an
    // odd count, so the lanes of a warp hit distinct banks) and stored to HBM
    // with coalesced writes at the end.
    extern __shared__ float s_vsh[];
    const ProjParams &p = q.f.p;
    const uint32_t K3 = q.f.K * 3;
    const uint32_t stride = K3 | 1u;
    const size_t first = (size_t)blockIdx.x * kFusedBwdThreads;
    const uint32_t tid = threadIdx.x;
    const size_t gi = first + tid; // flattened (b, g)
    const bool in_range = gi < (size_t)p.B * p.N;
    float *vsh = s_vsh + (size_t)tid * stride;
    for (uint32_t k = 0; k < K3; ++k) vsh[k] = 0.f;
    float v_mean[3] = {0.f, 0.f, 0.f}, v_op = 0.f;
    float v_q[4] = {0.f, 0.f, 0.f, 0.f}, v_s[3] = {0.f, 0.f, 0.f};
    if (in_range) {
        const uint32_t b = (uint32_t)(gi / p.N), g = (uint32_t)(gi % p.N);
        float mean[3], quat[4], scale[3];
        const float *mp = p.means + gi * 3;
        mean[0] = mp[0];
        mean[1] = mp[1];
        mean[2] = mp[2];
        const float *qp = p.quats + gi * 4;
        quat[0] = qp[0];
        quat[1] = qp[1];
        quat[2] = qp[2];
        quat[3] = qp[3];
        const float *sp = p.scales + gi * 3;
        scale[0] = sp[0];
        scale[1] = sp[1];
        scale[2] = sp[2];
        const float op = p.opacities[gi];
        const float *coef = q.f.sh + gi * K3;
        M3 covar;
        bool have_covar = false;
        M3 v_cov = m3_zero();
        bool any = false;
        for (uint32_t c = 0; c < p.C; ++c) {
            const size_t didx = ((size_t)b * p.C + c) * p.N + g;
            int64_t e;
            if (q.packed) {
                e = q.pair_index[didx];
            } else {
                e = (q.radii[didx * 2] > 0 && q.radii[didx * 2 + 1] > 0) ? (int64_t)didx : -1;
            }
            if (e < 0) continue;
            if (!have_covar) {
                covar = covar_from_quat_scale(quat, scale, nullptr);
                have_covar = true;
            }
            any = true;
            // opacity * compensation
            const float v_oe = q.v_opac ? q.v_opac[e] : 0.f;
            float comp = 0.f, v_comp = q.v_comps ? q.v_comps[e] : 0.f;
            if (p.calc_comp) {
                comp = q.comps[e];
                v_op += v_oe * comp;
                v_comp += v_oe * op;
            } else {
                v_op += v_oe;
            }
            const float conic[3] = {q.conics[e * 3], q.conics[e * 3 + 1], q.conics[e * 3 + 2]};
            const float v_m2d[2] = {q.v_means2d[e * 2], q.v_means2d[e * 2 + 1]};
            const float v_conic[3] = {q.v_conics[e * 3], q.v_conics[e * 3 + 1], q.v_conics[e * 3 + 2]};
            ProjGrads gr;
            project_one_vjp(p, b, c, mean, covar, conic, comp, v_m2d, q.v_depths ? q.v_depths[e] : 0.f, v_conic, v_comp,
                            p.calc_comp, gr);
            v_mean[0] += gr.v_mean[0];
            v_mean[1] += gr.v_mean[1];
            v_mean[2] += gr.v_mean[2];
            v_cov = m3_add(v_cov, gr.v_cov);
            // SH: colors = max(sh(dir) + 0.5, 0); the clamp passes the gradient
            // where sh + 0.5 >= 0 (torch.clamp_min semantics).
            const float *vm = p.viewmats + ((size_t)b * p.C + c) * 16;
            float cp[3];
            campos_of(vm, cp);
            const float d0 = mean[0] - cp[0], d1 = mean[1] - cp[1], d2 = mean[2] - cp[2];
            const float inv = rsqrtf(d0 * d0 + d1 * d1 + d2 * d2);
            const float x = d0 * inv, y = d1 * inv, z = d2 * inv;
            float Y[NB];
            sh_eval<D>(x, y, z, Y);
            float raw[3] = {0.f, 0.f, 0.f};
            // coefficient f = 3 k + ch, streamed in 128-bit pieces when aligned
            for_each_coef<D>(coef, q.f.sh_vec, [&](int f, float cf) { raw[f % 3] += Y[f / 3] * cf; });
            float vc[3];
#pragma unroll
            for (int ch = 0; ch < 3; ++ch) vc[ch] = (raw[ch] + 0.5f >= 0.f) ? q.v_colors[e * 3 + ch] : 0.f;
#pragma unroll
            for (int k = 0; k < NB; ++k) {
                vsh[k * 3 + 0] += Y[k] * vc[0];
                vsh[k * 3 + 1] += Y[k] * vc[1];
                vsh[k * 3 + 2] += Y[k] * vc[2];
            }
            if (D > 0) {
                float w[NB];
#pragma unroll
                for (int k = 0; k < NB; ++k) w[k] = 0.f;
                for_each_coef<D>(coef, q.f.sh_vec, [&](int f, float cf) { w[f / 3] += cf * vc[f % 3]; });
                float gn[3];
                sh_grad_dot<D>(x, y, z, w, gn);
                const float dd = gn[0] * x + gn[1] * y + gn[2] * z;
                v_mean[0] += (gn[0] - dd * x) * inv;
                v_mean[1] += (gn[1] - dd * y) * inv;
                v_mean[2] += (gn[2] - dd * z) * inv;
            }
        }
        if (any) {
            M3 Rq = quat_to_rotmat(quat[0], quat[1], quat[2], quat[3]);
            covar_from_quat_scale_vjp(quat, scale, Rq, v_cov, v_q, v_s);
        }
        q.v_means[gi * 3 + 0] = v_mean[0];
        q.v_means[gi * 3 + 1] = v_mean[1];
        q.v_means[gi * 3 + 2] = v_mean[2];
        q.v_quats[gi * 4 + 0] = v_q[0];
        q.v_quats[gi * 4 + 1] = v_q[1];
        q.v_quats[gi * 4 + 2] = v_q[2];
        q.v_quats[gi * 4 + 3] = v_q[3];
        q.v_scales[gi * 3 + 0] = v_s[0];
        q.v_scales[gi * 3 + 1] = v_s[1];
        q.v_scales[gi * 3 + 2] = v_s[2];
        q.v_opacities[gi] = v_op;
    }
    __syncthreads();
    // one warp per staged row: 32 lanes copy consecutive coefficients (no
    // index division), so each row leaves as coalesced 128-byte pieces
    const size_t total = (size_t)p.B * p.N;
    const uint32_t count = (total - first) < kFusedBwdThreads ? (uint32_t)(total - first) : kFusedBwdThreads;
    float *dst = q.v_sh + first * K3;
    const uint32_t lane = tid & 31u;
    for (uint32_t r = tid >> 5; r < count; r += kFusedBwdThreads / 32) {
        const float *row = s_vsh + (size_t)r * stride;
        float *out = dst + (size_t)r * K3;
        for (uint32_t c = lane; c < K3; c += 32) out[c] = row[c];
    }
}

template <int D> static void launch_dense_fwd(const FusedParams &f, int32_t *radii, float *means2d,
                                              float *depths, float *conics, float *comps,
                                              float *colors, float *opac, cudaStream_t s) {
    const uint32_t n = f.p.B * f.p.N;
    fused_dense_fwd_kernel<D><<<(n + 255) / 256, 256, 0, s>>>(f, radii, means2d, depths, conics,
                                                              comps, colors, opac);
}

template <int D>
static void launch_packed_write(const FusedParams &f, const uint32_t *vis, const int64_t *accum,
                                int64_t nnz, int32_t *indptr, int64_t *bids, int64_t *cids,
                                int64_t *gids, int32_t *radii, float *means2d, float *depths,
                                float *conics, float *comps, float *colors, float *opac,
                                int32_t *pair_index, cudaStream_t s) {
    dim3 grid((f.p.N + 255) / 256, f.p.B * f.p.C);
    fused_packed_write_kernel<D><<<grid, 256, 0, s>>>(f, vis, accum, nnz, indptr, bids, cids, gids,
                                                      radii, means2d, depths, conics, comps, colors,
                                                      opac, pair_index);
}

template <int D> static void launch_bwd(const FusedBwdParams &q, cudaStream_t s) {
    const uint32_t n = q.f.p.B * q.f.p.N;
    const size_t smem = (size_t)kFusedBwdThreads * ((q.f.K * 3) | 1u) * sizeof(float);
    if (smem > 48 * 1024)
        cudaFuncSetAttribute(fused_bwd_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    fused_bwd_kernel<D><<<(n + kFusedBwdThreads - 1) / kFusedBwdThreads, kFusedBwdThreads, smem, s>>>(q);
}

static int check_fused(int degree, int K, int camera_model, const float *quats, const float *scales,
                       const float *opacities, const float *sh) {
    if (camera_model != kPinhole && camera_model != kOrtho && camera_model != kFisheye)
        return set_error(kErrUnsupported, "camera_model %d is not supported (pinhole=0, ortho=1, fisheye=2)",
                         camera_model);
    if (degree < 0 || degree > 4)
        return set_error(kErrUnsupported, "spherical harmonics degree %d not in [0, 4]", degree);
    if ((degree + 1) * (degree + 1) > K || K > 64)
        return set_error(kErrInvalidArgument, "K=%d coefficients does not fit degree %d (K <= 64)", K, degree);
    if (!quats || !scales || !opacities || !sh)
        return set_error(kErrInvalidArgument, "fused projection needs quats, scales, opacities and sh");
    return kOk;
}

static FusedParams make_fused(int B, int C, int N, const float *means, const float *quats,
                              const float *scales, const float *opacities, const float *sh, int K,
                              const float *viewmats, const float *Ks, int W, int H, float eps2d,
                              float near_plane, float far_plane, float radius_clip, int calc_comp,
                              int camera_model) {
    FusedParams f;
    ProjParams &p = f.p;
    p.B = B;
    p.C = C;
    p.N = N;
    p.means = means;
    p.covars = nullptr;
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
    f.sh = sh;
    f.K = K;
    f.sh_vec = (K * 3) % 4 == 0 && (reinterpret_cast<uintptr_t>(sh) & 15u) == 0;
    return f;
}

#define GSB_SH_SWITCH(DEG, CALL)                                                                  \
    switch (DEG) {                                                                                \
    case 0: CALL(0); break;                                                                       \
    case 1: CALL(1); break;                                                                       \
    case 2: CALL(2); break;                                                                       \
    case 3: CALL(3); break;                                                                       \
    default: CALL(4); break;                                                                      \
    }

} // namespace gsb

using namespace gsb;

extern "C" int gsb_projection_sh_dense_fwd(int B, int C, int N, const float *means,
                                           const float *quats, const float *scales,
                                           const float *opacities, const float *sh, int K,
                                           int sh_degree, const float *viewmats, const float *Ks,
                                           int width, int height, float eps2d, float near_plane,
                                           float far_plane, float radius_clip,
                                           int calc_compensations, int camera_model,
                                           int32_t *radii, float *means2d, float *depths,
                                           float *conics, float *compensations, float *colors,
                                           float *opacities_out, cudaStream_t stream) {
    if ((size_t)B * N == 0 || C == 0) return kOk;
    if (int e = check_fused(sh_degree, K, camera_model, quats, scales, opacities, sh)) return e;
    FusedParams f = make_fused(B, C, N, means, quats, scales, opacities, sh, K, viewmats, Ks, width,
                               height, eps2d, near_plane, far_plane, radius_clip,
                               calc_compensations, camera_model);
    float *comps = calc_compensations ? compensations : nullptr;
#define GSB_CALL(D) launch_dense_fwd<D>(f, radii, means2d, depths, conics, comps, colors, opacities_out, stream)
    GSB_SH_SWITCH(sh_degree, GSB_CALL)
#undef GSB_CALL
    return check_launch("fused_dense_fwd_kernel");
}

extern "C" int gsb_projection_sh_packed_write(
    int B, int C, int N, const float *means, const float *quats, const float *scales,
    const float *opacities, const float *sh, int K, int sh_degree, const float *viewmats,
    const float *Ks, int width, int height, float eps2d, float near_plane, float far_plane,
    float radius_clip, int calc_compensations, int camera_model, const uint32_t *vis_bits,
    const int64_t *block_accum, long long nnz, int32_t *indptr, int64_t *batch_ids,
    int64_t *camera_ids, int64_t *gaussian_ids, int32_t *radii, float *means2d, float *depths,
    float *conics, float *compensations, float *colors, float *opacities_out, int32_t *pair_index,
    cudaStream_t stream) {
    if ((size_t)B * C == 0 || N == 0) return kOk;
    if (int e = check_fused(sh_degree, K, camera_model, quats, scales, opacities, sh)) return e;
    FusedParams f = make_fused(B, C, N, means, quats, scales, opacities, sh, K, viewmats, Ks, width,
                               height, eps2d, near_plane, far_plane, radius_clip,
                               calc_compensations, camera_model);
    float *comps = calc_compensations ? compensations : nullptr;
#define GSB_CALL(D)                                                                               \
    launch_packed_write<D>(f, vis_bits, block_accum, nnz, indptr, batch_ids, camera_ids,           \
                           gaussian_ids, radii, means2d, depths, conics, comps, colors,            \
                           opacities_out, pair_index, stream)
    GSB_SH_SWITCH(sh_degree, GSB_CALL)
#undef GSB_CALL
    return check_launch("fused_packed_write_kernel");
}

extern "C" int gsb_projection_sh_bwd(
    int B, int C, int N, int packed, const float *means, const float *quats, const float *scales,
    const float *opacities, const float *sh, int K, int sh_degree, const float *viewmats,
    const float *Ks, int width, int height, float eps2d, int calc_compensations, int camera_model,
    const int32_t *pair_index, const int32_t *radii, const float *conics,
    const float *compensations, const float *v_means2d, const float *v_depths,
    const float *v_conics, const float *v_compensations, const float *v_colors,
    const float *v_opacities_out, float *v_means, float *v_quats, float *v_scales,
    float *v_opacities, float *v_sh, cudaStream_t stream) {
    if ((size_t)B * N == 0) return kOk;
    if (int e = check_fused(sh_degree, K, camera_model, quats, scales, opacities, sh)) return e;
    if (packed ? pair_index == nullptr : radii == nullptr)
        return set_error(kErrInvalidArgument, "pair_index (packed) or radii (dense) is required");
    if (calc_compensations && compensations == nullptr)
        return set_error(kErrInvalidArgument, "compensations are required when calc_compensations is set");
    FusedBwdParams q;
    q.f = make_fused(B, C, N, means, quats, scales, opacities, sh, K, viewmats, Ks, width, height,
                     eps2d, 0.f, 0.f, 0.f, calc_compensations, camera_model);
    q.packed = packed != 0;
    q.pair_index = pair_index;
    q.radii = radii;
    q.conics = conics;
    q.comps = compensations;
    q.v_means2d = v_means2d;
    q.v_depths = v_depths;
    q.v_conics = v_conics;
    q.v_comps = v_compensations;
    q.v_colors = v_colors;
    q.v_opac = v_opacities_out;
    q.v_means = v_means;
    q.v_quats = v_quats;
    q.v_scales = v_scales;
    q.v_opacities = v_opacities;
    q.v_sh = v_sh;
#define GSB_CALL(D) launch_bwd<D>(q, stream)
    GSB_SH_SWITCH(sh_degree, GSB_CALL)
#undef GSB_CALL
    return check_launch("fused_bwd_kernel");
}
