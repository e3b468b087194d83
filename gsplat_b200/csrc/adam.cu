// Selective (masked) Adam update.
//
// Reference behaviour: gsplat/cuda/csrc/AdamCUDA.cu:34-69 -- for every element
// whose row is visible: m = b1 m + (1 - b1) g; v = b2 v + (1 - b2) g^2;
// p += -lr m / (sqrt(v) + eps). No bias correction. Rows with valid[row] == false
// are left untouched (neither the state nor the parameter is read or written).
//
// All parameter groups of one optimizer step go through a single launch. Each
// group is streamed with 128-bit loads/stores when its arrays are 16-byte
// aligned; a float4 whose four rows are all hidden is skipped without touching
// HBM, so the traffic is proportional to the visible fraction.
#include "common.cuh"
#include "gsb_internal.h"

namespace gsb {

constexpr int kAdamMaxGroups = 8;
constexpr int kAdamThreads = 256;

struct AdamBatch {
    GsbAdamGroup g[kAdamMaxGroups];
    long long block_start[kAdamMaxGroups + 1]; // first block of each group
    int n_groups;
    int vec[kAdamMaxGroups]; // 1 when the group uses float4 access
    float b1, b2;
    const bool *valid;
};

__device__ __forceinline__ void adam_elem(float &p, float g, float &m, float &v, float lr, float b1,
                                          float b2, float eps) {
    m = b1 * m + (1.f - b1) * g;
    v = b2 * v + (1.f - b2) * g * g;
    p += -lr * m / (sqrtf(v) + eps);
}

__global__ void __launch_bounds__(kAdamThreads) adam_multi_kernel(AdamBatch B) {
    int gi = 0;
    while (gi + 1 < B.n_groups && (long long)blockIdx.x >= B.block_start[gi + 1]) ++gi;
    const GsbAdamGroup &G = B.g[gi];
    const long long local_block = (long long)blockIdx.x - B.block_start[gi];
    const long long t = local_block * kAdamThreads + threadIdx.x;
    const int D = G.D;
    if (B.vec[gi]) {
        const long long e0 = t * 4;
        if (e0 >= G.numel) return;
        bool vis[4];
        bool anyv = false;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            vis[j] = B.valid == nullptr || B.valid[(e0 + j) / D];
            anyv |= vis[j];
        }
        if (!anyv) return;
        float4 p = *reinterpret_cast<float4 *>(G.param + e0);
        const float4 g = *reinterpret_cast<const float4 *>(G.grad + e0);
        float4 m = *reinterpret_cast<float4 *>(G.exp_avg + e0);
        float4 v = *reinterpret_cast<float4 *>(G.exp_avg_sq + e0);
        float pp[4] = {p.x, p.y, p.z, p.w}, gg[4] = {g.x, g.y, g.z, g.w};
        float mm[4] = {m.x, m.y, m.z, m.w}, vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j)
            if (vis[j]) adam_elem(pp[j], gg[j], mm[j], vv[j], G.lr, B.b1, B.b2, G.eps);
        *reinterpret_cast<float4 *>(G.param + e0) = make_float4(pp[0], pp[1], pp[2], pp[3]);
        *reinterpret_cast<float4 *>(G.exp_avg + e0) = make_float4(mm[0], mm[1], mm[2], mm[3]);
        *reinterpret_cast<float4 *>(G.exp_avg_sq + e0) = make_float4(vv[0], vv[1], vv[2], vv[3]);
    } else {
        if (t >= G.numel) return;
        if (B.valid != nullptr && !B.valid[t / D]) return;
        float p = G.param[t], m = G.exp_avg[t], v = G.exp_avg_sq[t];
        adam_elem(p, G.grad[t], m, v, G.lr, B.b1, B.b2, G.eps);
        G.param[t] = p;
        G.exp_avg[t] = m;
        G.exp_avg_sq[t] = v;
    }
}

static bool aligned16(const void *ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

} // namespace gsb

using namespace gsb;

extern "C" int gsb_adam_multi(int n_groups, const GsbAdamGroup *groups, const bool *valid,
                              float b1, float b2, cudaStream_t stream) {
    if (n_groups < 0) return set_error(kErrInvalidArgument, "negative group count");
    int done = 0;
    while (done < n_groups) {
        AdamBatch B = {};
        B.b1 = b1;
        B.b2 = b2;
        B.valid = valid;
        long long blocks = 0;
        int n = 0;
        for (; n < kAdamMaxGroups && done + n < n_groups; ++n) {
            const GsbAdamGroup &g = groups[done + n];
            if (g.D <= 0 && g.numel > 0) return set_error(kErrInvalidArgument, "group %d has D <= 0", done + n);
            B.g[n] = g;
            const bool vec = (g.numel % 4 == 0) && aligned16(g.param) && aligned16(g.grad) &&
                             aligned16(g.exp_avg) && aligned16(g.exp_avg_sq);
            B.vec[n] = vec ? 1 : 0;
            B.block_start[n] = blocks;
            const long long items = vec ? g.numel / 4 : g.numel;
            blocks += (items + kAdamThreads - 1) / kAdamThreads;
        }
        B.block_start[n] = blocks;
        B.n_groups = n;
        if (blocks > 0) {
            if (blocks > 0x7fffffffll) return set_error(kErrInvalidArgument, "adam: too many elements");
            adam_multi_kernel<<<(unsigned)blocks, kAdamThreads, 0, stream>>>(B);
            if (int e = check_launch("adam_multi_kernel")) return e;
        }
        done += n;
    }
    return kOk;
}

extern "C" int gsb_adam(float *param, const float *grad, float *exp_avg, float *exp_avg_sq,
                        const bool *valid, long long N, long long D, float lr, float b1, float b2,
                        float eps, cudaStream_t stream) {
    GsbAdamGroup g;
    g.param = param;
    g.grad = grad;
    g.exp_avg = exp_avg;
    g.exp_avg_sq = exp_avg_sq;
    g.numel = N * D;
    g.D = (int)D;
    g.lr = lr;
    g.eps = eps;
    if (N * D == 0) return kOk;
    return gsb_adam_multi(1, &g, valid, b1, b2, stream);
}
