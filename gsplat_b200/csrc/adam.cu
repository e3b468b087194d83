// Selective (masked) Adam update.
//
// Reference behaviour: gsplat/cuda/csrc/AdamCUDA.cu:34-69 -- for every element
// whose row is visible: m = b1 m + (1 - b1) g; v = b2 v + (1 - b2) g^2;
// p += -lr m / (sqrt(v) + eps). No bias correction. Rows with valid[row] == false
// are left untouched (neither the state nor the parameter is read or written).
//
// All parameter groups of one optimizer step go through a single launch (groups
// of any size: elements are indexed in 64 bits). Each
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
    unsigned long long row_magic[kAdamMaxGroups]; // ceil(2^64 / D), 0 for D = 1
    int n_groups;
    int vec[kAdamMaxGroups]; // 1 when the group uses float4 access
    float b1, b2;
    const bool *valid;
};

// Row of element e (< 2^32) of a group with D elements per row, without an
// integer division: division by an invariant integer through a multiply-high
// (Granlund and Montgomery, PLDI 1994). With M = ceil(2^64 / D) = (2^64 + r) / D,
// 0 <= r < D, e M / 2^64 = e / D + e r / (D 2^64), and the second term is below
// 2^-32 < 1 / D, so it never carries e / D past the next integer:
// floor(e M / 2^64) = floor(e / D). Groups of 2^32 elements or more are indexed
// from each block's first element (64-bit, one division per block), so the
// per-element offsets from that block's first row stay below 2^32.
__device__ __forceinline__ uint32_t row_of(uint32_t e, unsigned long long magic) {
    return magic == 0ull ? e : (uint32_t)__umul64hi((unsigned long long)e, magic);
}

// Hardware square root approximation (the reference's default fast-math build
// evaluates sqrtf this way; subnormal inputs are kept).
__device__ __forceinline__ float sqrt_approx(float x) {
    float y;
    asm("sqrt.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ void adam_elem(float &p, float g, float &m, float &v, float lr, float b1,
                                          float b2, float eps) {
    m = b1 * m + (1.f - b1) * g;
    v = b2 * v + (1.f - b2) * g * g;
    p += -lr * __fdividef(m, sqrt_approx(v) + eps);
}

#ifndef GSB_ADAM_VEC
#define GSB_ADAM_VEC 1
#endif
constexpr int kAdamVec = GSB_ADAM_VEC; // float4 (or scalar) items per thread, kAdamThreads apart

// Visibility of the rows of elements e .. e+3, where e = (first row of the
// block) * D + le: le is the offset from the block's first row (< 2^32).
__device__ __forceinline__ void rows_visible(const bool *valid, size_t row0, uint32_t le, uint32_t D,
                                             unsigned long long magic, bool vis[4]) {
    if (valid == nullptr) {
        vis[0] = vis[1] = vis[2] = vis[3] = true;
        return;
    }
    const uint32_t r0 = row_of(le, magic);
    const uint32_t rem = le - r0 * D;
#pragma unroll
    for (uint32_t j = 0; j < 4; ++j) {
        const uint32_t rr = rem + j;
        const uint32_t row = r0 + (rr >= D) + (rr >= 2 * D) + (rr >= 3 * D);
        vis[j] = valid[row0 + row];
    }
}

__global__ void __launch_bounds__(kAdamThreads) adam_multi_kernel(AdamBatch B) {
    int gi = 0;
    while (gi + 1 < B.n_groups && (long long)blockIdx.x >= B.block_start[gi + 1]) ++gi;
    const GsbAdamGroup &G = B.g[gi];
    const size_t local_block = (size_t)((long long)blockIdx.x - B.block_start[gi]);
    const uint32_t D = (uint32_t)G.D;
    const size_t numel = (size_t)G.numel;
    const float lr = G.lr, eps = G.eps, b1 = B.b1, b2 = B.b2;
    if (B.vec[gi]) {
        // elements of this block: [first, first + kAdamVec * kAdamThreads * 4)
        const size_t first = local_block * ((size_t)kAdamVec * kAdamThreads * 4);
        const size_t row0 = first / D;
        const uint32_t lbase = (uint32_t)(first - row0 * D);
        float4 p[kAdamVec], g[kAdamVec], m[kAdamVec], v[kAdamVec];
        bool vis[kAdamVec][4], act[kAdamVec];
        // issue every load of this thread before any arithmetic
#pragma unroll
        for (int it = 0; it < kAdamVec; ++it) {
            const uint32_t lo = ((uint32_t)it * kAdamThreads + threadIdx.x) * 4u;
            const size_t e0 = first + lo;
            act[it] = e0 < numel;
            if (act[it]) {
                rows_visible(B.valid, row0, lbase + lo, D, B.row_magic[gi], vis[it]);
                act[it] = vis[it][0] | vis[it][1] | vis[it][2] | vis[it][3];
            }
            if (act[it]) {
                p[it] = *reinterpret_cast<const float4 *>(G.param + e0);
                g[it] = *reinterpret_cast<const float4 *>(G.grad + e0);
                m[it] = *reinterpret_cast<const float4 *>(G.exp_avg + e0);
                v[it] = *reinterpret_cast<const float4 *>(G.exp_avg_sq + e0);
            }
        }
#pragma unroll
        for (int it = 0; it < kAdamVec; ++it) {
            if (!act[it]) continue;
            const size_t e0 = first + ((uint32_t)it * kAdamThreads + threadIdx.x) * 4u;
            float pp[4] = {p[it].x, p[it].y, p[it].z, p[it].w}, gg[4] = {g[it].x, g[it].y, g[it].z, g[it].w};
            float mm[4] = {m[it].x, m[it].y, m[it].z, m[it].w}, vv[4] = {v[it].x, v[it].y, v[it].z, v[it].w};
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (vis[it][j]) adam_elem(pp[j], gg[j], mm[j], vv[j], lr, b1, b2, eps);
            *reinterpret_cast<float4 *>(G.param + e0) = make_float4(pp[0], pp[1], pp[2], pp[3]);
            *reinterpret_cast<float4 *>(G.exp_avg + e0) = make_float4(mm[0], mm[1], mm[2], mm[3]);
            *reinterpret_cast<float4 *>(G.exp_avg_sq + e0) = make_float4(vv[0], vv[1], vv[2], vv[3]);
        }
    } else {
        const size_t first = local_block * ((size_t)kAdamVec * kAdamThreads);
        const size_t row0 = first / D;
        const uint32_t lbase = (uint32_t)(first - row0 * D);
#pragma unroll
        for (int it = 0; it < kAdamVec; ++it) {
            const uint32_t lo = (uint32_t)it * kAdamThreads + threadIdx.x;
            const size_t t = first + lo;
            if (t >= numel) continue;
            if (B.valid != nullptr && !B.valid[row0 + row_of(lbase + lo, B.row_magic[gi])]) continue;
            float p = G.param[t], m = G.exp_avg[t], v = G.exp_avg_sq[t];
            adam_elem(p, G.grad[t], m, v, lr, b1, b2, eps);
            G.param[t] = p;
            G.exp_avg[t] = m;
            G.exp_avg_sq[t] = v;
        }
    }
}

static bool aligned16(const void *ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

} // namespace gsb

using namespace gsb;

extern "C" int gsb_adam_multi(int n_groups, const GsbAdamGroup *groups, const bool *valid,
                              float b1, float b2, cudaStream_t stream) {
    if (n_groups < 0) return set_error(kErrInvalidArgument, "negative group count");
    if (n_groups > 0 && groups == nullptr) return set_error(kErrInvalidArgument, "adam: no group list");
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
            B.row_magic[n] = g.D <= 1 ? 0ull : ~0ull / (unsigned long long)g.D + 1ull;
            const bool vec = (g.numel % 4 == 0) && aligned16(g.param) && aligned16(g.grad) &&
                             aligned16(g.exp_avg) && aligned16(g.exp_avg_sq);
            B.vec[n] = vec ? 1 : 0;
            B.block_start[n] = blocks;
            const long long items = vec ? g.numel / 4 : g.numel;
            blocks += (items + (long long)kAdamThreads * kAdamVec - 1) / ((long long)kAdamThreads * kAdamVec);
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
