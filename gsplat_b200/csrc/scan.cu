// Inclusive prefix sum of int32 counts into int64 offsets.
//
// Replaces the at::cumsum calls of the reference's two-pass pipelines
// (gsplat/cuda/csrc/Intersect.cpp:100-101 for tiles per Gaussian,
// Projection.cpp:380-394 for the packed block counts). Three launches without any
// inter-block waiting: per-tile sums, a single-block scan of the tile sums, and a
// final pass that rescans each tile and adds its base. Each tile is 2048 values
// (256 threads x 8); the input is read twice, the output written once.
#include "common.cuh"
#include "gsb_internal.h"
#include "gsb_scan.cuh"

namespace gsb {

constexpr int kScanThreads = 256;
constexpr int kScanItems = 8;
constexpr int kScanTile = kScanThreads * kScanItems;

template <typename T> __device__ __forceinline__ T warp_incl_scan(T v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const T u = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += u;
    }
    return v;
}

// Block-wide exclusive scan of one value per thread; returns the block total.
template <typename T> __device__ T block_excl_scan(T v, T &excl) {
    __shared__ T warp_tot[kScanThreads / 32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const T incl = warp_incl_scan(v);
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        T w = lane < kScanThreads / 32 ? warp_tot[lane] : T(0);
        w = warp_incl_scan(w);
        if (lane < kScanThreads / 32) warp_tot[lane] = w;
    }
    __syncthreads();
    const T base = warp == 0 ? T(0) : warp_tot[warp - 1];
    excl = base + incl - v;
    const T total = warp_tot[kScanThreads / 32 - 1];
    __syncthreads();
    return total;
}

__global__ void __launch_bounds__(kScanThreads) scan_tile_sums(const int32_t *__restrict__ in,
                                                               size_t n, int64_t *tile_sums) {
    const size_t base = (size_t)blockIdx.x * kScanTile;
    int64_t s = 0;
#pragma unroll
    for (int i = 0; i < kScanItems; ++i) {
        const size_t k = base + (size_t)i * kScanThreads + threadIdx.x;
        if (k < n) s += in[k];
    }
    int64_t excl;
    const int64_t tot = block_excl_scan<int64_t>(s, excl);
    if (threadIdx.x == 0) tile_sums[blockIdx.x] = tot;
}

// Exclusive scan of the tile sums in place, one block looping over chunks.
__global__ void __launch_bounds__(kScanThreads) scan_tile_bases(int64_t *tile_sums, size_t ntiles) {
    __shared__ int64_t carry;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    for (size_t start = 0; start < ntiles; start += kScanThreads) {
        const size_t k = start + threadIdx.x;
        const int64_t v = k < ntiles ? tile_sums[k] : 0;
        int64_t excl;
        const int64_t tot = block_excl_scan<int64_t>(v, excl);
        const int64_t c = carry;
        if (k < ntiles) tile_sums[k] = c + excl;
        __syncthreads();
        if (threadIdx.x == 0) carry = c + tot;
        __syncthreads();
    }
}

__global__ void __launch_bounds__(kScanThreads) scan_tile_apply(const int32_t *__restrict__ in, size_t n,
                                                                const int64_t *__restrict__ tile_bases,
                                                                int64_t *__restrict__ out) {
    const size_t base = (size_t)blockIdx.x * kScanTile + (size_t)threadIdx.x * kScanItems;
    int64_t v[kScanItems];
    int64_t s = 0;
#pragma unroll
    for (int i = 0; i < kScanItems; ++i) {
        const size_t k = base + i;
        s += (k < n) ? in[k] : 0;
        v[i] = s;
    }
    int64_t excl;
    block_excl_scan<int64_t>(s, excl);
    const int64_t off = tile_bases[blockIdx.x] + excl;
#pragma unroll
    for (int i = 0; i < kScanItems; ++i) {
        const size_t k = base + i;
        if (k < n) out[k] = off + v[i];
    }
}

size_t scan_scratch_bytes(size_t n) {
    const size_t tiles = (n + kScanTile - 1) / kScanTile;
    return (tiles > 0 ? tiles : 1) * sizeof(int64_t);
}

int inclusive_scan_i32_i64(const int32_t *in, int64_t *out, size_t n, void *scratch,
                           size_t scratch_bytes, cudaStream_t stream) {
    if (n == 0) return kOk;
    if (scratch_bytes < scan_scratch_bytes(n))
        return set_error(kErrInvalidArgument, "scan scratch too small: %zu < %zu", scratch_bytes,
                         scan_scratch_bytes(n));
    const size_t tiles = (n + kScanTile - 1) / kScanTile;
    int64_t *tile_sums = static_cast<int64_t *>(scratch);
    scan_tile_sums<<<tiles, kScanThreads, 0, stream>>>(in, n, tile_sums);
    scan_tile_bases<<<1, kScanThreads, 0, stream>>>(tile_sums, tiles);
    scan_tile_apply<<<tiles, kScanThreads, 0, stream>>>(in, n, tile_sums, out);
    return check_launch("inclusive_scan_i32_i64");
}

} // namespace gsb

extern "C" size_t gsb_scan_scratch_bytes(long long n) { return gsb::scan_scratch_bytes((size_t)n); }

extern "C" int gsb_inclusive_scan_i32(const int32_t *in, int64_t *out, long long n, void *scratch,
                                      size_t scratch_bytes, cudaStream_t stream) {
    if (n < 0) return gsb::set_error(gsb::kErrInvalidArgument, "negative length");
    return gsb::inclusive_scan_i32_i64(in, out, (size_t)n, scratch, scratch_bytes, stream);
}
