// Inclusive prefix sum of int32 counts into int64 offsets.
//
// Replaces the at::cumsum calls of the reference's two-pass pipelines
// (gsplat/cuda/csrc/Intersect.cpp:100-101 for tiles per Gaussian,
// Projection.cpp:380-394 for the packed block counts). Three launches without any
// inter-block waiting: per-tile sums, a single-block scan of the tile sums, and a
// final pass that rescans each tile and adds its base. Each tile is 2048 values
// (256 threads x 8); the input is read twice, the output written once.
#include <mutex>

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

// ---------------------------------------------------------------------------
// Allocation-free variant
//
// Some callers cannot allocate device memory at the point where they need a
// prefix sum: code that runs inside a host application which owns every device
// allocation itself (a rendering engine or plugin host with a fixed, pre-reserved
// memory budget), or code called from an allocator's own callbacks, where a
// cudaMalloc would re-enter the allocator. For them the tile sums live in a
// file-scope device array instead of a caller-provided buffer.
//
// The array holds kNoAllocMaxTiles tile sums, i.e. inputs of up to
// kNoAllocMaxTiles * kScanTile = 2^27 values; every GPU that loads this library
// keeps the 512 KiB for the life of the process. Every call on a device shares
// the one array and leaves its tile sums behind; nothing in it needs to start at
// zero (each call writes the sums of all its tiles before reading them), but two
// calls that overlap on the GPU (different streams, no ordering) race on it.
// ---------------------------------------------------------------------------
constexpr size_t kNoAllocMaxTiles = 65536;
constexpr long long kNoAllocMaxN = (long long)kNoAllocMaxTiles * kScanTile;
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) int64_t g_noalloc_tile_sums[kNoAllocMaxTiles];

static std::mutex g_noalloc_mutex;
static void *g_noalloc_addr[kNoAllocMaxDevices] = {};

// Device address of g_noalloc_tile_sums on the current device. In host code the
// symbol is only a host-side stand-in, so the address is looked up once per
// device with that device current and cached.
static int noalloc_scratch(void **addr) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess)
        return set_error(kErrLaunch, "cudaGetDevice failed: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= kNoAllocMaxDevices)
        return set_error(kErrUnsupported, "device %d beyond the %d supported by the allocation-free scan", dev,
                         kNoAllocMaxDevices);
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (g_noalloc_addr[dev] == nullptr) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_tile_sums);
        if (e != cudaSuccess)
            return set_error(kErrLaunch, "cudaGetSymbolAddress(g_noalloc_tile_sums) failed: %s",
                             cudaGetErrorString(e));
        g_noalloc_addr[dev] = p;
    }
    *addr = g_noalloc_addr[dev];
    return kOk;
}

} // namespace gsb

extern "C" int gsb_inclusive_scan_i32_noalloc(const int32_t *in, int64_t *out, long long n,
                                              cudaStream_t stream) {
    using namespace gsb;
    if (n < 0) return set_error(kErrInvalidArgument, "negative length");
    if (n > kNoAllocMaxN)
        return set_error(kErrInvalidArgument,
                         "gsb_inclusive_scan_i32_noalloc: n = %lld exceeds the maximum of %lld values "
                         "held by its static scratch; use gsb_inclusive_scan_i32 with a caller buffer",
                         n, kNoAllocMaxN);
    if (n == 0) return kOk;
    void *scratch = nullptr;
    if (int e = noalloc_scratch(&scratch)) return e;
    return inclusive_scan_i32_i64(in, out, (size_t)n, scratch, kNoAllocMaxTiles * sizeof(int64_t),
                                  stream);
}

extern "C" size_t gsb_scan_scratch_bytes(long long n) { return gsb::scan_scratch_bytes((size_t)n); }

extern "C" int gsb_inclusive_scan_i32(const int32_t *in, int64_t *out, long long n, void *scratch,
                                      size_t scratch_bytes, cudaStream_t stream) {
    if (n < 0) return gsb::set_error(gsb::kErrInvalidArgument, "negative length");
    return gsb::inclusive_scan_i32_i64(in, out, (size_t)n, scratch, scratch_bytes, stream);
}
