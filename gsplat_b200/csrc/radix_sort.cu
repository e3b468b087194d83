// Stable LSD radix sort of (uint64 key, int32 value) pairs, 8-bit digits.
//
// Replaces cub::DeviceRadixSort::SortPairs in the reference
// (gsplat/cuda/csrc/IntersectTile.cu:478-521), which sorts bits [0, 32 +
// tile_bits + image_bits) of the intersection keys. Like cub's DoubleBuffer the
// sort ping-pongs between the caller's input arrays and an alternate pair and
// reports which pair holds the result.
//
// Each pass over 8 bits is three launches:
//   1. upsweep:   per-tile digit histograms (tile = 2048 keys), digit-major
//   2. scan:      inclusive scan of the [256 x tiles] histogram (scan.cu)
//   3. downsweep: stable in-tile ranking with warp match/popc, a local sort of
//                 the tile in shared memory, then coalesced runs written out.
// Ranking order inside a tile is (warp, round, lane) and each warp owns a
// contiguous 256-key slice, so the pass is stable.
#include "common.cuh"
#include "gsb_internal.h"
#include "gsb_scan.cuh"

namespace gsb {

constexpr int kSortThreads = 256;
constexpr int kSortWarps = kSortThreads / 32;
constexpr int kSortItems = 8; // per lane
constexpr int kSortTile = kSortThreads * kSortItems;
constexpr int kWarpSlice = 32 * kSortItems;
constexpr int kRadix = 256;

__global__ void __launch_bounds__(kSortThreads)
    radix_upsweep(const uint64_t *__restrict__ keys, uint32_t n, uint32_t shift, uint32_t ntiles,
                  int32_t *__restrict__ hist) {
    __shared__ uint32_t h[kSortWarps][kRadix];
    for (int i = threadIdx.x; i < kSortWarps * kRadix; i += kSortThreads) (&h[0][0])[i] = 0;
    __syncthreads();
    const int warp = threadIdx.x >> 5;
    const size_t base = (size_t)blockIdx.x * kSortTile;
#pragma unroll 4
    for (int i = 0; i < kSortItems; ++i) {
        const size_t k = base + (size_t)i * kSortThreads + threadIdx.x;
        if (k < n) atomicAdd(&h[warp][(uint32_t)(keys[k] >> shift) & 0xffu], 1u);
    }
    __syncthreads();
    for (int d = threadIdx.x; d < kRadix; d += kSortThreads) {
        uint32_t s = 0;
#pragma unroll
        for (int w = 0; w < kSortWarps; ++w) s += h[w][d];
        hist[(size_t)d * ntiles + blockIdx.x] = (int32_t)s;
    }
}

struct DownsweepSmem {
    uint64_t keys[kSortTile];
    int32_t vals[kSortTile];
    uint32_t cnt[kSortWarps][kRadix]; // per-warp digit counts, then exclusive warp prefix
    uint32_t local_start[kRadix];     // first position of each digit in the local sort
    int64_t gbase[kRadix];            // global position of each digit's first key of this tile
    uint32_t scan_tmp[kSortWarps];
};

__global__ void __launch_bounds__(kSortThreads)
    radix_downsweep(const uint64_t *__restrict__ keys_in, const int32_t *__restrict__ vals_in,
                    uint64_t *__restrict__ keys_out, int32_t *__restrict__ vals_out, uint32_t n,
                    uint32_t shift, uint32_t ntiles, const int64_t *__restrict__ hist_incl) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    DownsweepSmem &S = *reinterpret_cast<DownsweepSmem *>(smem_raw);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int i = threadIdx.x; i < kSortWarps * kRadix; i += kSortThreads) (&S.cnt[0][0])[i] = 0;
    __syncthreads();

    const size_t tile_base = (size_t)blockIdx.x * kSortTile;
    const size_t warp_base = tile_base + (size_t)warp * kWarpSlice;
    const uint32_t lt_mask = (1u << lane) - 1u;
    uint64_t k[kSortItems];
    int32_t v[kSortItems];
    uint32_t rank[kSortItems];
#pragma unroll
    for (int r = 0; r < kSortItems; ++r) {
        const size_t pos = warp_base + (size_t)r * 32 + lane;
        const bool valid = pos < n;
        k[r] = valid ? keys_in[pos] : 0ull;
        v[r] = valid ? vals_in[pos] : 0;
        const uint32_t d = valid ? ((uint32_t)(k[r] >> shift) & 0xffu) : kRadix;
        const uint32_t peers = __match_any_sync(0xffffffffu, d);
        const uint32_t before = __popc(peers & lt_mask);
        uint32_t prior = 0;
        if (valid) prior = S.cnt[warp][d];
        __syncwarp();
        if (valid && before == 0) S.cnt[warp][d] = prior + __popc(peers);
        __syncwarp();
        rank[r] = prior + before;
    }
    __syncthreads();
    // Exclusive prefix over warps per digit, digit totals, and the local digit starts.
    uint32_t total = 0;
    const int d = threadIdx.x; // kSortThreads == kRadix
    {
#pragma unroll
        for (int w = 0; w < kSortWarps; ++w) {
            const uint32_t c = S.cnt[w][d];
            S.cnt[w][d] = total;
            total += c;
        }
    }
    // block exclusive scan of digit totals
    uint32_t incl = total;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t u = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += u;
    }
    if (lane == 31) S.scan_tmp[warp] = incl;
    __syncthreads();
    uint32_t wbase = 0;
    for (int w = 0; w < warp; ++w) wbase += S.scan_tmp[w];
    S.local_start[d] = wbase + incl - total;
    S.gbase[d] = hist_incl[(size_t)d * ntiles + blockIdx.x] - (int64_t)total;
    __syncthreads();
    // Local sort into shared memory.
#pragma unroll
    for (int r = 0; r < kSortItems; ++r) {
        const size_t pos = warp_base + (size_t)r * 32 + lane;
        if (pos < n) {
            const uint32_t dd = (uint32_t)(k[r] >> shift) & 0xffu;
            const uint32_t lp = S.local_start[dd] + S.cnt[warp][dd] + rank[r];
            S.keys[lp] = k[r];
            S.vals[lp] = v[r];
        }
    }
    __syncthreads();
    const uint32_t count = (uint32_t)min((size_t)kSortTile, (size_t)n - tile_base);
    for (uint32_t i = threadIdx.x; i < count; i += kSortThreads) {
        const uint64_t key = S.keys[i];
        const uint32_t dd = (uint32_t)(key >> shift) & 0xffu;
        const int64_t gp = S.gbase[dd] + (int64_t)(i - S.local_start[dd]);
        if (gp >= 0 && gp < (int64_t)n) {
            keys_out[gp] = key;
            vals_out[gp] = S.vals[i];
        }
    }
}

size_t radix_sort_scratch_bytes(size_t n) {
    const size_t ntiles = (n + kSortTile - 1) / kSortTile;
    const size_t hn = (ntiles > 0 ? ntiles : 1) * kRadix;
    size_t bytes = hn * sizeof(int32_t);
    bytes = (bytes + 255) & ~(size_t)255;
    bytes += hn * sizeof(int64_t);
    bytes = (bytes + 255) & ~(size_t)255;
    bytes += scan_scratch_bytes(hn);
    return bytes;
}

// Sorts bits [0, end_bit). Returns 0 when the result is in (keys, vals), 1 when
// it is in (keys_alt, vals_alt), negative on error.
int radix_sort_pairs(uint64_t *keys, int32_t *vals, uint64_t *keys_alt, int32_t *vals_alt, size_t n,
                     int end_bit, void *scratch, size_t scratch_bytes, cudaStream_t stream) {
    if (n == 0) return 0;
    if (n > 0x7fffffffu) return set_error(kErrInvalidArgument, "radix sort: too many keys (%zu)", n);
    if (end_bit < 0 || end_bit > 64) return set_error(kErrInvalidArgument, "radix sort: bad end_bit");
    if (scratch_bytes < radix_sort_scratch_bytes(n))
        return set_error(kErrInvalidArgument, "radix sort scratch too small");
    const uint32_t ntiles = (uint32_t)((n + kSortTile - 1) / kSortTile);
    const size_t hn = (size_t)ntiles * kRadix;
    unsigned char *sp = static_cast<unsigned char *>(scratch);
    int32_t *hist = reinterpret_cast<int32_t *>(sp);
    size_t off = (hn * sizeof(int32_t) + 255) & ~(size_t)255;
    int64_t *hist_incl = reinterpret_cast<int64_t *>(sp + off);
    off += (hn * sizeof(int64_t) + 255) & ~(size_t)255;
    void *scan_scratch = sp + off;
    const size_t scan_bytes = scratch_bytes - off;

    const int smem = (int)sizeof(DownsweepSmem);
    cudaFuncSetAttribute(radix_downsweep, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    uint64_t *kin = keys, *kout = keys_alt;
    int32_t *vin = vals, *vout = vals_alt;
    int which = 0;
    for (int shift = 0; shift < end_bit; shift += 8) {
        radix_upsweep<<<ntiles, kSortThreads, 0, stream>>>(kin, (uint32_t)n, shift, ntiles, hist);
        if (int e = inclusive_scan_i32_i64(hist, hist_incl, hn, scan_scratch, scan_bytes, stream)) return e;
        radix_downsweep<<<ntiles, kSortThreads, smem, stream>>>(kin, vin, kout, vout, (uint32_t)n,
                                                                shift, ntiles, hist_incl);
        if (int e = check_launch("radix_downsweep")) return e;
        uint64_t *tk = kin;
        kin = kout;
        kout = tk;
        int32_t *tv = vin;
        vin = vout;
        vout = tv;
        which ^= 1;
    }
    return which;
}

} // namespace gsb

extern "C" size_t gsb_radix_sort_scratch_bytes(long long n) {
    return gsb::radix_sort_scratch_bytes((size_t)(n > 0 ? n : 0));
}

extern "C" int gsb_radix_sort_pairs(int64_t *keys, int32_t *vals, int64_t *keys_alt,
                                    int32_t *vals_alt, long long n, int end_bit, void *scratch,
                                    size_t scratch_bytes, cudaStream_t stream) {
    if (n < 0) return gsb::set_error(gsb::kErrInvalidArgument, "negative length");
    return gsb::radix_sort_pairs(reinterpret_cast<uint64_t *>(keys), vals,
                                 reinterpret_cast<uint64_t *>(keys_alt), vals_alt, (size_t)n,
                                 end_bit, scratch, scratch_bytes, stream);
}
