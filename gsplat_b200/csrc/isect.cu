// Tile intersection: per-splat tile counts, 64-bit key emission and tile offsets.
//
// Reference behaviour: gsplat/cuda/csrc/IntersectTile.cu:132-288 (count / emit
// with the AccuTile ellipse sweep at :40-126 and :195-253, AABB fallback at
// :254-287) and :391-439 (offset encode); host pipeline Intersect.cpp:33-176.
// Keys are image_id << (32 + tile_bits) | tile_id << 32 | float_bits(depth).
//
// Every float operation that decides which tiles a splat touches goes through
// the explicitly rounded helpers of detmath.h, so the CPU checker reproduces the
// tile sets bit for bit. The reference evaluates the ellipse level set with the
// hardware approximate logarithm (__logf); this implementation uses det_logf, a
// portable logarithm accurate to ~1 ulp, as documented in detmath.h.
#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "gsb_internal.h"
#include "gsb_scan.cuh"

namespace gsb {

struct IsectParams {
    bool packed;
    uint32_t I, N, nnz;
    const int64_t *image_ids;
    const float *means2d;
    const int32_t *radii;
    const float *depths;
    const float *conics;    // optional: AccuTile when conics and opacities are given
    const float *opacities; // optional
    uint32_t tile_size, tile_width, tile_height, tile_n_bits;
    // 1 / tile_size when tile_size is a power of two: x / 2^k and x * 2^-k are
    // the same correctly rounded value, so the multiplication is bit-identical
    // to the division (0 otherwise)
    float inv_tile_pow2;
    // packed only, optional: the splat count lives in device memory (nnz is then
    // the capacity of the arrays); lets the caller skip reading it back
    const int64_t *nnz_device;
};

struct EmitSink {
    int64_t *keys;
    int32_t *ids;
    int64_t cursor;
    int64_t limit; // end of this splat's slot range (count pass result)
    int64_t key_hi_base; // image_id << (32 + tile_bits)
    int64_t depth_bits;
    int32_t flat_id;
    __device__ __forceinline__ void put(int64_t tile_id) {
        // The emit pass repeats the count pass's arithmetic exactly; the bound
        // only guards the output arrays should the two ever disagree.
        if (cursor < limit) {
            keys[cursor] = key_hi_base | (tile_id << 32) | depth_bits;
            ids[cursor] = flat_id;
        }
        ++cursor;
    }
};

// x / tile_size, correctly rounded.
__device__ __forceinline__ float tile_div(const IsectParams &p, float x) {
    return p.inv_tile_pow2 != 0.f ? DET_MUL(x, p.inv_tile_pow2) : DET_DIV(x, (float)p.tile_size);
}

struct LinePair {
    float lo, hi;
};

// Intersection of the ellipse level set with the line u = coord (u = x when
// !is_y, u = y when is_y); IntersectTile.cu:40-52.
__device__ __forceinline__ LinePair ellipse_line(float A, float B, float C, float disc, float t,
                                                 float px, float py, bool is_y, float coord) {
    const float p_u = is_y ? py : px;
    const float p_v = is_y ? px : py;
    const float coeff = is_y ? A : C;
    const float h = DET_SUB(coord, p_u);
    const float sq = DET_SQRT(DET_ADD(DET_MUL(DET_MUL(disc, h), h), DET_MUL(t, coeff)));
    const float bh = DET_MUL(-B, h);
    LinePair r;
    r.lo = DET_ADD(DET_DIV(DET_SUB(bh, sq), coeff), p_v);
    r.hi = DET_ADD(DET_DIV(DET_ADD(bh, sq), coeff), p_v);
    return r;
}

// AccuTile sweep (IntersectTile.cu:54-126 and 195-253), in two parts: the set-up
// (level set, tile box, sweep direction) and the sweep over the box's columns.
// After the set-up the sweep runs along x when is_y is false and along y
// otherwise (the shorter side of the box, swapped into the *_x fields);
// ellipse_line still takes the unswapped centre.
struct TileSweep {
    float A, B, C, disc, t, mx, my;
    float bmin_x, bmax_x, bmin_y, bmax_y, amin_y, amax_y;
    int rmin_x, rmax_x, rmin_y, rmax_y;
    bool is_y;
};

// False when the splat's tile box is empty.
__device__ __forceinline__ bool accutile_setup(const IsectParams &p, float mx, float my, float A, float B,
                                               float C, float opacity, TileSweep &s) {
    const float disc = DET_SUB(DET_MUL(B, B), DET_MUL(A, C));
    const float t = det_fmin(kGaussianExtend * kGaussianExtend,
                             DET_MUL(2.0f, det_logf(DET_DIV(opacity, kAlphaThreshold))));
    const float ntd = DET_DIV(-t, disc);
    const float x_ext = DET_SQRT(DET_MUL(ntd, C));
    const float y_ext = DET_SQRT(DET_MUL(ntd, A));
    float bmin_x = DET_SUB(mx, x_ext), bmin_y = DET_SUB(my, y_ext);
    float bmax_x = DET_ADD(mx, x_ext), bmax_y = DET_ADD(my, y_ext);
    const float bxc = DET_DIV(DET_MUL(B, x_ext), C);
    const float bya = DET_DIV(DET_MUL(B, y_ext), A);
    float amin_y = DET_ADD(mx, bya), amax_y = DET_SUB(mx, bya);
    float amin_x = DET_ADD(my, bxc), amax_x = DET_SUB(my, bxc);
    const int tw = (int)p.tile_width, th = (int)p.tile_height;
    int rmin_x = max(0, min(tw, det_f2i_rz(tile_div(p, bmin_x))));
    int rmin_y = max(0, min(th, det_f2i_rz(tile_div(p, bmin_y))));
    int rmax_x = max(0, min(tw, det_f2i_rz(DET_ADD(tile_div(p, bmax_x), 1.f))));
    int rmax_y = max(0, min(th, det_f2i_rz(DET_ADD(tile_div(p, bmax_y), 1.f))));
    const int y_span = rmax_y - rmin_y, x_span = rmax_x - rmin_x;
    if (y_span * x_span == 0) return false;
    s.is_y = y_span < x_span;
    if (s.is_y) {
        int ti;
        float tf;
        ti = rmin_x; rmin_x = rmin_y; rmin_y = ti;
        ti = rmax_x; rmax_x = rmax_y; rmax_y = ti;
        tf = bmin_x; bmin_x = bmin_y; bmin_y = tf;
        tf = bmax_x; bmax_x = bmax_y; bmax_y = tf;
        tf = amin_x; amin_x = amin_y; amin_y = tf;
        tf = amax_x; amax_x = amax_y; amax_y = tf;
    }
    s.A = A;
    s.B = B;
    s.C = C;
    s.disc = disc;
    s.t = t;
    s.mx = mx;
    s.my = my;
    s.bmin_x = bmin_x;
    s.bmax_x = bmax_x;
    s.bmin_y = bmin_y;
    s.bmax_y = bmax_y;
    s.amin_y = amin_y;
    s.amax_y = amax_y;
    s.rmin_x = rmin_x;
    s.rmax_x = rmax_x;
    s.rmin_y = rmin_y;
    s.rmax_y = rmax_y;
    return true;
}

__device__ __forceinline__ LinePair sweep_line(const TileSweep &s, float coord) {
    return ellipse_line(s.A, s.B, s.C, s.disc, s.t, s.mx, s.my, s.is_y, coord);
}

// Tiles [v0, v1) of column u (absolute) between the lines min_line and
// max_line with the level set's extents lo / hi on them.
__device__ __forceinline__ void sweep_rows(const IsectParams &p, const TileSweep &s, float min_line,
                                           float max_line, const LinePair &lo, const LinePair &hi, int &v0,
                                           int &v1) {
    const float emin = (min_line <= s.amin_y && s.amin_y < max_line) ? s.bmin_y : det_fmin(lo.lo, hi.lo);
    const float emax = (min_line <= s.amax_y && s.amax_y < max_line) ? s.bmax_y : det_fmax(lo.hi, hi.hi);
    v0 = max(s.rmin_y, min(s.rmax_y, det_f2i_rz(tile_div(p, emin))));
    v1 = min(s.rmax_y, max(s.rmin_y, det_f2i_rz(DET_ADD(tile_div(p, emax), 1.f))));
}

__device__ __forceinline__ int64_t sweep_tile(const IsectParams &p, const TileSweep &s, int u, int v) {
    const int tw = (int)p.tile_width;
    return s.is_y ? (int64_t)u * tw + v : (int64_t)v * tw + u;
}

// The sequential sweep: each column's lower line is the previous column's
// upper one. Returns the number of tiles; emits them when EMIT.
template <bool EMIT, class Sink>
__device__ uint32_t accutile_sweep(const IsectParams &p, const TileSweep &s, Sink *sink) {
    const float ts = (float)p.tile_size;
    uint32_t count = 0;
    LinePair cur_hi = {s.bmax_y, s.bmin_y};
    float min_line = DET_MUL((float)s.rmin_x, ts);
    LinePair cur_lo = (s.bmin_x <= min_line) ? sweep_line(s, min_line) : cur_hi;
    for (int u = s.rmin_x; u < s.rmax_x; ++u) {
        const float max_line = DET_ADD(min_line, ts);
        if (max_line <= s.bmax_x) cur_hi = sweep_line(s, max_line);
        int v0, v1;
        sweep_rows(p, s, min_line, max_line, cur_lo, cur_hi, v0, v1);
        if (v1 > v0) {
            count += (uint32_t)(v1 - v0);
            if (EMIT) {
                for (int v = v0; v < v1; ++v) sink->put(sweep_tile(p, s, u, v));
            }
        }
        cur_lo = cur_hi;
        min_line = max_line;
    }
    return count;
}

template <bool EMIT, class Sink>
__device__ uint32_t accutile(const IsectParams &p, float mx, float my, float A, float B, float C,
                             float opacity, Sink *sink) {
    TileSweep s;
    if (!accutile_setup(p, mx, my, A, B, C, opacity, s)) return 0;
    return accutile_sweep<EMIT, Sink>(p, s, sink);
}

// Column k (0-based) of the sweep on its own, with the values the sequential
// sweep carries recomputed: its lines are (rmin_x + k) ts and (rmin_x + k + 1)
// ts (the sequential sweep's repeated additions of ts are exact: integers below
// 2^24), and the upper extent a column carries is that of the last line W + 1 <=
// k + 1 with line(W + 1) <= bmax_x (the lines increase), or the box's corner
// values {bmax_y, bmin_y} when there is none.
__device__ __forceinline__ void accutile_column(const IsectParams &p, const TileSweep &s, int k, int &v0,
                                                int &v1) {
    const float ts = (float)p.tile_size;
    const int ncol = s.rmax_x - s.rmin_x;
    int W = ncol - 1; // largest w with line(w + 1) <= bmax_x, or -1
    while (W >= 0 && !(DET_MUL((float)(s.rmin_x + W + 1), ts) <= s.bmax_x)) --W;
    const LinePair corner = {s.bmax_y, s.bmin_y};
    auto upper = [&](int j) -> LinePair { // the extent carried after column j
        if (W < 0) return corner;
        return sweep_line(s, DET_MUL((float)(s.rmin_x + min(j, W) + 1), ts));
    };
    const float min_line = DET_MUL((float)(s.rmin_x + k), ts);
    const float max_line = DET_MUL((float)(s.rmin_x + k + 1), ts);
    LinePair lo;
    if (k == 0) lo = (s.bmin_x <= min_line) ? sweep_line(s, min_line) : corner;
    else lo = upper(k - 1);
    sweep_rows(p, s, min_line, max_line, lo, upper(k), v0, v1);
}

// Sweep of a splat by the whole warp (all 32 lanes call with the same s and
// their own sink for that splat): each lane takes columns lane, lane + 32, ...;
// a warp scan over the columns' tile counts then spreads the tiles evenly over
// the lanes. Returns the splat's tile count (in every lane).
template <bool EMIT, class Sink>
__device__ uint32_t accutile_warp(const IsectParams &p, const TileSweep &s, Sink *sink) {
    const int lane = (int)(threadIdx.x & 31u);
    const int ncol = s.rmax_x - s.rmin_x;
    uint32_t total = 0;
    for (int cbase = 0; cbase < ncol; cbase += 32) {
        const int k = cbase + lane;
        int v0 = 0, v1 = 0;
        if (k < ncol) accutile_column(p, s, k, v0, v1);
        const int cnt = v1 > v0 ? v1 - v0 : 0;
        int incl = cnt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += y;
        }
        const int excl = incl - cnt;
        const int tot = __shfl_sync(0xffffffffu, incl, 31);
        total += (uint32_t)tot;
        if (EMIT) {
            for (int tb = 0; tb < tot; tb += 32) {
                const int t = tb + lane;
                // column j of tile t: the number of lanes whose inclusive count is <= t
                int j = 0;
#pragma unroll
                for (int step = 16; step > 0; step >>= 1) {
                    const int val = __shfl_sync(0xffffffffu, incl, j + step - 1);
                    if (val <= t) j += step;
                }
                const int ej = __shfl_sync(0xffffffffu, excl, j & 31);
                const int vj = __shfl_sync(0xffffffffu, v0, j & 31);
                if (t < tot) sink->put(sweep_tile(p, s, s.rmin_x + cbase + j, vj + (t - ej)));
            }
        }
    }
    return total;
}

template <bool EMIT, class Sink>
__device__ uint32_t aabb_tiles(const IsectParams &p, float mx, float my, int32_t rx, int32_t ry,
                               Sink *sink) {
    const float trx = tile_div(p, (float)rx), try_ = tile_div(p, (float)ry);
    const float tx = tile_div(p, mx), ty = tile_div(p, my);
    const int tw = (int)p.tile_width, th = (int)p.tile_height;
    const int x0 = min(max(0, det_f2i_rz(floorf(DET_SUB(tx, trx)))), tw);
    const int y0 = min(max(0, det_f2i_rz(floorf(DET_SUB(ty, try_)))), th);
    const int x1 = min(max(0, det_f2i_rz(ceilf(DET_ADD(tx, trx)))), tw);
    const int y1 = min(max(0, det_f2i_rz(ceilf(DET_ADD(ty, try_)))), th);
    if (EMIT) {
        for (int y = y0; y < y1; ++y)
            for (int x = x0; x < x1; ++x) sink->put((int64_t)y * tw + x);
    }
    return (uint32_t)((y1 - y0) * (x1 - x0));
}

template <bool EMIT, class Sink = EmitSink>
__device__ __forceinline__ uint32_t splat_tiles(const IsectParams &p, uint32_t idx, Sink *sink) {
    const int32_t rx = p.radii[(size_t)idx * 2], ry = p.radii[(size_t)idx * 2 + 1];
    if (rx <= 0 || ry <= 0) return 0;
    const float mx = p.means2d[(size_t)idx * 2], my = p.means2d[(size_t)idx * 2 + 1];
    if (p.conics != nullptr && p.opacities != nullptr) {
        return accutile<EMIT, Sink>(p, mx, my, p.conics[(size_t)idx * 3], p.conics[(size_t)idx * 3 + 1],
                                    p.conics[(size_t)idx * 3 + 2], p.opacities[idx], sink);
    }
    return aabb_tiles<EMIT, Sink>(p, mx, my, rx, ry, sink);
}

__global__ void __launch_bounds__(256) isect_count_kernel(IsectParams p, int32_t *tiles_per_gauss) {
    const uint32_t idx = blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t n = p.packed ? p.nnz : p.I * p.N;
    if (idx >= n) return;
    tiles_per_gauss[idx] = (int32_t)splat_tiles<false, EmitSink>(p, idx, nullptr);
}

__global__ void __launch_bounds__(256) isect_emit_kernel(IsectParams p, const int64_t *cum_tiles,
                                                         int64_t *keys, int32_t *ids) {
    const uint32_t idx = blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t n = p.packed ? p.nnz : p.I * p.N;
    if (idx >= n) return;
    const int64_t start = idx == 0 ? 0 : cum_tiles[idx - 1];
    const int64_t limit = cum_tiles[idx];
    if (limit == start) return;
    const int64_t iid = p.packed ? p.image_ids[idx] : (int64_t)(idx / p.N);
    EmitSink sink;
    sink.keys = keys;
    sink.ids = ids;
    sink.cursor = start;
    sink.limit = limit;
    sink.key_hi_base = iid << (32 + p.tile_n_bits);
    sink.depth_bits = (int64_t)det_f2u(p.depths[idx]);
    sink.flat_id = (int32_t)idx;
    splat_tiles<true>(p, idx, &sink);
}

// offsets[i] = index of the first key whose (image, tile) id is >= i, for
// i in [0, I * n_tiles): the same array IntersectTile.cu:391-439 produces. Thread
// k handles the run boundary before key k and, for k > last id, the tail entry k.
__global__ void __launch_bounds__(256) isect_offsets_kernel(const int64_t *__restrict__ keys,
                                                            uint32_t n_isects, uint32_t n_tiles,
                                                            uint32_t tile_n_bits, uint32_t total,
                                                            int32_t *__restrict__ offsets) {
    const uint32_t k = blockIdx.x * blockDim.x + threadIdx.x;
    const uint64_t tmask = (1ull << tile_n_bits) - 1ull;
    auto flat_id = [&](int64_t key) -> int64_t {
        const int64_t hi = key >> 32;
        return (hi >> tile_n_bits) * (int64_t)n_tiles + (int64_t)((uint64_t)hi & tmask);
    };
    if (k < n_isects) {
        const int64_t cur = flat_id(keys[k]);
        const int64_t prev = k == 0 ? -1 : flat_id(keys[k - 1]);
        for (int64_t i = prev + 1; i <= cur && i < (int64_t)total; ++i) offsets[i] = (int32_t)k;
    }
    if (k < total) {
        const int64_t last = flat_id(keys[n_isects - 1]);
        if ((int64_t)k > last) offsets[k] = (int32_t)n_isects;
    }
}

__global__ void fill_i32_kernel(int32_t *p, uint32_t n, int32_t v) {
    const uint32_t k = blockIdx.x * blockDim.x + threadIdx.x;
    if (k < n) p[k] = v;
}

// ---------------------------------------------------------------------------
// Tile-bucket pipeline for the sorted intersection list.
//
// The reference sorts all keys with one global stable radix sort
// (Intersect.cpp:140-170, cub::DeviceRadixSort::SortPairs). Inside one
// (image, tile) bucket the keys differ only in their depth bits, and the emit
// order of a bucket's entries is by increasing splat index (every splat emits a
// given tile at most once, and splats emit in index order). A stable sort by
// depth inside a bucket is therefore the same as a sort by the unique pair
// (depth bits, splat index). The pipeline:
//   1. count: every splat's tile count, and per bucket the entries of each
//      "shard" of splats (below);
//   2. offsets: exclusive scan over (bucket, shard) in bucket-major order,
//      giving each shard's first slot and each bucket's start -- exactly the
//      offsets array of isect_offset_encode -- and the largest bucket;
//   3. emit: every entry (depth bits, splat index) goes to the next free slot
//      of its (bucket, shard), in arbitrary order inside the shard;
//   4. sort: each bucket is sorted on chip by (depth bits, splat index), and
//      the final 64-bit keys and flatten ids are written.
// The output is bit-identical to the global stable sort of the emitted keys.
//
// Shards. With few buckets (the usual case: one image has a few thousand
// tiles) the splats are cut into G contiguous ranges, one per CTA, and each CTA
// counts and places its entries through a histogram / cursor array of all
// buckets in its shared memory: no global atomics. With more buckets than fit
// in shared memory, 16 shards per bucket live in global memory and splat idx
// uses shard idx % 16, so that the hottest buckets do not serialise their
// atomics on one address.
// ---------------------------------------------------------------------------
#ifndef GSB_SHARDS
#define GSB_SHARDS GSB_ISECT_BUCKET_SHARDS
#endif
constexpr int kBucketShards = GSB_SHARDS; // global-memory path
static_assert((kBucketShards & (kBucketShards - 1)) == 0, "shards: power of two");
#ifndef GSB_CTA_BUCKET_MAX
#define GSB_CTA_BUCKET_MAX 24576
#endif
constexpr uint32_t kCtaBucketMax = GSB_CTA_BUCKET_MAX; // buckets of the shared-memory path (96 KiB)
#ifndef GSB_CTA_THREADS
#define GSB_CTA_THREADS 1024
#define GSB_CTAS_PER_SM 1
#endif
#ifndef GSB_CTA_MINB
#define GSB_CTA_MINB 1
#endif
constexpr int kCtaThreads = GSB_CTA_THREADS;

struct BucketPlan {
    bool cta;       // shared-memory histograms, one CTA per contiguous splat range
    uint32_t shards; // counters per bucket: G CTAs, or kBucketShards
};

static BucketPlan bucket_plan(uint64_t n_buckets, int num_sms) {
    BucketPlan pl;
    pl.cta = n_buckets > 0 && n_buckets <= kCtaBucketMax;
    if (!pl.cta) {
        pl.shards = kBucketShards;
        return pl;
    }
    // one 1024-thread CTA per SM, fewer when the (bucket x CTA) counter matrix would pass
    // ~4M entries
    uint64_t g = (uint64_t)GSB_CTAS_PER_SM * (uint64_t)(num_sms > 0 ? num_sms : 148);
    const uint64_t cap = (4ull << 20) / n_buckets;
    if (g > cap) g = cap < 32 ? 32 : cap;
    pl.shards = (uint32_t)g;
    return pl;
}

static int device_sms() {
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 148;
    return sms;
}

struct CountSink {
    int32_t *counts; // [I * n_tiles * kBucketShards]
    int64_t base;    // image * n_tiles
    int32_t shard;
    __device__ __forceinline__ void put(int64_t tile_id) {
        atomicAdd(counts + (base + tile_id) * kBucketShards + shard, 1);
    }
    __device__ __forceinline__ void flush() {}
};

struct SmemCountSink {
    int32_t *hist; // shared memory, one counter per bucket
    int64_t base;
    __device__ __forceinline__ void put(int64_t tile_id) { atomicAdd(hist + base + tile_id, 1); }
    __device__ __forceinline__ void flush() {}
};

// Places one entry (depth bits << 32 | splat index) at the slot returned by an
// atomic increment of its cursor (global or shared memory). Tiles are taken in
// batches of K: the batch's increments are issued back to back, so the round
// trips of global atomics overlap, and the 8-byte stores follow. The bound
// keeps the slot inside the array; flush() places a partial batch.
#ifndef GSB_EMIT_BATCH
#define GSB_EMIT_BATCH 4 // global cursors (shared-memory cursors take one tile at a time)
#endif

template <int K> struct BucketSink {
    uint64_t *out;
    int32_t *cursor;
    int64_t base;   // first cursor of the splat's image
    int32_t stride; // cursors per bucket in `cursor`
    int32_t shard;
    uint32_t limit; // n_isects
    uint64_t entry;
    uint32_t pend[K];
    int npend = 0;
    __device__ __forceinline__ void put(int64_t tile_id) {
#pragma unroll
        for (int k = 0; k < K; ++k)
            if (k == npend) pend[k] = (uint32_t)tile_id;
        if (++npend == K) flush();
    }
    __device__ __forceinline__ void flush() {
        uint32_t pos[K];
#pragma unroll
        for (int k = 0; k < K; ++k)
            if (k < npend) pos[k] = (uint32_t)atomicAdd(cursor + (base + pend[k]) * stride + shard, 1);
#pragma unroll
        for (int k = 0; k < K; ++k)
            if (k < npend && pos[k] < limit) out[pos[k]] = entry;
        npend = 0;
    }
};

__device__ __forceinline__ int64_t splat_image(const IsectParams &p, uint32_t idx) {
    return p.packed ? p.image_ids[idx] : (int64_t)(idx / p.N);
}

__device__ __forceinline__ uint32_t n_splats(const IsectParams &p) {
    if (!p.packed) return p.I * p.N;
    if (p.nnz_device == nullptr) return p.nnz;
    const int64_t n = *p.nnz_device;
    return n < 0 ? 0u : (n < (int64_t)p.nnz ? (uint32_t)n : p.nnz);
}

// Shared-memory (CTA) path: splats whose tile box holds more than this many
// tiles are swept by their whole warp (accutile_warp) after the lanes' own
// small splats, since one thread per splat leaves the warp waiting on its
// largest splat (config 1: count 52 -> 39 us, emit 81 -> 68 us at 96; 8 and 32
// were slower). The global-shard kernels keep one thread per splat: there the
// warp sweep's registers (48 -> 80 for the batched-cursor emit) cost more
// than it saved (config 4: emit 27.6 -> 32.7 ms).
#ifndef GSB_WARP_SWEEP_TILES
#define GSB_WARP_SWEEP_TILES 96
#endif
constexpr uint32_t kWarpSweepTiles = GSB_WARP_SWEEP_TILES;

__device__ __forceinline__ TileSweep shfl_sweep(const TileSweep &s, int src) {
    TileSweep w;
    w.A = __shfl_sync(0xffffffffu, s.A, src);
    w.B = __shfl_sync(0xffffffffu, s.B, src);
    w.C = __shfl_sync(0xffffffffu, s.C, src);
    w.disc = __shfl_sync(0xffffffffu, s.disc, src);
    w.t = __shfl_sync(0xffffffffu, s.t, src);
    w.mx = __shfl_sync(0xffffffffu, s.mx, src);
    w.my = __shfl_sync(0xffffffffu, s.my, src);
    w.bmin_x = __shfl_sync(0xffffffffu, s.bmin_x, src);
    w.bmax_x = __shfl_sync(0xffffffffu, s.bmax_x, src);
    w.bmin_y = __shfl_sync(0xffffffffu, s.bmin_y, src);
    w.bmax_y = __shfl_sync(0xffffffffu, s.bmax_y, src);
    w.amin_y = __shfl_sync(0xffffffffu, s.amin_y, src);
    w.amax_y = __shfl_sync(0xffffffffu, s.amax_y, src);
    w.rmin_x = __shfl_sync(0xffffffffu, s.rmin_x, src);
    w.rmax_x = __shfl_sync(0xffffffffu, s.rmax_x, src);
    w.rmin_y = __shfl_sync(0xffffffffu, s.rmin_y, src);
    w.rmax_y = __shfl_sync(0xffffffffu, s.rmax_y, src);
    w.is_y = __shfl_sync(0xffffffffu, (int)s.is_y, src) != 0;
    return w;
}

// The tiles of splat idx of every lane (valid: the lane has a splat), counted
// or emitted through sink_of(splat) -> Sink; called by all 32 lanes of the
// warp. Returns the lane's splat's tile count.
template <bool EMIT, class Sink, class SinkOf>
__device__ __forceinline__ uint32_t splat_tiles_warp(const IsectParams &p, uint32_t idx, bool valid,
                                                     SinkOf sink_of) {
    uint32_t count = 0;
    bool big = false;
    TileSweep s{}; // lanes without a swept splat shuffle defined values
    if (valid) {
        const int32_t rx = p.radii[(size_t)idx * 2], ry = p.radii[(size_t)idx * 2 + 1];
        if (rx > 0 && ry > 0) {
            const float mx = p.means2d[(size_t)idx * 2], my = p.means2d[(size_t)idx * 2 + 1];
            if (p.conics != nullptr && p.opacities != nullptr) {
                if (accutile_setup(p, mx, my, p.conics[(size_t)idx * 3], p.conics[(size_t)idx * 3 + 1],
                                   p.conics[(size_t)idx * 3 + 2], p.opacities[idx], s)) {
                    big = (uint32_t)(s.rmax_x - s.rmin_x) * (uint32_t)(s.rmax_y - s.rmin_y) > kWarpSweepTiles;
                    if (!big) {
                        Sink k = sink_of(idx);
                        count = accutile_sweep<EMIT, Sink>(p, s, &k);
                        k.flush();
                    }
                }
            } else {
                Sink k = sink_of(idx);
                count = aabb_tiles<EMIT, Sink>(p, mx, my, rx, ry, &k);
                k.flush();
            }
        }
    }
    uint32_t todo = __ballot_sync(0xffffffffu, big);
    while (todo) {
        const int src = __ffs(todo) - 1;
        todo &= todo - 1;
        const TileSweep w = shfl_sweep(s, src);
        Sink k = sink_of(__shfl_sync(0xffffffffu, idx, src));
        const uint32_t c = accutile_warp<EMIT, Sink>(p, w, &k);
        k.flush();
        if ((int)(threadIdx.x & 31u) == src) count = c;
    }
    return count;
}

// global-memory shards
__global__ void __launch_bounds__(256) isect_count_tiles_kernel(IsectParams p, int32_t *tiles_per_gauss,
                                                                int32_t *shard_counts) {
    const uint32_t idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= n_splats(p)) return;
    CountSink sink;
    sink.counts = shard_counts;
    sink.base = splat_image(p, idx) * (int64_t)p.tile_width * p.tile_height;
    sink.shard = (int32_t)(idx & (kBucketShards - 1));
    tiles_per_gauss[idx] = (int32_t)splat_tiles<true, CountSink>(p, idx, &sink);
}

// shared-memory shards: CTA c counts splats [c chunk, (c + 1) chunk) and writes
// its histogram to column c of the bucket-major (bucket x G) matrix
__global__ void __launch_bounds__(kCtaThreads, GSB_CTA_MINB) isect_count_cta_kernel(IsectParams p, uint32_t n_buckets,
                                                                      int32_t *tiles_per_gauss,
                                                                      int32_t *matrix) {
    extern __shared__ int32_t hist[];
    for (uint32_t b = threadIdx.x; b < n_buckets; b += blockDim.x) hist[b] = 0;
    __syncthreads();
    const uint32_t n = n_splats(p), G = gridDim.x;
    const uint32_t chunk = (n + G - 1) / G;
    const uint32_t lo = blockIdx.x * chunk, hi = min(n, lo + chunk);
    const int64_t n_tiles = (int64_t)p.tile_width * p.tile_height;
    // the same number of rounds for every thread: the warp sweep needs whole warps
    for (uint32_t base = lo; base < hi; base += blockDim.x) {
        const uint32_t idx = base + threadIdx.x;
        const bool valid = idx < hi;
        const uint32_t c = splat_tiles_warp<true, SmemCountSink>(p, idx, valid, [&](uint32_t i) {
            SmemCountSink sink;
            sink.hist = hist;
            sink.base = splat_image(p, i) * n_tiles;
            return sink;
        });
        if (valid) tiles_per_gauss[idx] = (int32_t)c;
    }
    __syncthreads();
    for (uint32_t b = threadIdx.x; b < n_buckets; b += blockDim.x) matrix[(size_t)b * G + blockIdx.x] = hist[b];
}

// cursor[k] = first slot of (bucket, shard) k = exclusive scan of the counts
__global__ void __launch_bounds__(256) shard_bases_kernel(const int64_t *__restrict__ incl, uint32_t n,
                                                          int32_t *__restrict__ cursor) {
    const uint32_t k = blockIdx.x * blockDim.x + threadIdx.x;
    if (k < n) cursor[k] = k == 0 ? 0 : (int32_t)incl[k - 1];
}

// Bucket b occupies [incl[b S - 1], incl[b S + S - 1]).
// totals[0] = number of entries (-1 when it does not fit int32, like every
// offset here), totals[1] = largest bucket, totals[2] = *nnz_device if given,
// totals[3] / totals[4] = buckets of the sort classes (1024, 4096] / (4096, inf).
__global__ void __launch_bounds__(256) bucket_starts_kernel(const int64_t *__restrict__ incl, uint32_t n_buckets,
                                                            uint32_t shards, int32_t *__restrict__ starts,
                                                            int32_t *__restrict__ sizes, const int64_t *nnz_device,
                                                            int32_t *totals, int32_t *__restrict__ class_list) {
    const uint32_t b = blockIdx.x * blockDim.x + threadIdx.x;
    int32_t c = 0;
    if (b < n_buckets) {
        const size_t s0 = (size_t)b * shards;
        const int64_t first = s0 == 0 ? 0 : incl[s0 - 1];
        starts[b] = (int32_t)first;
        c = (int32_t)(incl[s0 + shards - 1] - first);
        sizes[b] = c;
    }
    if (b == n_buckets - 1) {
        const int64_t total = incl[(size_t)n_buckets * shards - 1];
        totals[0] = total > 0x7fffffffll ? -1 : (int32_t)total;
        if (nnz_device != nullptr) {
            const int64_t v = *nnz_device;
            totals[2] = v > 0x7fffffffll ? -1 : (int32_t)v;
        }
    }
    // the radix-sorted size classes: counts, and the bucket ids listed
    // (1024, 4096] from the front of class_list, > 4096 from its back
    const uint32_t mid = __ballot_sync(0xffffffffu, c > 1024 && c <= 4096);
    const uint32_t large = __ballot_sync(0xffffffffu, c > 4096);
    const int lane = threadIdx.x & 31;
    int mbase = 0, lbase = 0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) c = max(c, __shfl_xor_sync(0xffffffffu, c, o));
    if (lane == 0) {
        if (c > 0) atomicMax(totals + 1, c);
        if (mid) mbase = atomicAdd(totals + 3, __popc(mid));
        if (large) lbase = atomicAdd(totals + 4, __popc(large));
    }
    mbase = __shfl_sync(0xffffffffu, mbase, 0);
    lbase = __shfl_sync(0xffffffffu, lbase, 0);
    const uint32_t below = (1u << lane) - 1u;
    if ((mid >> lane) & 1u) class_list[mbase + __popc(mid & below)] = (int32_t)b;
    if ((large >> lane) & 1u) class_list[n_buckets - 1u - (uint32_t)(lbase + __popc(large & below))] = (int32_t)b;
}

__global__ void __launch_bounds__(256) isect_bucket_emit_kernel(IsectParams p, uint32_t n_isects,
                                                                int32_t *cursor, uint64_t *out) {
    const uint32_t idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= n_splats(p)) return;
    BucketSink<GSB_EMIT_BATCH> sink;
    sink.out = out;
    sink.cursor = cursor;
    sink.base = splat_image(p, idx) * (int64_t)p.tile_width * p.tile_height;
    sink.stride = kBucketShards;
    sink.shard = (int32_t)(idx & (kBucketShards - 1));
    sink.limit = n_isects;
    sink.entry = ((uint64_t)det_f2u(p.depths[idx]) << 32) | idx;
    splat_tiles<true, BucketSink<GSB_EMIT_BATCH>>(p, idx, &sink);
    sink.flush();
}

__global__ void __launch_bounds__(kCtaThreads, GSB_CTA_MINB) isect_emit_cta_kernel(IsectParams p, uint32_t n_buckets,
                                                                     uint32_t n_isects, const int32_t *cursor,
                                                                     uint64_t *out) {
    extern __shared__ int32_t cur[];
    const uint32_t n = n_splats(p), G = gridDim.x;
    for (uint32_t b = threadIdx.x; b < n_buckets; b += blockDim.x) cur[b] = cursor[(size_t)b * G + blockIdx.x];
    __syncthreads();
    const uint32_t chunk = (n + G - 1) / G;
    const uint32_t lo = blockIdx.x * chunk, hi = min(n, lo + chunk);
    const int64_t n_tiles = (int64_t)p.tile_width * p.tile_height;
    for (uint32_t base = lo; base < hi; base += blockDim.x) {
        const uint32_t idx = base + threadIdx.x;
        splat_tiles_warp<true, BucketSink<1>>(p, idx, idx < hi, [&](uint32_t i) {
            BucketSink<1> sink;
            sink.out = out;
            sink.cursor = cur;
            sink.base = splat_image(p, i) * n_tiles;
            sink.stride = 1;
            sink.shard = 0;
            sink.limit = n_isects;
            sink.entry = ((uint64_t)det_f2u(p.depths[i]) << 32) | i;
            return sink;
        });
    }
}

constexpr int kBucketSortMax = 16384; // largest bucket sorted on chip (1024 threads x 16 entries)
#ifndef GSB_SPLIT_MIN
#define GSB_SPLIT_MIN 16384
#endif
// buckets above kSplitMin entries are split into sub-buckets (kSplitMin >= 4096:
// the split walks the class list of buckets above 4096 entries)
constexpr int kSplitMin = GSB_SPLIT_MIN;
static_assert(kSplitMin >= 4096 && kSplitMin <= kBucketSortMax, "split threshold");
// Buckets above kBucketSortMax entries are first split into sub-buckets by
// the leading bits of their entries (depth bits << 32 | splat index: the order
// of the final sort), written in sub-bucket order to a second array; every
// sub-bucket then goes through the on-chip sort below like a bucket of its own,
// at its final position. The list of sub-buckets lives on the device.
struct SubBuckets {
    const int *count;    // number of sub-buckets (device); null: not a sub-bucket pass
    const int32_t *start, *size, *bucket; // first entry, entries, (image, tile) bucket
    int cap;             // records the arrays hold (a larger count has overflowed)
};

constexpr int kSplitThreads = 1024;
constexpr int kSplitBits = 12; // at most 4096 sub-buckets per split bucket
constexpr int kSplitTargetBits = 8; // ~256 entries per sub-bucket on average

// One CTA per bucket of more than kBucketSortMax entries (persistent over the
// class list of buckets above 4096 entries, skipping the others): the smallest
// and largest entry, a histogram of the top kSplitBits bits of (entry - smallest),
// its exclusive scan, the scatter of the entries into `out` at the bucket's
// positions in sub-bucket order, and one sub-bucket record per non-empty bin.
// A sub-bucket above kBucketSortMax entries (more than that many entries with
// the same leading bits: equal depths) sets *overflow.
__global__ void __launch_bounds__(kSplitThreads)
    bucket_split_kernel(const int32_t *__restrict__ starts, const int32_t *__restrict__ sizes,
                        const int32_t *__restrict__ list, int count, uint32_t n_buckets,
                        const uint64_t *__restrict__ entries, uint64_t *__restrict__ out,
                        int *sub_count, int32_t *__restrict__ sub_start, int32_t *__restrict__ sub_size,
                        int32_t *__restrict__ sub_bucket, int sub_cap, int *overflow) {
    constexpr int NB = 1 << kSplitBits;
    constexpr int PER = NB / kSplitThreads;
    __shared__ uint32_t hist[NB];
    __shared__ uint32_t cur[NB];
    __shared__ unsigned long long red[2][32];
    __shared__ uint32_t wsum[32];
    __shared__ int sbase;
    const int t = threadIdx.x, lane = t & 31, w = t >> 5;
    for (int c = blockIdx.x; c < count; c += gridDim.x) {
        const uint32_t b = (uint32_t)list[(int)n_buckets - 1 - c];
        const int n = sizes[b];
        if (n <= kSplitMin) continue;
        const int start = starts[b];
        unsigned long long lo = ~0ull, hi = 0ull;
        for (int i = t; i < n; i += kSplitThreads) {
            const unsigned long long e = entries[start + i];
            lo = min(lo, e);
            hi = max(hi, e);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, o));
            hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, o));
        }
        if (lane == 0) {
            red[0][w] = lo;
            red[1][w] = hi;
        }
        for (int k = t; k < NB; k += kSplitThreads) hist[k] = 0;
        __syncthreads();
        lo = red[0][lane];
        hi = red[1][lane];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, o));
            hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, o));
        }
        const unsigned long long range = hi - lo;
        const int bits = range ? 64 - __clzll((long long)range) : 0;
        // about kSplitTarget entries per sub-bucket on average (fewer, larger
        // sub-buckets keep the per-sub-bucket cost of the sorts small)
        const int nbits = 32 - __clz((unsigned)(n - 1));
        const int sbits = min(kSplitBits, max(1, nbits - kSplitTargetBits));
        const int shift = bits > sbits ? bits - sbits : 0;
        for (int i = t; i < n; i += kSplitThreads)
            atomicAdd(&hist[(uint32_t)((entries[start + i] - lo) >> shift)], 1u);
        __syncthreads();
        // exclusive scan of the histogram: PER consecutive bins per thread
        uint32_t v[PER], tot = 0, nonempty = 0;
#pragma unroll
        for (int k = 0; k < PER; ++k) {
            v[k] = hist[t * PER + k];
            tot += v[k];
            nonempty += v[k] > 0;
        }
        uint32_t incl = tot;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += y;
        }
        if (lane == 31) wsum[w] = incl;
        __syncthreads();
        if (w == 0) {
            uint32_t x = wsum[lane], xi = x;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t y = __shfl_up_sync(0xffffffffu, xi, o);
                if (lane >= o) xi += y;
            }
            wsum[lane] = xi - x;
        }
        // the sub-bucket records: one block-wide count of the non-empty bins
        uint32_t ne_incl = nonempty;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xffffffffu, ne_incl, o);
            if (lane >= o) ne_incl += y;
        }
        __syncthreads();
        uint32_t base = wsum[w] + incl - tot;
        __syncthreads();
        if (lane == 31) wsum[w] = ne_incl;
        __syncthreads();
        if (w == 0) {
            uint32_t x = wsum[lane], xi = x;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t y = __shfl_up_sync(0xffffffffu, xi, o);
                if (lane >= o) xi += y;
            }
            wsum[lane] = xi - x;
            if (lane == 31) sbase = atomicAdd(sub_count, (int)xi);
        }
        __syncthreads();
        uint32_t rec = (uint32_t)sbase + wsum[w] + ne_incl - nonempty;
#pragma unroll
        for (int k = 0; k < PER; ++k) {
            cur[t * PER + k] = base;
            if (v[k] > 0) {
                if ((int)rec < sub_cap) {
                    sub_start[rec] = start + (int)base;
                    sub_size[rec] = (int)v[k];
                    sub_bucket[rec] = (int32_t)b;
                } else {
                    *overflow = 1;
                }
                if (v[k] > (uint32_t)kBucketSortMax) *overflow = 1;
                ++rec;
            }
            base += v[k];
        }
        __syncthreads();
        for (int i = t; i < n; i += kSplitThreads) {
            const unsigned long long e = entries[start + i];
            const uint32_t pos = atomicAdd(&cur[(uint32_t)((e - lo) >> shift)], 1u);
            out[start + pos] = e;
        }
        __syncthreads(); // hist / cur are reused by the next bucket
    }
}

// The on-chip sort of one bucket (or sub-bucket) per CTA: stable LSD radix sort
// in shared memory, in three shapes by bucket size (256 threads x 4 entries up
// to 1024, 256 x 16 up to 4096, 1024 x 16 up to kBucketSortMax).
// The keys are the depth bits minus the bucket's smallest, so only the bits
// of the bucket's depth range are sorted, in as few passes of at most DBITS
// bits as cover them (three for the usual 25-bit range at DBITS = 9): O(n) per
// pass where a bitonic network is O(n log^2 n). Warp w owns the contiguous
// entries [32 R w, 32 R (w + 1)) (R = rounds of this bucket), entry
// 32 R w + 32 r + lane in round r of that lane, key and splat index in
// registers. A pass ranks each warp's entries in index order with
// warp-private digit counters (match_any groups the lanes of one digit), one
// scan over the counters in digit-major order turns them into run bases, and
// the entries are scattered to base + rank in shared memory and read back.
//
// The stable sort by depth leaves equal depths in emit order, which is not the
// splat-index order of the reference's stable global sort: each run of equal
// depths is then sorted by splat index by the thread holding its first entry
// (runs of float depths are a few entries long). A bucket with a run longer
// than kTieRun re-sorts its (depth, index) pairs with a bitonic network in
// place.
constexpr int kTieRun = 32;
#ifndef GSB_BIN_COST
#define GSB_BIN_COST 32 // most comparisons per entry of the one-pass bin sort
#endif
constexpr int kBinCost = GSB_BIN_COST;
constexpr int kBinTarget = 4; // entries per sub-bin of the one-pass sort, at most
#ifndef GSB_RADIX_MATCH
#define GSB_RADIX_MATCH 1 // peers of a digit by match_any (1) or by one ballot per digit bit (0)
#endif

// sub-bins of the one-pass sort: fewer than 2 n / kBinTarget + 256 for n entries
template <int CAP> constexpr int sub_bin_max() { return 2 * CAP / kBinTarget + 256; }
// counter words: the radix digit counters [2^DBITS][warps + 1], or the one-pass
// sort's sub-bin ends and 2 x 256 coarse-bin words
template <int THREADS, int RMAX, int DBITS> constexpr int radix_counter_words() {
    return (1 << DBITS) * (THREADS / 32 + 1) > sub_bin_max<THREADS * RMAX>() + 512
               ? (1 << DBITS) * (THREADS / 32 + 1)
               : sub_bin_max<THREADS * RMAX>() + 512;
}
template <int THREADS, int RMAX, int DBITS> constexpr size_t radix_smem_bytes() {
    // keys, indices, counters, warp totals
    return (size_t)(2 * THREADS * RMAX + radix_counter_words<THREADS, RMAX, DBITS>() + 72) * sizeof(uint32_t);
}

template <int THREADS, int RMAX, int DBITS, int MINB>
__global__ void __launch_bounds__(THREADS, MINB)
    bucket_radix_kernel(const int32_t *__restrict__ starts, const int32_t *__restrict__ sizes,
                        const int32_t *__restrict__ list, int count, int from_back,
                        const uint64_t *__restrict__ entries,
                        uint32_t n_buckets, uint32_t n_tiles, uint32_t tile_bits,
                        int64_t *__restrict__ keys_out, int32_t *__restrict__ ids_out,
                        const SubBuckets sub, int lo_size, int hi_size) {
    constexpr int CAP = THREADS * RMAX;
    constexpr int NW = THREADS / 32;
    constexpr int ND = 1 << DBITS;
    constexpr int CW = NW + 1;               // words per digit row: (digit, warp) at digit * CW + warp
    constexpr int NC = radix_counter_words<THREADS, RMAX, DBITS>(); // counter words
    constexpr int kSubBinMax = sub_bin_max<CAP>();
    constexpr int PER = ND * NW / THREADS;   // counters per thread in the scan (digit-major order)
    static_assert(PER * THREADS == ND * NW && (PER % NW == 0 || NW % PER == 0), "scan split");
    static_assert(NC % 4 == 0 && (2 * CAP) % 4 == 0, "vector zeroing");
    static_assert(NW <= 32 && CAP <= 65536, "warp minima / maxima in misc[0, 64); 16-bit ranks");
    static_assert(THREADS >= 256, "one coarse bin per thread");
    extern __shared__ __align__(16) uint32_t smem[];
    uint32_t *skey = smem;            // [CAP] keys
    uint32_t *sval = smem + CAP;      // [CAP] splat indices
    uint32_t *wcnt = smem + 2 * CAP;  // [ND][CW] digit counters, then run bases (LSD passes)
    uint32_t *misc = wcnt + NC;       // [72] warp minima / maxima, warp scan totals, sub-bin count
    const int t = threadIdx.x, lane = t & 31, w = t >> 5;
    // counter k of this thread in the scan: q = PER t + k at q + q / NW
    const int cbase = PER >= NW ? t * (PER / NW) * CW : (PER * t / NW) * CW + (PER * t) % NW;
    // the buckets of this size class: list[0, count) or list[n_buckets - count,
    // n_buckets); or, with sub.count set, the sub-buckets of split buckets
    // (list == nullptr: every bucket, filtered by size)
    if (sub.count != nullptr) count = min(*sub.count, sub.cap);
    for (int c = blockIdx.x; c < count; c += gridDim.x) {
        uint32_t b, hb;
        int n, start;
        if (sub.count != nullptr) {
            b = (uint32_t)c;
            n = sub.size[c];
            start = sub.start[c];
            hb = (uint32_t)sub.bucket[c];
        } else {
            b = list == nullptr ? (uint32_t)c : (uint32_t)list[from_back ? (int)n_buckets - 1 - c : c];
            n = sizes[b];
            start = starts[b];
            hb = b;
        }
        if (n <= lo_size || n > hi_size) continue; // another size class
        const int64_t hi = ((int64_t)(hb / n_tiles) << (32 + tile_bits)) | ((int64_t)(hb % n_tiles) << 32);
        const int R = (n + THREADS - 1) / THREADS;
        const int wbase = 32 * R * w + lane; // entry of round 0
        uint32_t key[RMAX], val[RMAX], rank2[RMAX / 2]; // two 16-bit ranks per word
        uint32_t kmin = 0xffffffffu, kmax = 0;
#pragma unroll
        for (int r = 0; r < RMAX; ++r) {
            const int i = wbase + 32 * r;
            key[r] = 0;
            val[r] = 0;
            if (r < R && i < n) {
                const uint64_t en = entries[start + i];
                key[r] = (uint32_t)(en >> 32);
                val[r] = (uint32_t)en;
                kmin = min(kmin, key[r]);
                kmax = max(kmax, key[r]);
            }
        }
        kmin = __reduce_min_sync(0xffffffffu, kmin);
        kmax = __reduce_max_sync(0xffffffffu, kmax);
        if (lane == 0) {
            misc[w] = kmin;
            misc[32 + w] = kmax;
        }
        __syncthreads();
        {
            const uint32_t m0 = lane < NW ? misc[lane] : 0xffffffffu;
            const uint32_t m1 = lane < NW ? misc[32 + lane] : 0u;
            kmin = __reduce_min_sync(0xffffffffu, m0);
            kmax = __reduce_max_sync(0xffffffffu, m1);
        }
        const uint32_t range = kmax - kmin;
        const int bits = range ? 32 - __clz(range) : 0;
        const int passes = (bits + DBITS - 1) / DBITS;
        const int width = passes ? (bits + passes - 1) / passes : 0;
        const uint32_t dmask = (1u << width) - 1u;
#pragma unroll
        for (int r = 0; r < RMAX; ++r) key[r] -= kmin;
        {
            // One pass for spread-out depths: a counting sort of the entries
            // into bins of about kBinTarget entries, then the rank of each entry
            // inside its bin from comparisons of (depth, splat index) with the
            // bin's other entries, which orders ties by splat index too. The
            // bins follow the depth distribution: a histogram of the top 8 bits
            // of the key, and each of those 256 coarse bins split into 2^s
            // sub-bins by the next s bits, s chosen from its count. A bucket
            // whose bins would still cost more than kBinCost comparisons per
            // entry (many equal depths) takes the LSD passes below instead.
            const int sh1 = bits > 8 ? bits - 8 : 0;
            uint32_t *bend = wcnt;                 // [sub-bins] counts, cursors, then bin ends
            uint32_t *ccnt = wcnt + kSubBinMax;    // [256] coarse counts
            uint32_t *cinfo = ccnt + 256;          // [256] first sub-bin | split bits << 24
            __syncthreads(); // the warp minima / maxima are read
            for (int k = t; k < 256; k += THREADS) ccnt[k] = 0;
            __syncthreads();
#pragma unroll
            for (int r = 0; r < RMAX; ++r) {
                const int i = wbase + 32 * r;
                if (r < R && i < n) atomicAdd(&ccnt[key[r] >> sh1], 1u);
            }
            __syncthreads();
            // split bits per coarse bin and the exclusive scan of 2^s (threads
            // 0..255, one coarse bin each)
            {
                uint32_t nsub = 0, split = 0;
                if (t < 256) {
                    const uint32_t nc = ccnt[t];
                    split = nc > (uint32_t)kBinTarget ? 32u - __clz((nc - 1u) / (uint32_t)kBinTarget) : 0u;
                    split = min(split, (uint32_t)sh1);
                    nsub = 1u << split;
                }
                uint32_t incl = nsub;
#pragma unroll
                for (int off = 1; off < 32; off <<= 1) {
                    const uint32_t u = __shfl_up_sync(0xffffffffu, incl, off);
                    if (lane >= off) incl += u;
                }
                if (lane == 31) misc[w] = incl;
                __syncthreads();
                uint32_t m = lane < 8 ? misc[lane] : 0u;
#pragma unroll
                for (int off = 1; off < 8; off <<= 1) {
                    const uint32_t u = __shfl_up_sync(0xffffffffu, m, off);
                    if (lane >= off) m += u;
                }
                const uint32_t before_w = __shfl_sync(0xffffffffu, m, (w + 31) & 31);
                if (t < 256) cinfo[t] = ((w > 0 ? before_w : 0u) + incl - nsub) | (split << 24);
                misc[64] = __shfl_sync(0xffffffffu, m, 7); // sub-bins in all (every thread writes the same)
            }
            __syncthreads();
            const int nsb = (int)misc[64];
            for (int k = t; k < nsb; k += THREADS) bend[k] = 0;
            __syncthreads();
#pragma unroll
            for (int r = 0; r < RMAX; ++r) {
                const int i = wbase + 32 * r;
                if (r < R && i < n) {
                    const uint32_t ci = cinfo[key[r] >> sh1], sp = ci >> 24;
                    atomicAdd(&bend[(ci & 0xffffffu) + ((key[r] >> (sh1 - sp)) & ((1u << sp) - 1u))], 1u);
                }
            }
            __syncthreads();
            // exclusive scan of the sub-bin counts (thread t owns a chunk) and
            // the sum of squared counts = comparisons of the rank step
            const int chunk = (nsb + THREADS - 1) / THREADS;
            const int first = min(t * chunk, nsb), last = min(first + chunk, nsb);
            uint32_t tot = 0, sq = 0;
            for (int k = first; k < last; ++k) {
                const uint32_t v = bend[k];
                tot += v;
                sq += v * v;
            }
            uint32_t incl = tot;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const uint32_t u = __shfl_up_sync(0xffffffffu, incl, off);
                if (lane >= off) incl += u;
            }
            sq = __reduce_add_sync(0xffffffffu, sq);
            if (lane == 31) misc[w] = incl;
            if (lane == 0) misc[32 + w] = sq;
            __syncthreads();
            uint32_t m = lane < NW ? misc[lane] : 0u;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const uint32_t u = __shfl_up_sync(0xffffffffu, m, off);
                if (lane >= off) m += u;
            }
            const uint32_t before_w = __shfl_sync(0xffffffffu, m, (w + 31) & 31);
            const uint32_t sq_all = __reduce_add_sync(0xffffffffu, lane < NW ? misc[32 + lane] : 0u);
            if (sq_all <= (uint32_t)kBinCost * (uint32_t)n) {
                uint32_t run = (w > 0 ? before_w : 0u) + incl - tot;
                for (int k = first; k < last; ++k) {
                    const uint32_t v = bend[k];
                    bend[k] = run;
                    run += v;
                }
                __syncthreads();
                // scatter by sub-bin (in no particular order inside one)
#pragma unroll
                for (int r = 0; r < RMAX; ++r) {
                    const int i = wbase + 32 * r;
                    if (r < R && i < n) {
                        const uint32_t ci = cinfo[key[r] >> sh1], sp = ci >> 24;
                        const uint32_t x = (ci & 0xffffffu) + ((key[r] >> (sh1 - sp)) & ((1u << sp) - 1u));
                        const uint32_t q = atomicAdd(&bend[x], 1u);
                        skey[q] = key[r];
                        sval[q] = val[r];
                    }
                }
                __syncthreads();
                // rank inside the sub-bin (bend[x] is now the end of sub-bin x,
                // bend[x - 1] its start); the lanes of a warp hold neighbouring
                // entries, mostly of one sub-bin
                for (int q = t; q < n; q += THREADS) {
                    const uint32_t k = skey[q], v = sval[q];
                    const uint32_t ci = cinfo[k >> sh1], sp = ci >> 24;
                    const uint32_t x = (ci & 0xffffffu) + ((k >> (sh1 - sp)) & ((1u << sp) - 1u));
                    const int s0 = x > 0 ? (int)bend[x - 1] : 0, e0 = (int)bend[x];
                    int rank = 0;
                    for (int j = s0; j < e0; ++j) {
                        const uint32_t kj = skey[j];
                        rank += (kj < k || (kj == k && sval[j] < v)) ? 1 : 0;
                    }
                    keys_out[start + s0 + rank] = hi | (int64_t)(k + kmin);
                    ids_out[start + s0 + rank] = (int32_t)v;
                }
                __syncthreads(); // shared memory is reused by the next bucket
                continue;
            }
        }
        for (int shift = 0; shift < bits; shift += width) {
            __syncthreads(); // misc and the counters of the previous pass are read
            for (int k = t; k < NC / 4; k += THREADS) reinterpret_cast<uint4 *>(wcnt)[k] = make_uint4(0, 0, 0, 0);
            __syncthreads();
            // warp-local ranks in index order
#pragma unroll
            for (int r = 0; r < RMAX / 2; ++r) rank2[r] = 0;
#pragma unroll
            for (int r = 0; r < RMAX; ++r) {
                if (r < R) {
                    const bool valid = wbase + 32 * r < n;
                    const uint32_t vm = __ballot_sync(0xffffffffu, valid);
                    if (valid) {
                        const uint32_t d = (key[r] >> shift) & dmask;
#if GSB_RADIX_MATCH
                        const uint32_t peers = __match_any_sync(vm, d);
#else
                        // lanes of digit d: one ballot per digit bit
                        uint32_t peers = vm;
#pragma unroll
                        for (int bit = 0; bit < DBITS; ++bit) {
                            if (bit < width) {
                                const uint32_t bb = __ballot_sync(vm, (d >> bit) & 1u);
                                peers &= ((d >> bit) & 1u) ? bb : ~bb;
                            }
                        }
#endif
                        uint32_t *cnt = &wcnt[d * CW + w];
                        const uint32_t before = *cnt;
                        __syncwarp(vm);
                        if (lane == 31 - __clz(peers)) *cnt = before + (uint32_t)__popc(peers);
                        rank2[r >> 1] |= (before + (uint32_t)__popc(peers & ((1u << lane) - 1u))) << (16 * (r & 1));
                    }
                    __syncwarp();
                }
            }
            __syncthreads();
            {
                // run bases: exclusive scan over the counters in digit-major order
                uint32_t tot = 0;
#pragma unroll
                for (int k = 0; k < PER; ++k) tot += wcnt[cbase + (k / NW) * CW + k % NW];
                uint32_t incl = tot;
#pragma unroll
                for (int off = 1; off < 32; off <<= 1) {
                    const uint32_t u = __shfl_up_sync(0xffffffffu, incl, off);
                    if (lane >= off) incl += u;
                }
                if (lane == 31) misc[w] = incl;
                __syncthreads();
                uint32_t m = lane < NW ? misc[lane] : 0u;
#pragma unroll
                for (int off = 1; off < 32; off <<= 1) {
                    const uint32_t u = __shfl_up_sync(0xffffffffu, m, off);
                    if (lane >= off) m += u;
                }
                const uint32_t before_w = __shfl_sync(0xffffffffu, m, (w + 31) & 31);
                uint32_t run = (w > 0 ? before_w : 0u) + incl - tot;
#pragma unroll
                for (int k = 0; k < PER; ++k) {
                    uint32_t *cp = &wcnt[cbase + (k / NW) * CW + k % NW];
                    const uint32_t v = *cp;
                    *cp = run;
                    run += v;
                }
            }
            __syncthreads();
#pragma unroll
            for (int r = 0; r < RMAX; ++r) {
                const int i = wbase + 32 * r;
                if (r < R && i < n) {
                    const uint32_t q = wcnt[((key[r] >> shift) & dmask) * CW + w] +
                                       ((rank2[r >> 1] >> (16 * (r & 1))) & 0xffffu);
                    skey[q] = key[r];
                    sval[q] = val[r];
                }
            }
            __syncthreads();
#pragma unroll
            for (int r = 0; r < RMAX; ++r) {
                const int i = wbase + 32 * r;
                if (r < R && i < n) {
                    key[r] = skey[i];
                    val[r] = sval[i];
                }
            }
        }
        if (bits == 0) { // one depth: no pass ran
#pragma unroll
            for (int r = 0; r < RMAX; ++r) {
                const int i = wbase + 32 * r;
                if (r < R && i < n) {
                    skey[i] = key[r];
                    sval[i] = val[r];
                }
            }
        }
        __syncthreads();
        // runs of equal depth, sorted by splat index
        bool long_run = false;
        for (int i = t; i < n; i += THREADS) {
            const uint32_t k = skey[i];
            if ((i == 0 || skey[i - 1] != k) && i + 1 < n && skey[i + 1] == k) {
                int e = i + 1; // the run is [i, e)
                while (e < n && e - i <= kTieRun && skey[e] == k) ++e;
                if (e - i > kTieRun) {
                    long_run = true;
                } else {
                    for (int a = i + 1; a < e; ++a) {
                        const uint32_t v = sval[a];
                        int c2 = a;
                        for (; c2 > i && sval[c2 - 1] > v; --c2) sval[c2] = sval[c2 - 1];
                        sval[c2] = v;
                    }
                }
            }
        }
        if (__syncthreads_or(long_run)) {
            // bitonic sort of the (depth, index) pairs in place; padding
            // (~0, ~0) sorts last (indices are below 2^31)
            int npad = 2;
            while (npad < n) npad <<= 1;
            for (int i = n + t; i < npad; i += THREADS) {
                skey[i] = 0xffffffffu;
                sval[i] = 0xffffffffu;
            }
            __syncthreads();
            for (int k = 2; k <= npad; k <<= 1) {
                for (int j = k >> 1; j > 0; j >>= 1) {
                    const int lj = 31 - __clz(j);
                    for (int q = t; q < npad / 2; q += THREADS) {
                        const int i = ((q >> lj) << (lj + 1)) | (q & (j - 1));
                        const uint32_t xk = skey[i], yk = skey[i + j], xv = sval[i], yv = sval[i + j];
                        const bool gt = xk > yk || (xk == yk && xv > yv);
                        if (gt == ((i & k) == 0)) {
                            skey[i] = yk;
                            skey[i + j] = xk;
                            sval[i] = yv;
                            sval[i + j] = xv;
                        }
                    }
                    __syncthreads();
                }
            }
        }
        for (int i = t; i < n; i += THREADS) {
            keys_out[start + i] = hi | (int64_t)(skey[i] + kmin);
            ids_out[start + i] = (int32_t)sval[i];
        }
        __syncthreads(); // shared memory is reused by the next bucket
    }
}

// radix kernel shapes: threads, entries per thread, digit bits, CTAs per SM
#ifndef GSB_RADIX_MID_SHAPE // buckets of (1024, 4096] entries
#define GSB_RADIX_MID_T 256
#define GSB_RADIX_MID_R 16
#define GSB_RADIX_MID_D 9
#define GSB_RADIX_MID_B 3
#endif
#ifndef GSB_RADIX_LARGE_SHAPE // buckets of (4096, 16384] entries (config 4's ~6,800-entry
// buckets: 1024 x 16 sorted them in 35.5 ms per step against 39.9 ms for 512 x 32)
#define GSB_RADIX_LARGE_T 1024
#define GSB_RADIX_LARGE_R 16
#define GSB_RADIX_LARGE_D 9
#define GSB_RADIX_LARGE_B 1
#endif
#define GSB_RADIX_MID GSB_RADIX_MID_T, GSB_RADIX_MID_R, GSB_RADIX_MID_D, GSB_RADIX_MID_B
#ifndef GSB_RADIX_SMALL_B
#define GSB_RADIX_SMALL_B 6
#endif
#define GSB_RADIX_SMALL 256, 4, 9, GSB_RADIX_SMALL_B
#define GSB_RADIX_LARGE GSB_RADIX_LARGE_T, GSB_RADIX_LARGE_R, GSB_RADIX_LARGE_D, GSB_RADIX_LARGE_B

template <int THREADS, int RMAX, int DBITS, int MINB> struct RadixShape {
    static constexpr int threads = THREADS;
    static constexpr int cap = THREADS * RMAX;
    static constexpr int per_sm = MINB;
    static constexpr size_t smem = radix_smem_bytes<THREADS, RMAX, DBITS>();
};

static uint32_t bit_length(uint64_t v) {
    uint32_t b = 0;
    while (v) {
        ++b;
        v >>= 1;
    }
    return b;
}

static int make_isect_params(IsectParams &p, int packed, int I, int N, int nnz,
                             const int64_t *image_ids, const float *means2d, const int32_t *radii,
                             const float *depths, const float *conics, const float *opacities,
                             int tile_size, int tile_width, int tile_height) {
    if (tile_size <= 0 || tile_width <= 0 || tile_height <= 0)
        return set_error(kErrInvalidArgument, "tile sizes must be positive");
    if (packed && image_ids == nullptr)
        return set_error(kErrInvalidArgument,
                         "When packed is set, image_ids and gaussian_ids must be provided.");
    const uint32_t n_tiles = (uint32_t)tile_width * (uint32_t)tile_height;
    const uint32_t tile_bits = bit_length(n_tiles);
    const uint32_t image_bits = bit_length((uint64_t)(I > 0 ? I : 1));
    if (tile_bits + image_bits > 32)
        return set_error(kErrInvalidArgument, "image bits (%u) + tile bits (%u) exceed 32", image_bits,
                         tile_bits);
    p.packed = packed != 0;
    p.I = I;
    p.N = N;
    p.nnz = nnz;
    p.image_ids = image_ids;
    p.means2d = means2d;
    p.radii = radii;
    p.depths = depths;
    p.conics = conics;
    p.opacities = opacities;
    p.tile_size = tile_size;
    p.tile_width = tile_width;
    p.tile_height = tile_height;
    p.tile_n_bits = tile_bits;
    p.inv_tile_pow2 = (tile_size & (tile_size - 1)) == 0 ? 1.f / (float)tile_size : 0.f;
    p.nnz_device = nullptr;
    return kOk;
}

} // namespace gsb

using namespace gsb;

extern "C" int gsb_isect_key_bits(int I, int tile_width, int tile_height) {
    return (int)(32 + bit_length((uint64_t)tile_width * tile_height) + bit_length(I > 0 ? I : 1));
}

extern "C" int gsb_isect_count(int packed, int I, int N, int nnz, const int64_t *image_ids,
                               const float *means2d, const int32_t *radii, const float *depths,
                               const float *conics, const float *opacities, int tile_size,
                               int tile_width, int tile_height, int32_t *tiles_per_gauss,
                               cudaStream_t stream) {
    IsectParams p;
    if (int e = make_isect_params(p, packed, I, N, nnz, image_ids, means2d, radii, depths, conics,
                                  opacities, tile_size, tile_width, tile_height))
        return e;
    const size_t n = packed ? (size_t)nnz : (size_t)I * N;
    if (n == 0) return kOk;
    if (n > 0x7fffffffu) return set_error(kErrInvalidArgument, "too many splats: %zu", n);
    isect_count_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(p, tiles_per_gauss);
    return check_launch("isect_count_kernel");
}

extern "C" int gsb_isect_emit(int packed, int I, int N, int nnz, const int64_t *image_ids,
                              const float *means2d, const int32_t *radii, const float *depths,
                              const float *conics, const float *opacities, int tile_size,
                              int tile_width, int tile_height, const int64_t *cum_tiles_per_gauss,
                              int64_t *isect_ids, int32_t *flatten_ids, cudaStream_t stream) {
    IsectParams p;
    if (int e = make_isect_params(p, packed, I, N, nnz, image_ids, means2d, radii, depths, conics,
                                  opacities, tile_size, tile_width, tile_height))
        return e;
    const size_t n = packed ? (size_t)nnz : (size_t)I * N;
    if (n == 0) return kOk;
    isect_emit_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(p, cum_tiles_per_gauss,
                                                                        isect_ids, flatten_ids);
    return check_launch("isect_emit_kernel");
}

extern "C" int gsb_isect_offset_encode(const int64_t *isect_ids, long long n_isects, int I,
                                       int tile_width, int tile_height, int32_t *offsets,
                                       cudaStream_t stream) {
    const uint32_t n_tiles = (uint32_t)tile_width * (uint32_t)tile_height;
    const uint64_t total = (uint64_t)I * n_tiles;
    if (total == 0) return kOk;
    if (n_isects > 0x7fffffffll) return set_error(kErrInvalidArgument, "too many intersections");
    if (n_isects <= 0) {
        fill_i32_kernel<<<(unsigned)((total + 255) / 256), 256, 0, stream>>>(offsets, (uint32_t)total, 0);
        return check_launch("fill_i32_kernel");
    }
    const uint64_t threads = total > (uint64_t)n_isects ? total : (uint64_t)n_isects;
    isect_offsets_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, stream>>>(
        isect_ids, (uint32_t)n_isects, n_tiles, bit_length(n_tiles), (uint32_t)total, offsets);
    return check_launch("isect_offsets_kernel");
}

// ---------------------------------------------------------------------------
// Tile-bucket pipeline entry points
// ---------------------------------------------------------------------------
extern "C" int gsb_isect_bucket_shards(int I, int tile_width, int tile_height) {
    if (I <= 0 || tile_width <= 0 || tile_height <= 0) return kBucketShards;
    return (int)bucket_plan((uint64_t)I * tile_width * tile_height, device_sms()).shards;
}

// One internal stream per device (non-blocking, created at first use) with a
// fork and a join event, for work that can run next to the caller's stream.
struct SideStream {
    cudaStream_t stream = nullptr;
    cudaEvent_t fork = nullptr, join = nullptr;
};
constexpr int kMaxSideDevices = 64;
static std::mutex g_side_mutex;
static SideStream g_side[kMaxSideDevices];

// Caller holds g_side_mutex (the events are shared by all calls on a device).
static int side_stream(SideStream **out) {
    int dev = 0;
    cudaError_t ce = cudaGetDevice(&dev);
    if (ce != cudaSuccess) return set_error(kErrLaunch, "cudaGetDevice: %s", cudaGetErrorString(ce));
    if (dev < 0 || dev >= kMaxSideDevices) return set_error(kErrUnsupported, "device %d out of range", dev);
    SideStream &s = g_side[dev];
    if (s.stream == nullptr) {
        if ((ce = cudaStreamCreateWithFlags(&s.stream, cudaStreamNonBlocking)) != cudaSuccess ||
            (ce = cudaEventCreateWithFlags(&s.fork, cudaEventDisableTiming)) != cudaSuccess ||
            (ce = cudaEventCreateWithFlags(&s.join, cudaEventDisableTiming)) != cudaSuccess)
            return set_error(kErrLaunch, "side stream set-up: %s", cudaGetErrorString(ce));
    }
    *out = &s;
    return kOk;
}

static int set_cta_smem(const void *kern, size_t smem) {
    if (smem <= 48 * 1024) return kOk;
    cudaError_t ce = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (ce != cudaSuccess) return set_error(kErrLaunch, "cudaFuncSetAttribute: %s", cudaGetErrorString(ce));
    return kOk;
}

extern "C" int gsb_isect_count_tiles(int packed, int I, int N, int nnz, const int64_t *image_ids,
                                     const float *means2d, const int32_t *radii, const float *depths,
                                     const float *conics, const float *opacities, int tile_size,
                                     int tile_width, int tile_height, const int64_t *nnz_device,
                                     int32_t *tiles_per_gauss, int32_t *shard_counts, cudaStream_t stream) {
    IsectParams p;
    if (int e = make_isect_params(p, packed, I, N, nnz, image_ids, means2d, radii, depths, conics,
                                  opacities, tile_size, tile_width, tile_height))
        return e;
    p.nnz_device = packed ? nnz_device : nullptr;
    const uint64_t n_buckets = (uint64_t)I * tile_width * tile_height;
    const size_t n = packed ? (size_t)nnz : (size_t)I * N;
    if (n > 0x7fffffffu) return set_error(kErrInvalidArgument, "too many splats: %zu", n);
    const BucketPlan pl = bucket_plan(n_buckets, device_sms());
    if (pl.cta) {
        // every matrix entry is written, also with no splats
        const size_t smem = n_buckets * sizeof(int32_t);
        if (int e = set_cta_smem((const void *)isect_count_cta_kernel, smem)) return e;
        isect_count_cta_kernel<<<pl.shards, kCtaThreads, smem, stream>>>(p, (uint32_t)n_buckets,
                                                                         tiles_per_gauss, shard_counts);
        return check_launch("isect_count_cta_kernel");
    }
    if (n_buckets > 0) {
        cudaError_t ce = cudaMemsetAsync(shard_counts, 0, n_buckets * kBucketShards * sizeof(int32_t), stream);
        if (ce != cudaSuccess) return set_error(kErrLaunch, "cudaMemsetAsync: %s", cudaGetErrorString(ce));
    }
    if (n == 0) return kOk;
    isect_count_tiles_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(p, tiles_per_gauss,
                                                                              shard_counts);
    return check_launch("isect_count_tiles_kernel");
}

extern "C" size_t gsb_isect_bucket_offsets_scratch_bytes(long long n_buckets, int shards) {
    const size_t n = (n_buckets > 0 ? (size_t)n_buckets : 1) * (size_t)(shards > 0 ? shards : 1);
    return ((n * sizeof(int64_t) + 255) / 256) * 256 + scan_scratch_bytes(n);
}

extern "C" int gsb_isect_bucket_offsets(const int32_t *shard_counts, long long n_buckets, int shards,
                                        int32_t *offsets, int32_t *bucket_sizes, int32_t *cursor,
                                        const int64_t *nnz_device, int32_t *totals, int32_t *class_list,
                                        void *scratch, size_t scratch_bytes, cudaStream_t stream) {
    if (shards <= 0 || n_buckets < 0 || n_buckets > 0x7fffffffll / shards)
        return set_error(kErrInvalidArgument, "bad bucket count %lld x %d shards", n_buckets, shards);
    cudaError_t ce = cudaMemsetAsync(totals, 0, 5 * sizeof(int32_t), stream);
    if (ce != cudaSuccess) return set_error(kErrLaunch, "cudaMemsetAsync: %s", cudaGetErrorString(ce));
    if (n_buckets == 0) return kOk;
    if (scratch_bytes < gsb_isect_bucket_offsets_scratch_bytes(n_buckets, shards))
        return set_error(kErrInvalidArgument, "bucket offsets scratch too small");
    const size_t n_shards = (size_t)n_buckets * shards;
    int64_t *incl = static_cast<int64_t *>(scratch);
    const size_t incl_bytes = ((n_shards * sizeof(int64_t) + 255) / 256) * 256;
    void *scan_scratch = static_cast<char *>(scratch) + incl_bytes;
    if (int e = inclusive_scan_i32_i64(shard_counts, incl, n_shards, scan_scratch, scratch_bytes - incl_bytes,
                                       stream))
        return e;
    shard_bases_kernel<<<(unsigned)((n_shards + 255) / 256), 256, 0, stream>>>(incl, (uint32_t)n_shards, cursor);
    bucket_starts_kernel<<<(unsigned)((n_buckets + 255) / 256), 256, 0, stream>>>(
        incl, (uint32_t)n_buckets, (uint32_t)shards, offsets, bucket_sizes, nnz_device, totals, class_list);
    return check_launch("bucket_starts_kernel");
}

extern "C" int gsb_isect_bucket_emit(int packed, int I, int N, int nnz, const int64_t *image_ids,
                                     const float *means2d, const int32_t *radii, const float *depths,
                                     const float *conics, const float *opacities, int tile_size,
                                     int tile_width, int tile_height, long long n_isects, int32_t *cursor,
                                     uint64_t *bucket_entries, cudaStream_t stream) {
    IsectParams p;
    if (int e = make_isect_params(p, packed, I, N, nnz, image_ids, means2d, radii, depths, conics,
                                  opacities, tile_size, tile_width, tile_height))
        return e;
    if (n_isects < 0 || n_isects > 0x7fffffffll)
        return set_error(kErrInvalidArgument, "bad intersection count %lld", n_isects);
    const size_t n = packed ? (size_t)nnz : (size_t)I * N;
    if (n == 0 || n_isects == 0) return kOk;
    const uint64_t n_buckets = (uint64_t)I * tile_width * tile_height;
    const BucketPlan pl = bucket_plan(n_buckets, device_sms());
    if (pl.cta) {
        const size_t smem = n_buckets * sizeof(int32_t);
        if (int e = set_cta_smem((const void *)isect_emit_cta_kernel, smem)) return e;
        isect_emit_cta_kernel<<<pl.shards, kCtaThreads, smem, stream>>>(
            p, (uint32_t)n_buckets, (uint32_t)n_isects, cursor, bucket_entries);
        return check_launch("isect_emit_cta_kernel");
    }
    isect_bucket_emit_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(
        p, (uint32_t)n_isects, cursor, bucket_entries);
    return check_launch("isect_bucket_emit_kernel");
}

extern "C" int gsb_isect_bucket_sort_max(void) { return kSplitMin; }

// Scratch of the split path for buckets above kBucketSortMax entries: the
// sub-bucket count, the entries in sub-bucket order and the sub-bucket records
// (a split bucket has more than kBucketSortMax entries and at most 2^kSplitBits
// sub-buckets, so there are fewer than n_isects / 4 of them).
struct SplitScratch {
    int *count;
    uint64_t *entries;
    int32_t *start, *size, *bucket;
    int cap;
};

static size_t align256(size_t v) { return (v + 255) / 256 * 256; }

static size_t split_scratch_layout(long long n_isects, char *base, SplitScratch *ss) {
    const size_t n = n_isects > 0 ? (size_t)n_isects : 0;
    const size_t cap = n / (kSplitMin / (1 << kSplitBits)) + 4096;
    size_t off = 0;
    const size_t o_count = off;
    off += 256;
    const size_t o_entries = off;
    off += align256(n * sizeof(uint64_t));
    const size_t o_start = off;
    off += align256(cap * sizeof(int32_t));
    const size_t o_size = off;
    off += align256(cap * sizeof(int32_t));
    const size_t o_bucket = off;
    off += align256(cap * sizeof(int32_t));
    if (ss != nullptr) {
        ss->count = reinterpret_cast<int *>(base + o_count);
        ss->entries = reinterpret_cast<uint64_t *>(base + o_entries);
        ss->start = reinterpret_cast<int32_t *>(base + o_start);
        ss->size = reinterpret_cast<int32_t *>(base + o_size);
        ss->bucket = reinterpret_cast<int32_t *>(base + o_bucket);
        ss->cap = (int)std::min<size_t>(cap, 0x7fffffff);
    }
    return off;
}

static int bucket_sort(int I, int tile_width, int tile_height, const int32_t *offsets,
                       const int32_t *bucket_sizes, int max_count, int mid_buckets, int large_buckets,
                       const int32_t *class_list, const uint64_t *bucket_entries, long long n_isects,
                       void *scratch, size_t scratch_bytes, int *overflow, int64_t *isect_ids,
                       int32_t *flatten_ids, cudaStream_t stream) {
    const uint64_t n_tiles = (uint64_t)tile_width * (uint64_t)tile_height;
    const uint64_t n_buckets = (uint64_t)I * n_tiles;
    const bool split = max_count > kSplitMin;
    SplitScratch ss = {};
    if (split) {
        if (scratch == nullptr || overflow == nullptr)
            return set_error(kErrUnsupported, "bucket of %d entries exceeds the on-chip sort (%d)", max_count,
                             kBucketSortMax);
        if (scratch_bytes < split_scratch_layout(n_isects, nullptr, nullptr))
            return set_error(kErrInvalidArgument, "bucket sort scratch too small");
        split_scratch_layout(n_isects, static_cast<char *>(scratch), &ss);
    }
    if (n_buckets == 0 || max_count <= 0) return kOk;
    if (n_buckets > 0x7fffffffull) return set_error(kErrInvalidArgument, "too many buckets");
    const uint32_t tb = bit_length(n_tiles);
    // Buckets of up to 1024 entries (most of them): one CTA (256 threads x 4
    // entries) per bucket; a CTA whose bucket is larger returns at once. Larger
    // buckets: the same sort in larger shapes over the class lists, 256 threads
    // x 16 entries up to 4096 entries, 1024 x 16 above, on a side stream next to
    // the first class (forked from and joined back to the caller's stream with
    // events).
    {
        auto kern = bucket_radix_kernel<GSB_RADIX_SMALL>;
        const size_t smem = RadixShape<GSB_RADIX_SMALL>::smem;
        if (int e = set_cta_smem((const void *)kern, smem)) return e;
        kern<<<(unsigned)n_buckets, RadixShape<GSB_RADIX_SMALL>::threads, smem, stream>>>(
            offsets, bucket_sizes, nullptr, (int)n_buckets, 0, bucket_entries, (uint32_t)n_buckets,
            (uint32_t)n_tiles, tb, isect_ids, flatten_ids, SubBuckets{}, 0, 1024);
        if (int e = check_launch("bucket_radix_kernel")) return e;
    }
    if (mid_buckets < 0 || large_buckets < 0 || (uint64_t)mid_buckets + (uint64_t)large_buckets > n_buckets)
        return set_error(kErrInvalidArgument, "bad size class counts %d, %d", mid_buckets, large_buckets);
    if (max_count > 1024 && mid_buckets + large_buckets == 0)
        return set_error(kErrInvalidArgument, "buckets above 1024 entries but empty class lists");
    cudaStream_t side = stream;
    SideStream *sstream = nullptr;
    std::unique_lock<std::mutex> side_lock(g_side_mutex, std::defer_lock);
    if (mid_buckets + large_buckets > 0) {
        side_lock.lock(); // held until the join is recorded
        if (int e = side_stream(&sstream)) return e;
        side = sstream->stream;
        cudaEventRecord(sstream->fork, stream);
        cudaStreamWaitEvent(side, sstream->fork, 0);
    }
    const int sms = device_sms();
    if (mid_buckets > 0) {
        auto kern = bucket_radix_kernel<GSB_RADIX_MID>;
        const int threads = RadixShape<GSB_RADIX_MID>::threads;
        const size_t smem = RadixShape<GSB_RADIX_MID>::smem;
        static_assert(RadixShape<GSB_RADIX_MID>::cap >= 4096, "mid class capacity");
        if (int e = set_cta_smem((const void *)kern, smem)) return e;
        kern<<<(unsigned)std::min(mid_buckets, RadixShape<GSB_RADIX_MID>::per_sm * sms), threads, smem, side>>>(
            offsets, bucket_sizes, class_list, mid_buckets, 0, bucket_entries, (uint32_t)n_buckets,
            (uint32_t)n_tiles, tb, isect_ids, flatten_ids, SubBuckets{}, 1024, 4096);
        if (int e = check_launch("bucket_radix_kernel")) return e;
    }
    if (large_buckets > 0) {
        auto kern = bucket_radix_kernel<GSB_RADIX_LARGE>;
        const int threads = RadixShape<GSB_RADIX_LARGE>::threads;
        const size_t smem = RadixShape<GSB_RADIX_LARGE>::smem;
        static_assert(RadixShape<GSB_RADIX_LARGE>::cap >= kBucketSortMax, "large class capacity");
        if (int e = set_cta_smem((const void *)kern, smem)) return e;
        kern<<<(unsigned)std::min(large_buckets, RadixShape<GSB_RADIX_LARGE>::per_sm * sms), threads, smem, side>>>(
            offsets, bucket_sizes, class_list, large_buckets, 1, bucket_entries, (uint32_t)n_buckets,
            (uint32_t)n_tiles, tb, isect_ids, flatten_ids, SubBuckets{}, 4096, kSplitMin);
        if (int e = check_launch("bucket_radix_kernel")) return e;
    }
    if (split && large_buckets > 0) {
        // buckets above kBucketSortMax: split into sub-buckets, then the same
        // on-chip sorts over the device list of sub-buckets
        cudaError_t ce = cudaMemsetAsync(ss.count, 0, sizeof(int), side);
        if (ce == cudaSuccess) ce = cudaMemsetAsync(overflow, 0, sizeof(int), side);
        if (ce != cudaSuccess) return set_error(kErrLaunch, "cudaMemsetAsync: %s", cudaGetErrorString(ce));
        bucket_split_kernel<<<(unsigned)std::min(large_buckets, 2 * sms), kSplitThreads, 0, side>>>(
            offsets, bucket_sizes, class_list, large_buckets, (uint32_t)n_buckets, bucket_entries, ss.entries,
            ss.count, ss.start, ss.size, ss.bucket, ss.cap, overflow);
        if (int e = check_launch("bucket_split_kernel")) return e;
        const SubBuckets sub{ss.count, ss.start, ss.size, ss.bucket, ss.cap};
        {
            auto kern = bucket_radix_kernel<GSB_RADIX_SMALL>;
            const size_t smem = RadixShape<GSB_RADIX_SMALL>::smem;
            if (int e = set_cta_smem((const void *)kern, smem)) return e;
            kern<<<(unsigned)(RadixShape<GSB_RADIX_SMALL>::per_sm * sms), RadixShape<GSB_RADIX_SMALL>::threads, smem,
                   side>>>(offsets, bucket_sizes, nullptr, 0, 0, ss.entries, (uint32_t)n_buckets,
                           (uint32_t)n_tiles, tb, isect_ids, flatten_ids, sub, 0, 1024);
            if (int e = check_launch("bucket_radix_kernel")) return e;
        }
        {
            auto kern = bucket_radix_kernel<GSB_RADIX_MID>;
            const size_t smem = RadixShape<GSB_RADIX_MID>::smem;
            if (int e = set_cta_smem((const void *)kern, smem)) return e;
            kern<<<(unsigned)(RadixShape<GSB_RADIX_MID>::per_sm * sms), RadixShape<GSB_RADIX_MID>::threads, smem,
                   side>>>(offsets, bucket_sizes, class_list, 0, 0, ss.entries, (uint32_t)n_buckets,
                           (uint32_t)n_tiles, tb, isect_ids, flatten_ids, sub, 1024, 4096);
            if (int e = check_launch("bucket_radix_kernel")) return e;
        }
        {
            auto kern = bucket_radix_kernel<GSB_RADIX_LARGE>;
            const size_t smem = RadixShape<GSB_RADIX_LARGE>::smem;
            if (int e = set_cta_smem((const void *)kern, smem)) return e;
            kern<<<(unsigned)(RadixShape<GSB_RADIX_LARGE>::per_sm * sms), RadixShape<GSB_RADIX_LARGE>::threads,
                   smem, side>>>(offsets, bucket_sizes, class_list, 0, 0, ss.entries, (uint32_t)n_buckets,
                                 (uint32_t)n_tiles, tb, isect_ids, flatten_ids, sub, 4096, kBucketSortMax);
            if (int e = check_launch("bucket_radix_kernel")) return e;
        }
    }
    if (sstream != nullptr) {
        cudaEventRecord(sstream->join, side);
        cudaStreamWaitEvent(stream, sstream->join, 0);
        const cudaError_t ce = cudaGetLastError();
        if (ce != cudaSuccess) return set_error(kErrLaunch, "bucket sort stream join: %s", cudaGetErrorString(ce));
    }
    return kOk;
}

extern "C" int gsb_isect_bucket_sort(int I, int tile_width, int tile_height, const int32_t *offsets,
                                     const int32_t *bucket_sizes, int max_count, int mid_buckets,
                                     int large_buckets, const int32_t *class_list, const uint64_t *bucket_entries,
                                     int64_t *isect_ids, int32_t *flatten_ids,
                                     cudaStream_t stream) {
    return bucket_sort(I, tile_width, tile_height, offsets, bucket_sizes, max_count, mid_buckets, large_buckets,
                       class_list, bucket_entries, 0, nullptr, 0, nullptr, isect_ids, flatten_ids, stream);
}

extern "C" size_t gsb_isect_bucket_sort_scratch_bytes(long long n_isects) {
    return split_scratch_layout(n_isects, nullptr, nullptr);
}

extern "C" int gsb_isect_bucket_sort_ex(int I, int tile_width, int tile_height, const int32_t *offsets,
                                        const int32_t *bucket_sizes, int max_count, int mid_buckets,
                                        int large_buckets, const int32_t *class_list,
                                        const uint64_t *bucket_entries, long long n_isects, void *scratch,
                                        size_t scratch_bytes, int *overflow, int64_t *isect_ids,
                                        int32_t *flatten_ids, cudaStream_t stream) {
    return bucket_sort(I, tile_width, tile_height, offsets, bucket_sizes, max_count, mid_buckets, large_buckets,
                       class_list, bucket_entries, n_isects, scratch, scratch_bytes, overflow, isect_ids,
                       flatten_ids, stream);
}
