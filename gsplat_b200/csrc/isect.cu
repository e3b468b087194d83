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
#include "common.cuh"
#include "gsb_internal.h"

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

// AccuTile sweep (IntersectTile.cu:54-126 and 195-253). Returns the number of
// tiles; emits them when `sink` is non-null.
template <bool EMIT>
__device__ uint32_t accutile(const IsectParams &p, float mx, float my, float A, float B, float C,
                             float opacity, EmitSink *sink) {
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
    float amin_x = DET_ADD(my, bxc), amin_y = DET_ADD(mx, bya);
    float amax_x = DET_SUB(my, bxc), amax_y = DET_SUB(mx, bya);
    const float ts = (float)p.tile_size;
    const int tw = (int)p.tile_width, th = (int)p.tile_height;
    int rmin_x = max(0, min(tw, det_f2i_rz(DET_DIV(bmin_x, ts))));
    int rmin_y = max(0, min(th, det_f2i_rz(DET_DIV(bmin_y, ts))));
    int rmax_x = max(0, min(tw, det_f2i_rz(DET_ADD(DET_DIV(bmax_x, ts), 1.f))));
    int rmax_y = max(0, min(th, det_f2i_rz(DET_ADD(DET_DIV(bmax_y, ts), 1.f))));
    const int y_span = rmax_y - rmin_y, x_span = rmax_x - rmin_x;
    if (y_span * x_span == 0) return 0;
    const bool is_y = y_span < x_span;
    if (is_y) {
        int ti;
        float tf;
        ti = rmin_x; rmin_x = rmin_y; rmin_y = ti;
        ti = rmax_x; rmax_x = rmax_y; rmax_y = ti;
        tf = bmin_x; bmin_x = bmin_y; bmin_y = tf;
        tf = bmax_x; bmax_x = bmax_y; bmax_y = tf;
        tf = amin_x; amin_x = amin_y; amin_y = tf;
        tf = amax_x; amax_x = amax_y; amax_y = tf;
    }
    uint32_t count = 0;
    LinePair cur_hi = {bmax_y, bmin_y};
    float min_line = DET_MUL((float)rmin_x, ts);
    LinePair cur_lo = (bmin_x <= min_line) ? ellipse_line(A, B, C, disc, t, mx, my, is_y, min_line)
                                           : cur_hi;
    for (int u = rmin_x; u < rmax_x; ++u) {
        const float max_line = DET_ADD(min_line, ts);
        if (max_line <= bmax_x) cur_hi = ellipse_line(A, B, C, disc, t, mx, my, is_y, max_line);
        const float emin = (min_line <= amin_y && amin_y < max_line) ? bmin_y
                                                                    : det_fmin(cur_lo.lo, cur_hi.lo);
        const float emax = (min_line <= amax_y && amax_y < max_line) ? bmax_y
                                                                    : det_fmax(cur_lo.hi, cur_hi.hi);
        const int v0 = max(rmin_y, min(rmax_y, det_f2i_rz(DET_DIV(emin, ts))));
        const int v1 = min(rmax_y, max(rmin_y, det_f2i_rz(DET_ADD(DET_DIV(emax, ts), 1.f))));
        if (v1 > v0) {
            count += (uint32_t)(v1 - v0);
            if (EMIT) {
                for (int v = v0; v < v1; ++v)
                    sink->put(is_y ? (int64_t)u * tw + v : (int64_t)v * tw + u);
            }
        }
        cur_lo = cur_hi;
        min_line = max_line;
    }
    return count;
}

template <bool EMIT>
__device__ uint32_t aabb_tiles(const IsectParams &p, float mx, float my, int32_t rx, int32_t ry,
                               EmitSink *sink) {
    const float ts = (float)p.tile_size;
    const float trx = DET_DIV((float)rx, ts), try_ = DET_DIV((float)ry, ts);
    const float tx = DET_DIV(mx, ts), ty = DET_DIV(my, ts);
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

template <bool EMIT>
__device__ __forceinline__ uint32_t splat_tiles(const IsectParams &p, uint32_t idx, EmitSink *sink) {
    const int32_t rx = p.radii[(size_t)idx * 2], ry = p.radii[(size_t)idx * 2 + 1];
    if (rx <= 0 || ry <= 0) return 0;
    const float mx = p.means2d[(size_t)idx * 2], my = p.means2d[(size_t)idx * 2 + 1];
    if (p.conics != nullptr && p.opacities != nullptr) {
        return accutile<EMIT>(p, mx, my, p.conics[(size_t)idx * 3], p.conics[(size_t)idx * 3 + 1],
                              p.conics[(size_t)idx * 3 + 2], p.opacities[idx], sink);
    }
    return aabb_tiles<EMIT>(p, mx, my, rx, ry, sink);
}

__global__ void __launch_bounds__(256) isect_count_kernel(IsectParams p, int32_t *tiles_per_gauss) {
    const uint32_t idx = blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t n = p.packed ? p.nnz : p.I * p.N;
    if (idx >= n) return;
    tiles_per_gauss[idx] = (int32_t)splat_tiles<false>(p, idx, nullptr);
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
