// rasterize_to_indices_in_range: the (Gaussian, pixel) pairs that a range of
// front-to-back splat batches contributes to each pixel, given the pixels'
// transmittances so far (reference RasterizeToIndices3DGS.cu:36-200,
// Rasterization.cpp:216-300). Used by the reference's PyTorch compositing path
// (_torch_impl.py:573-683) and for debugging; two passes like the reference:
// per-pixel counts, then (after a prefix sum over pixels in (image, row,
// column) order) the pairs written in that order, front to back within a pixel.
//
// One CTA per (image, tile) with one thread per pixel; each batch of
// tile_size^2 tile-list entries is staged in shared memory and walked by every
// pixel of the tile until the pixel's transmittance falls to the threshold.
#include "common.cuh"
#include "gsb_internal.h"

namespace gsb {

struct IndicesParams {
    uint32_t range_start, range_end, I, N, n_isects;
    const float *means2d, *conics, *opacities;
    uint32_t W, H, tile_size, tile_width, tile_height;
    const int32_t *tile_offsets, *flatten_ids;
    const float *transmittances;
    const int64_t *chunk_ends; // inclusive prefix sum of the counts (write pass), or NULL (count pass)
    int32_t *chunk_cnts;
    int64_t *gaussian_ids, *pixel_ids;
};

__global__ void __launch_bounds__(1024) raster_indices_kernel(IndicesParams p) {
    extern __shared__ float sm[];
    const uint32_t bs = blockDim.x * blockDim.y;
    int32_t *ids = reinterpret_cast<int32_t *>(sm);  // [bs]
    float *xyo = sm + bs;                            // [bs][3]: x, y, opacity
    float *con = xyo + 3 * bs;                       // [bs][3]
    const uint32_t image = blockIdx.y;
    const uint32_t tile = blockIdx.x;
    const uint32_t ty = tile / p.tile_width, tx = tile % p.tile_width;
    const uint32_t i = ty * p.tile_size + threadIdx.y;
    const uint32_t j = tx * p.tile_size + threadIdx.x;
    const uint32_t tr = threadIdx.y * blockDim.x + threadIdx.x;
    const bool inside = i < p.H && j < p.W;
    const size_t pix = (size_t)i * p.W + j;
    const size_t gpix = (size_t)image * p.H * p.W + pix;
    const float px = (float)j + 0.5f, py = (float)i + 0.5f;
    const uint32_t n_tiles = p.tile_width * p.tile_height;
    const int32_t range0 = p.tile_offsets[(size_t)image * n_tiles + tile];
    const int32_t range1 = (image == p.I - 1 && tile == n_tiles - 1)
                               ? (int32_t)p.n_isects
                               : p.tile_offsets[(size_t)image * n_tiles + tile + 1];
    const uint32_t n_batches = (uint32_t)(range1 - range0 + (int32_t)bs - 1) / bs;
    if (p.range_start >= n_batches) return; // uniform over the CTA
    const bool first_pass = p.chunk_ends == nullptr;
    int64_t base = 0;
    if (!first_pass && inside) base = gpix == 0 ? 0 : p.chunk_ends[gpix - 1];
    float trans = inside ? p.transmittances[gpix] : 0.f;
    bool done = !inside;
    int32_t cnt = 0;
    const uint32_t b_end = min(p.range_end, n_batches);
    for (uint32_t b = p.range_start; b < b_end; ++b) {
        if (__syncthreads_count(done) >= (int)bs) break;
        const int32_t start = range0 + (int32_t)(bs * b);
        const int32_t idx = start + (int32_t)tr;
        if (idx < range1) {
            const int32_t g = p.flatten_ids[idx];
            ids[tr] = g;
            xyo[tr * 3] = p.means2d[(size_t)g * 2];
            xyo[tr * 3 + 1] = p.means2d[(size_t)g * 2 + 1];
            xyo[tr * 3 + 2] = p.opacities[g];
            con[tr * 3] = p.conics[(size_t)g * 3];
            con[tr * 3 + 1] = p.conics[(size_t)g * 3 + 1];
            con[tr * 3 + 2] = p.conics[(size_t)g * 3 + 2];
        }
        __syncthreads();
        const uint32_t n = min(bs, (uint32_t)(range1 - start));
        for (uint32_t t = 0; t < n && !done; ++t) {
            const float dx = xyo[t * 3] - px, dy = xyo[t * 3 + 1] - py;
            const float sigma = 0.5f * (con[t * 3] * dx * dx + con[t * 3 + 2] * dy * dy) + con[t * 3 + 1] * dx * dy;
            const float alpha = fminf(kMaxAlpha, xyo[t * 3 + 2] * __expf(-sigma));
            if (sigma < 0.f || alpha < kAlphaThreshold) continue;
            const float next = trans * (1.f - alpha);
            if (next <= kTransmittanceThreshold) { // exclusive: this splat is not counted
                done = true;
                break;
            }
            if (!first_pass) {
                p.gaussian_ids[base + cnt] = (int64_t)(ids[t] % (int32_t)p.N);
                p.pixel_ids[base + cnt] = (int64_t)gpix;
            }
            ++cnt;
            trans = next;
        }
        __syncthreads(); // the batch is overwritten next
    }
    if (first_pass && inside) p.chunk_cnts[gpix] = cnt;
}

} // namespace gsb

using namespace gsb;

extern "C" int gsb_rasterize_to_indices(int range_start, int range_end, int I, int N, long long n_isects,
                                        const float *means2d, const float *conics, const float *opacities,
                                        int width, int height, int tile_size, int tile_width, int tile_height,
                                        const int32_t *tile_offsets, const int32_t *flatten_ids,
                                        const float *transmittances, const int64_t *chunk_ends,
                                        int32_t *chunk_cnts, int64_t *gaussian_ids, int64_t *pixel_ids,
                                        cudaStream_t stream) {
    if (tile_size <= 0 || tile_size > 32)
        return set_error(kErrUnsupported, "tile_size %d: one thread per pixel needs 1..32", tile_size);
    if (I < 0 || N <= 0 || width < 0 || height < 0 || range_start < 0 || range_end < 0 || n_isects < 0 ||
        n_isects > 0x7fffffffll)
        return set_error(kErrInvalidArgument, "bad sizes");
    if ((long long)tile_width * tile_size < width || (long long)tile_height * tile_size < height)
        return set_error(kErrInvalidArgument, "tiles %dx%d of %d px do not cover %dx%d", tile_width, tile_height,
                         tile_size, width, height);
    if (chunk_ends == nullptr ? chunk_cnts == nullptr : (gaussian_ids == nullptr || pixel_ids == nullptr))
        return set_error(kErrInvalidArgument, "count pass needs chunk_cnts, write pass the id outputs");
    if (I > 65535) return set_error(kErrUnsupported, "%d images (at most 65535 per call)", I);
    if (I == 0 || n_isects == 0 || range_end <= range_start) return kOk;
    IndicesParams p;
    p.range_start = (uint32_t)range_start;
    p.range_end = (uint32_t)range_end;
    p.I = (uint32_t)I;
    p.N = (uint32_t)N;
    p.n_isects = (uint32_t)n_isects;
    p.means2d = means2d;
    p.conics = conics;
    p.opacities = opacities;
    p.W = (uint32_t)width;
    p.H = (uint32_t)height;
    p.tile_size = (uint32_t)tile_size;
    p.tile_width = (uint32_t)tile_width;
    p.tile_height = (uint32_t)tile_height;
    p.tile_offsets = tile_offsets;
    p.flatten_ids = flatten_ids;
    p.transmittances = transmittances;
    p.chunk_ends = chunk_ends;
    p.chunk_cnts = chunk_cnts;
    p.gaussian_ids = gaussian_ids;
    p.pixel_ids = pixel_ids;
    const dim3 block((unsigned)tile_size, (unsigned)tile_size);
    const dim3 grid((unsigned)(tile_width * tile_height), (unsigned)I);
    const size_t smem = (size_t)tile_size * tile_size * 7 * sizeof(float);
    raster_indices_kernel<<<grid, block, smem, stream>>>(p);
    return check_launch("raster_indices_kernel");
}
