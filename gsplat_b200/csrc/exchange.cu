// Row packing for the Gaussian-sharded exchange.
//
// The reference's distributed rasterization (gsplat/rendering.py:907-975,
// gsplat/distributed.py:182-272) concatenates the projected splat attributes
// column-wise into one buffer, exchanges rows with an all-to-all and splits the
// received buffer again, and remaps camera / Gaussian ids with a few torch ops.
// These kernels do each of those steps in one launch: gather the columns of
// several row-major arrays into one row-major buffer of 4-byte words (float,
// int32, or int64 as two words), scatter such a buffer back into separate
// arrays, and remap the ids. One thread per row: the source / destination
// arrays are read and written coalesced, the packed rows are contiguous per
// thread.
#include "common.cuh"
#include "gsb_internal.h"

namespace gsb {

constexpr int kMaxRowArrays = 16;

struct RowArrays {
    void *ptr[kMaxRowArrays]; // 4-byte words, row-major; NULL = zeros (pack) / skipped (unpack)
    int words[kMaxRowArrays]; // words per row of each array
    int n;
    int total; // sum of words
};

__global__ void __launch_bounds__(256) pack_rows_kernel(RowArrays a, long long rows,
                                                        const int64_t *__restrict__ rows_device,
                                                        uint32_t *__restrict__ buf) {
    if (rows_device != nullptr && *rows_device < rows) rows = *rows_device;
    for (long long r = (long long)blockIdx.x * blockDim.x + threadIdx.x; r < rows;
         r += (long long)gridDim.x * blockDim.x) {
        uint32_t *dst = buf + r * a.total;
        for (int j = 0; j < a.n; ++j) {
            const int w = a.words[j];
            const uint32_t *src = static_cast<const uint32_t *>(a.ptr[j]);
            if (src) {
                src += r * w;
                for (int k = 0; k < w; ++k) dst[k] = src[k];
            } else {
                for (int k = 0; k < w; ++k) dst[k] = 0u;
            }
            dst += w;
        }
    }
}

__global__ void __launch_bounds__(256) unpack_rows_kernel(RowArrays a, long long rows, int row_words,
                                                          const uint32_t *__restrict__ buf) {
    for (long long r = (long long)blockIdx.x * blockDim.x + threadIdx.x; r < rows;
         r += (long long)gridDim.x * blockDim.x) {
        const uint32_t *src = buf + r * row_words;
        for (int j = 0; j < a.n; ++j) {
            const int w = a.words[j];
            uint32_t *dst = static_cast<uint32_t *>(a.ptr[j]);
            if (dst) {
                dst += r * w;
                for (int k = 0; k < w; ++k) dst[k] = src[k];
            }
            src += w;
        }
    }
}

// Destination rank of camera c is c / cams_per_rank; camera ids become local to
// that rank and Gaussian ids are shifted by that rank's Gaussian offset, the
// Gaussian counts of the ranks before it (reference rendering.py:944-959).
__global__ void exchange_ids_kernel(long long n, const int64_t *__restrict__ n_device,
                                    const int64_t *__restrict__ camera_ids,
                                    const int64_t *__restrict__ gaussian_ids, int cams_per_rank,
                                    const int64_t *__restrict__ gauss_counts, int64_t *__restrict__ cam_out,
                                    int64_t *__restrict__ gid_out) {
    if (n_device != nullptr && *n_device < n) n = *n_device;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        const int64_t c = camera_ids[i];
        const int64_t dst = c / cams_per_rank;
        int64_t off = 0;
        for (int64_t r = 0; r < dst; ++r) off += gauss_counts[r];
        cam_out[i] = c - dst * cams_per_rank;
        gid_out[i] = gaussian_ids[i] + off;
    }
}

static int make_arrays(RowArrays &a, int n_arrays, void *const *ptrs, const int *words) {
    if (n_arrays <= 0 || n_arrays > kMaxRowArrays)
        return set_error(kErrInvalidArgument, "row packing: %d arrays (1..%d)", n_arrays, kMaxRowArrays);
    a.n = n_arrays;
    a.total = 0;
    for (int j = 0; j < n_arrays; ++j) {
        if (words[j] <= 0) return set_error(kErrInvalidArgument, "row packing: array %d has %d words", j, words[j]);
        a.ptr[j] = ptrs[j];
        a.words[j] = words[j];
        a.total += words[j];
    }
    return kOk;
}

static unsigned grid_for(long long work) {
    const long long blocks = (work + 255) / 256;
    return (unsigned)(blocks < 148 * 16 ? (blocks > 0 ? blocks : 1) : 148 * 16);
}

} // namespace gsb

using namespace gsb;

extern "C" int gsb_pack_rows(long long rows, const int64_t *rows_device, int n_arrays, void *const *srcs,
                             const int *words, uint32_t *buf, cudaStream_t stream) {
    RowArrays a;
    if (int e = make_arrays(a, n_arrays, srcs, words)) return e;
    if (rows <= 0) return kOk;
    pack_rows_kernel<<<grid_for(rows), 256, 0, stream>>>(a, rows, rows_device, buf);
    return check_launch("pack_rows_kernel");
}

extern "C" int gsb_unpack_rows(long long rows, int row_words, const uint32_t *buf, int n_arrays,
                               void *const *dsts, const int *words, cudaStream_t stream) {
    RowArrays a;
    if (int e = make_arrays(a, n_arrays, dsts, words)) return e;
    if (a.total > row_words)
        return set_error(kErrInvalidArgument, "row unpacking: %d words requested from rows of %d", a.total,
                         row_words);
    if (rows <= 0) return kOk;
    unpack_rows_kernel<<<grid_for(rows), 256, 0, stream>>>(a, rows, row_words, buf);
    return check_launch("unpack_rows_kernel");
}

extern "C" int gsb_exchange_ids(long long n, const int64_t *n_device, const int64_t *camera_ids,
                                const int64_t *gaussian_ids, int cams_per_rank, const int64_t *gauss_counts,
                                int64_t *cam_out, int64_t *gid_out, cudaStream_t stream) {
    if (cams_per_rank <= 0) return set_error(kErrInvalidArgument, "cams_per_rank must be positive");
    if (n <= 0) return kOk;
    exchange_ids_kernel<<<grid_for(n), 256, 0, stream>>>(n, n_device, camera_ids, gaussian_ids, cams_per_rank,
                                                         gauss_counts, cam_out, gid_out);
    return check_launch("exchange_ids_kernel");
}
