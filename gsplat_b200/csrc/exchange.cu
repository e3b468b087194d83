// Row packing for the Gaussian-sharded exchange.
//
// The reference's distributed rasterization (gsplat/rendering.py:907-975,
// gsplat/distributed.py:182-272) concatenates the projected splat attributes
// column-wise into one buffer, exchanges rows with an all-to-all and splits the
// received buffer again, and remaps camera / Gaussian ids with a few torch ops.
// These kernels do each of those steps in one launch: gather the columns of
// several row-major arrays into one row-major buffer of 4-byte words (float,
// int32, or int64 as two words), scatter such a buffer back into separate
// arrays, and remap the ids.
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

// Packing: a CTA moves a block of consecutive rows through shared memory so
// that both sides are read and written coalesced: each array's rows of the
// block are one contiguous range, and so are the block's packed rows.
constexpr int kRowThreads = 256;
constexpr int kRowSmemWords = 12 * 1024; // 48 KiB of staging per CTA

// Staged rows are padded to an odd word count so that threads walking one
// column of the block (stride = the row) hit distinct banks.
__device__ __forceinline__ int stage_stride(int total) { return total | 1; }

__device__ __forceinline__ int block_rows(int total) {
    const int r = kRowSmemWords / stage_stride(total);
    return r < 1 ? 1 : r;
}

__global__ void __launch_bounds__(kRowThreads) pack_rows_kernel(RowArrays a, long long rows,
                                                                const int64_t *__restrict__ rows_device,
                                                                uint32_t *__restrict__ buf) {
    __shared__ uint32_t stage[kRowSmemWords];
    if (rows_device != nullptr && *rows_device < rows) rows = *rows_device;
    const int S = stage_stride(a.total);
    const int R = block_rows(a.total);
    for (long long r0 = (long long)blockIdx.x * R; r0 < rows; r0 += (long long)gridDim.x * R) {
        const int nr = (int)min((long long)R, rows - r0);
        int first = 0;
        for (int j = 0; j < a.n; ++j) {
            const int w = a.words[j];
            const uint32_t *src = static_cast<const uint32_t *>(a.ptr[j]);
            for (int i = threadIdx.x; i < nr * w; i += kRowThreads) {
                const int r = i / w, k = i - r * w;
                stage[r * S + first + k] = src ? src[r0 * w + i] : 0u;
            }
            first += w;
        }
        __syncthreads();
        uint32_t *dst = buf + r0 * a.total;
        for (int i = threadIdx.x; i < nr * a.total; i += kRowThreads) {
            const int r = i / a.total, k = i - r * a.total;
            dst[i] = stage[r * S + k];
        }
        __syncthreads();
    }
}

// Unpacking reads each packed row whole and writes every array's row: one
// thread per row (measured faster than the staged form for this direction).
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
    if ((a.total | 1) > kRowSmemWords)
        return set_error(kErrInvalidArgument, "row packing: %d words per row (at most %d)", a.total, kRowSmemWords);
    return kOk;
}

static unsigned grid_for(long long work) {
    const long long blocks = (work + 255) / 256;
    return (unsigned)(blocks < 148 * 16 ? (blocks > 0 ? blocks : 1) : 148 * 16);
}

// CTAs for a row block loop: one per block of rows, at most 4 per SM worth
static unsigned grid_for_rows(long long rows, int total) {
    const long long R = kRowSmemWords / (total | 1) > 0 ? kRowSmemWords / (total | 1) : 1;
    const long long blocks = (rows + R - 1) / R;
    return (unsigned)(blocks < 148 * 4 ? (blocks > 0 ? blocks : 1) : 148 * 4);
}

} // namespace gsb

using namespace gsb;

extern "C" int gsb_pack_rows(long long rows, const int64_t *rows_device, int n_arrays, void *const *srcs,
                             const int *words, uint32_t *buf, cudaStream_t stream) {
    RowArrays a;
    if (int e = make_arrays(a, n_arrays, srcs, words)) return e;
    if (rows <= 0) return kOk;
    pack_rows_kernel<<<grid_for_rows(rows, a.total), kRowThreads, 0, stream>>>(a, rows, rows_device, buf);
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
