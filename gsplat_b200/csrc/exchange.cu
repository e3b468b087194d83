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
#include <cstring>

#include <atomic>

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
__global__ void __launch_bounds__(256) unpack_rows_kernel(RowArrays a, long long rows, const int64_t *rows_device,
                                                          int row_words, const uint32_t *__restrict__ buf) {
    if (rows_device != nullptr && *rows_device < rows) rows = *rows_device;
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
    if (ptrs == nullptr || words == nullptr) return set_error(kErrInvalidArgument, "row packing: no array list");
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

// --------------------------------------------------------------------------
// Peer-memory exchange (GPUs of one node, CUDA IPC mappings over NVLink)
//
// Each rank owns one arena, mapped by every other rank:
//   [0, kMailboxBytes)          PeerMailbox, written by the peers
//   recv buffer 0 / 1           rows received from every source, source r's rows
//                               in its region [region(r), region(r) + count)
//                               (exchanges alternate between the two)
//   grad buffer                 gradient rows of this rank's own packed rows,
//                               written back by the ranks that rendered them
// A sender stores rows straight into the destinations' receive buffers; the
// last CTA to finish publishes counts and a flag per destination (release,
// system scope) after a system fence, so a receiver that acquires the flag sees
// every row. Flags hold the exchange's sequence number, so they never need
// resetting. Every wait is bounded: a wait that gives up records its kind in the
// group's error word (host-mapped) and lets the kernel finish.
constexpr int kMaxPeers = 8;
constexpr long long kMailboxBytes = 4096;
constexpr int kPeerStageWords = 11 * 1024; // staging of the peer kernels (44 KiB, beside their small tables)

__device__ __forceinline__ int peer_block_rows(int total) {
    const int r = kPeerStageWords / stage_stride(total);
    return r < 1 ? 1 : r;
}
constexpr long long kSpinLimit = 1ll << 21; // x ~0.5-2 us per poll: a few seconds at most

// Polls a wait makes before it gives up (gsb_peer_set_wait_limit); read when a
// launch is set up, so it applies to the launches that follow the call.
static std::atomic<long long> g_wait_limit{kSpinLimit};

struct PeerMailbox {
    unsigned long long rows_flag[kMaxPeers];     // [src]: exchange number of src's rows for this rank
    long long rows_count[kMaxPeers];             // [src]: rows src sent here
    long long rows_first[kMaxPeers];             // [src]: src's local index of the first of them
    unsigned long long consumed_flag[kMaxPeers]; // [dst]: dst has read this rank's rows of that exchange
    unsigned long long grad_flag[kMaxPeers];     // [dst]: dst's gradients for this rank's rows are written
    unsigned int done_ctas;                      // last-CTA counters of this rank's kernels
    unsigned int done_ctas_grad;
};
static_assert(sizeof(PeerMailbox) <= kMailboxBytes, "mailbox");

struct PeerView {
    char *arena[kMaxPeers];
    long long recv_offset, recv_stride, grad_offset;
    long long wait_limit; // polls before a wait gives up
    int rank, world;
    int *error;
};

__device__ __forceinline__ PeerMailbox *mailbox(const PeerView &v, int r) {
    return reinterpret_cast<PeerMailbox *>(v.arena[r]);
}

__device__ __forceinline__ void store_release_sys(unsigned long long *p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long load_acquire_sys(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Waits until *flag >= want; returns false (after recording `kind`) when the
// bound of `limit` polls runs out.
__device__ bool wait_flag(const unsigned long long *flag, unsigned long long want, int *error, int kind,
                          long long limit) {
    for (long long it = 0; it < limit; ++it) {
        if (load_acquire_sys(flag) >= want) return true;
        __nanosleep(128);
    }
    volatile int *e = error; // host-mapped: a plain store (no atomics over the host link)
    if (*e == 0) *e = kind;
    return false;
}

// Rows of source r start at region[r] in every receive buffer: C_per x the
// Gaussian counts of the ranks before r.
__device__ __forceinline__ long long region_start(const int64_t *n_world, int cams_per_rank, int r) {
    long long s = 0;
    for (int k = 0; k < r; ++k) s += n_world[k];
    return s * cams_per_rank;
}

// The sender waits until every destination has read the rows (and counts) of
// the previous exchange, so neither a receive buffer nor a mailbox entry is
// overwritten while in use, even by forward-only exchanges back to back.
__global__ void peer_wait_consumed_kernel(PeerView v, unsigned long long epoch) {
    const int d = threadIdx.x;
    if (d >= v.world || epoch < 2) return;
    wait_flag(&mailbox(v, v.rank)->consumed_flag[d], epoch - 1, v.error, 1, v.wait_limit);
}

// Row block staging as in pack_rows_kernel; each staged word goes to the
// destination of its row: dest d = the rank whose local row range
// [bounds[d], bounds[d + 1]) holds it.
__global__ void __launch_bounds__(kRowThreads) peer_send_rows_kernel(RowArrays a, long long rows, const int64_t *rows_device,
                                                                   const int64_t *__restrict__ bounds,
                                                                   const int64_t *__restrict__ n_world,
                                                                   int cams_per_rank, long long cap_recv, PeerView v,
                                                                   unsigned long long epoch, int buf) {
    __shared__ uint32_t stage[kPeerStageWords];
    __shared__ long long s_bounds[kMaxPeers + 1];
    __shared__ long long s_base[kMaxPeers]; // region of this rank in every destination
    __shared__ bool s_last;
    if (rows_device != nullptr && *rows_device < rows) rows = *rows_device;
    if (threadIdx.x <= (unsigned)v.world) s_bounds[threadIdx.x] = bounds[threadIdx.x];
    if (threadIdx.x == 0) {
        const long long base = region_start(n_world, cams_per_rank, v.rank);
        for (int d = 0; d < v.world; ++d) s_base[d] = base;
    }
    __syncthreads();
    const int S = stage_stride(a.total);
    const int R = peer_block_rows(a.total);
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
        for (int i = threadIdx.x; i < nr * a.total; i += kRowThreads) {
            const int r = i / a.total, k = i - r * a.total;
            const long long row = r0 + r;
            int d = 0;
            while (d + 1 < v.world && row >= s_bounds[d + 1]) ++d;
            const long long slot = s_base[d] + (row - s_bounds[d]);
            if (slot < cap_recv) {
                uint32_t *dst = reinterpret_cast<uint32_t *>(v.arena[d] + v.recv_offset + buf * v.recv_stride);
                dst[slot * a.total + k] = stage[r * S + k];
            }
        }
        __syncthreads();
    }
    // publish: every CTA fences its stores, the last one raises the flags
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(&mailbox(v, v.rank)->done_ctas, 1u) == gridDim.x - 1;
    __syncthreads();
    if (s_last && threadIdx.x < (unsigned)v.world) {
        __threadfence_system();
        const int d = threadIdx.x;
        PeerMailbox *box = mailbox(v, d);
        box->rows_count[v.rank] = s_bounds[d + 1] - s_bounds[d];
        box->rows_first[v.rank] = s_bounds[d];
        __threadfence_system();
        store_release_sys(&box->rows_flag[v.rank], epoch);
        if (d == 0) mailbox(v, v.rank)->done_ctas = 0u;
    }
}

// Receiver: wait for every source's rows, then the route of this exchange:
// route[0..world] = prefix of the received counts by source, route[world + 1
// + r] = source r's local index of its first row sent here (kept with the
// exchange, for the gradients), and the received-row total.
__global__ void peer_wait_rows_kernel(PeerView v, unsigned long long epoch, int64_t *route, int64_t *nnz_recv) {
    __shared__ long long cnt[kMaxPeers];
    const int r = threadIdx.x;
    PeerMailbox *me = mailbox(v, v.rank);
    if (r < v.world) {
        const bool ok = wait_flag(&me->rows_flag[r], epoch, v.error, 2, v.wait_limit);
        cnt[r] = ok ? me->rows_count[r] : 0;
        route[v.world + 1 + r] = ok ? me->rows_first[r] : 0;
    }
    __syncthreads();
    if (r == 0) {
        long long s = 0;
        for (int k = 0; k < v.world; ++k) {
            route[k] = s;
            s += cnt[k];
        }
        route[v.world] = s;
        *nnz_recv = s;
    }
}

// One thread per received row: source r found from the prefix, row copied out
// of r's region into the separate arrays.
__global__ void __launch_bounds__(256) peer_unpack_rows_kernel(RowArrays a, long long cap, const int64_t *nnz_recv,
                                                             const int64_t *__restrict__ route,
                                                             const int64_t *__restrict__ n_world, int cams_per_rank,
                                                             long long cap_recv, PeerView v, int buf) {
    __shared__ long long s_prefix[kMaxPeers + 1];
    __shared__ long long s_region[kMaxPeers];
    if (threadIdx.x <= (unsigned)v.world) s_prefix[threadIdx.x] = route[threadIdx.x];
    if (threadIdx.x < (unsigned)v.world) s_region[threadIdx.x] = region_start(n_world, cams_per_rank, threadIdx.x);
    __syncthreads();
    long long rows = *nnz_recv < cap ? *nnz_recv : cap;
    const uint32_t *buf_base = reinterpret_cast<const uint32_t *>(v.arena[v.rank] + v.recv_offset + buf * v.recv_stride);
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < rows;
         i += (long long)gridDim.x * blockDim.x) {
        int r = 0;
        while (r + 1 < v.world && i >= s_prefix[r + 1]) ++r;
        const long long slot = s_region[r] + (i - s_prefix[r]);
        if (slot >= cap_recv) continue;
        const uint32_t *src = buf_base + slot * a.total;
        for (int j = 0; j < a.n; ++j) {
            const int w = a.words[j];
            uint32_t *dst = static_cast<uint32_t *>(a.ptr[j]);
            if (dst) {
                dst += i * w;
                for (int k = 0; k < w; ++k) dst[k] = src[k];
            }
            src += w;
        }
    }
}

// After the unpack (stream order): tell every source its rows were read.
__global__ void peer_signal_consumed_kernel(PeerView v, unsigned long long epoch) {
    const int d = threadIdx.x;
    if (d >= v.world) return;
    store_release_sys(&mailbox(v, d)->consumed_flag[v.rank], epoch);
}

// Gradients of the received rows back to their sources: received row i of
// source r is r's local row rows_first[r] + (i - prefix[r]); its gradient row
// goes to that row of r's gradient buffer. Staged like peer_send_rows_kernel.
__global__ void __launch_bounds__(kRowThreads) peer_send_grads_kernel(RowArrays a, long long cap,
                                                                    const int64_t *nnz_recv,
                                                                    const int64_t *__restrict__ route,
                                                                    long long cap_grad, PeerView v,
                                                                    unsigned long long epoch) {
    __shared__ uint32_t stage[kPeerStageWords];
    __shared__ long long s_prefix[kMaxPeers + 1];
    __shared__ long long s_first[kMaxPeers];
    __shared__ bool s_last;
    PeerMailbox *me = mailbox(v, v.rank);
    if (threadIdx.x <= (unsigned)v.world) s_prefix[threadIdx.x] = route[threadIdx.x];
    if (threadIdx.x < (unsigned)v.world) s_first[threadIdx.x] = route[v.world + 1 + threadIdx.x];
    __syncthreads();
    const long long rows = *nnz_recv < cap ? *nnz_recv : cap;
    const int S = stage_stride(a.total);
    const int R = peer_block_rows(a.total);
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
        for (int i = threadIdx.x; i < nr * a.total; i += kRowThreads) {
            const int r = i / a.total, k = i - r * a.total;
            const long long row = r0 + r;
            int src = 0;
            while (src + 1 < v.world && row >= s_prefix[src + 1]) ++src;
            const long long slot = s_first[src] + (row - s_prefix[src]);
            if (slot < cap_grad) {
                uint32_t *dst = reinterpret_cast<uint32_t *>(v.arena[src] + v.grad_offset);
                dst[slot * a.total + k] = stage[r * S + k];
            }
        }
        __syncthreads();
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(&me->done_ctas_grad, 1u) == gridDim.x - 1;
    __syncthreads();
    if (s_last && threadIdx.x < (unsigned)v.world) {
        __threadfence_system();
        store_release_sys(&mailbox(v, threadIdx.x)->grad_flag[v.rank], epoch);
        if (threadIdx.x == 0) me->done_ctas_grad = 0u;
    }
}

__global__ void peer_wait_grads_kernel(PeerView v, unsigned long long epoch) {
    const int d = threadIdx.x;
    if (d >= v.world) return;
    wait_flag(&mailbox(v, v.rank)->grad_flag[d], epoch, v.error, 3, v.wait_limit);
}

static int make_view(PeerView &v, const GsbPeerGroup *g) {
    if (g == nullptr || g->world < 1 || g->world > kMaxPeers || g->rank < 0 || g->rank >= g->world)
        return set_error(kErrInvalidArgument, "peer group: bad rank / world");
    for (int r = 0; r < g->world; ++r) {
        if (g->arena[r] == nullptr) return set_error(kErrInvalidArgument, "peer group: arena %d not mapped", r);
        v.arena[r] = static_cast<char *>(g->arena[r]);
    }
    v.recv_offset = g->recv_offset;
    v.recv_stride = g->recv_stride;
    v.grad_offset = g->grad_offset;
    v.rank = g->rank;
    v.world = g->world;
    v.error = g->error;
    v.wait_limit = g_wait_limit.load();
    if (v.error == nullptr) return set_error(kErrInvalidArgument, "peer group: no error word");
    return kOk;
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

extern "C" int gsb_unpack_rows(long long rows, const int64_t *rows_device, int row_words, const uint32_t *buf,
                               int n_arrays, void *const *dsts, const int *words, cudaStream_t stream) {
    RowArrays a;
    if (int e = make_arrays(a, n_arrays, dsts, words)) return e;
    if (a.total > row_words)
        return set_error(kErrInvalidArgument, "row unpacking: %d words requested from rows of %d", a.total,
                         row_words);
    if (rows <= 0) return kOk;
    unpack_rows_kernel<<<grid_for(rows), 256, 0, stream>>>(a, rows, rows_device, row_words, buf);
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

// ---- peer-memory exchange ---------------------------------------------------

extern "C" size_t gsb_peer_mailbox_bytes(void) { return (size_t)kMailboxBytes; }

extern "C" long long gsb_peer_set_wait_limit(long long polls) {
    const long long prev = g_wait_limit.load();
    g_wait_limit.store(polls > 0 ? polls : kSpinLimit);
    return prev;
}

extern "C" int gsb_peer_alloc(size_t bytes, void **ptr, void *ipc_handle) {
    if (ptr == nullptr || ipc_handle == nullptr || bytes == 0) return set_error(kErrInvalidArgument, "peer alloc");
    void *p = nullptr;
    cudaError_t ce = cudaMalloc(&p, bytes);
    if (ce != cudaSuccess) return set_error(kErrLaunch, "cudaMalloc(%zu): %s", bytes, cudaGetErrorString(ce));
    ce = cudaMemset(p, 0, bytes);
    if (ce == cudaSuccess) ce = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t *>(ipc_handle), p);
    if (ce != cudaSuccess) {
        cudaFree(p);
        return set_error(kErrLaunch, "peer arena: %s", cudaGetErrorString(ce));
    }
    *ptr = p;
    return kOk;
}

extern "C" int gsb_peer_open(const void *ipc_handle, void **ptr) {
    if (ipc_handle == nullptr || ptr == nullptr) return set_error(kErrInvalidArgument, "peer open");
    cudaIpcMemHandle_t h;
    memcpy(&h, ipc_handle, sizeof(h));
    const cudaError_t ce = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (ce != cudaSuccess) return set_error(kErrLaunch, "cudaIpcOpenMemHandle: %s", cudaGetErrorString(ce));
    return kOk;
}

extern "C" int gsb_peer_close(void *ptr) {
    const cudaError_t ce = cudaIpcCloseMemHandle(ptr);
    if (ce != cudaSuccess) return set_error(kErrLaunch, "cudaIpcCloseMemHandle: %s", cudaGetErrorString(ce));
    return kOk;
}

extern "C" int gsb_peer_free(void *ptr) {
    const cudaError_t ce = cudaFree(ptr);
    if (ce != cudaSuccess) return set_error(kErrLaunch, "cudaFree: %s", cudaGetErrorString(ce));
    return kOk;
}

extern "C" int gsb_peer_error_alloc(int **host_ptr, int **device_ptr) {
    if (host_ptr == nullptr || device_ptr == nullptr) return set_error(kErrInvalidArgument, "peer error word");
    void *h = nullptr;
    cudaError_t ce = cudaHostAlloc(&h, sizeof(int), cudaHostAllocMapped);
    if (ce != cudaSuccess) return set_error(kErrLaunch, "cudaHostAlloc: %s", cudaGetErrorString(ce));
    *static_cast<int *>(h) = 0;
    void *d = nullptr;
    ce = cudaHostGetDevicePointer(&d, h, 0);
    if (ce != cudaSuccess) {
        cudaFreeHost(h);
        return set_error(kErrLaunch, "cudaHostGetDevicePointer: %s", cudaGetErrorString(ce));
    }
    *host_ptr = static_cast<int *>(h);
    *device_ptr = static_cast<int *>(d);
    return kOk;
}

extern "C" int gsb_peer_error_free(int *host_ptr) {
    const cudaError_t ce = cudaFreeHost(host_ptr);
    if (ce != cudaSuccess) return set_error(kErrLaunch, "cudaFreeHost: %s", cudaGetErrorString(ce));
    return kOk;
}

extern "C" int gsb_peer_send_rows(const GsbPeerGroup *g, unsigned long long epoch, long long cap_rows,
                                  const int64_t *nnz_device, const int64_t *bounds, const int64_t *n_world,
                                  int cams_per_rank, long long cap_recv, int n_arrays, void *const *srcs,
                                  const int *words, cudaStream_t stream) {
    PeerView v;
    if (int e = make_view(v, g)) return e;
    RowArrays a;
    if (int e = make_arrays(a, n_arrays, srcs, words)) return e;
    if (cap_rows < 0 || cams_per_rank <= 0 || epoch == 0) return set_error(kErrInvalidArgument, "peer send rows");
    if ((a.total | 1) > kPeerStageWords)
        return set_error(kErrInvalidArgument, "peer rows of %d words (at most %d)", a.total, kPeerStageWords - 1);
    peer_wait_consumed_kernel<<<1, 32, 0, stream>>>(v, epoch);
    if (int e = check_launch("peer_wait_consumed_kernel")) return e;
    peer_send_rows_kernel<<<grid_for_rows(cap_rows, a.total), kRowThreads, 0, stream>>>(
        a, cap_rows, nnz_device, bounds, n_world, cams_per_rank, cap_recv, v, epoch, (int)(epoch & 1));
    return check_launch("peer_send_rows_kernel");
}

extern "C" int gsb_peer_recv_rows(const GsbPeerGroup *g, unsigned long long epoch, long long cap_rows,
                                  int64_t *route, int64_t *nnz_recv, const int64_t *n_world, int cams_per_rank,
                                  long long cap_recv, int n_arrays, void *const *dsts, const int *words,
                                  cudaStream_t stream) {
    PeerView v;
    if (int e = make_view(v, g)) return e;
    RowArrays a;
    if (int e = make_arrays(a, n_arrays, dsts, words)) return e;
    if (cap_rows < 0 || cams_per_rank <= 0 || epoch == 0) return set_error(kErrInvalidArgument, "peer recv rows");
    peer_wait_rows_kernel<<<1, 32, 0, stream>>>(v, epoch, route, nnz_recv);
    if (int e = check_launch("peer_wait_rows_kernel")) return e;
    peer_unpack_rows_kernel<<<grid_for(cap_rows), 256, 0, stream>>>(a, cap_rows, nnz_recv, route, n_world,
                                                                    cams_per_rank, cap_recv, v, (int)(epoch & 1));
    if (int e = check_launch("peer_unpack_rows_kernel")) return e;
    peer_signal_consumed_kernel<<<1, 32, 0, stream>>>(v, epoch);
    return check_launch("peer_signal_consumed_kernel");
}

extern "C" int gsb_peer_send_grads(const GsbPeerGroup *g, unsigned long long epoch, long long cap_rows,
                                   const int64_t *nnz_recv, const int64_t *route, long long cap_grad, int n_arrays,
                                   void *const *srcs, const int *words, cudaStream_t stream) {
    PeerView v;
    if (int e = make_view(v, g)) return e;
    RowArrays a;
    if (int e = make_arrays(a, n_arrays, srcs, words)) return e;
    if (cap_rows < 0 || epoch == 0) return set_error(kErrInvalidArgument, "peer send grads");
    if ((a.total | 1) > kPeerStageWords)
        return set_error(kErrInvalidArgument, "peer rows of %d words (at most %d)", a.total, kPeerStageWords - 1);
    peer_send_grads_kernel<<<grid_for_rows(cap_rows, a.total), kRowThreads, 0, stream>>>(a, cap_rows, nnz_recv,
                                                                                        route, cap_grad, v, epoch);
    return check_launch("peer_send_grads_kernel");
}

extern "C" int gsb_peer_recv_grads(const GsbPeerGroup *g, unsigned long long epoch, long long cap_rows,
                                   const int64_t *nnz_device, int n_arrays, void *const *dsts, const int *words,
                                   cudaStream_t stream) {
    PeerView v;
    if (int e = make_view(v, g)) return e;
    RowArrays a;
    if (int e = make_arrays(a, n_arrays, dsts, words)) return e;
    if (cap_rows < 0 || epoch == 0) return set_error(kErrInvalidArgument, "peer recv grads");
    peer_wait_grads_kernel<<<1, 32, 0, stream>>>(v, epoch);
    if (int e = check_launch("peer_wait_grads_kernel")) return e;
    if (cap_rows == 0) return kOk;
    const uint32_t *buf = reinterpret_cast<const uint32_t *>(static_cast<char *>(g->arena[g->rank]) + g->grad_offset);
    unpack_rows_kernel<<<grid_for(cap_rows), 256, 0, stream>>>(a, cap_rows, nnz_device, a.total, buf);
    return check_launch("unpack_rows_kernel");
}
