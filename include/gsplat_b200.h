/*
 * gsplat_b200 C ABI: the drop-in boundary of the Gaussian-splatting training hot
 * path (projection, spherical harmonics, tile intersection + sort + offsets,
 * rasterization, selective Adam) for NVIDIA B200 (sm_100a).
 *
 * Conventions
 *  - All tensors are device pointers to contiguous row-major fp32 / int32 / int64
 *    arrays; the caller allocates every output and scratch buffer. The compute
 *    entry points never allocate device memory. The exceptions are the set-up
 *    calls of the peer-memory exchange: gsb_peer_alloc allocates the calling
 *    rank's exchange arena (cudaMalloc) and gsb_peer_error_alloc a host-mapped
 *    error word (cudaHostAlloc); gsb_peer_free / gsb_peer_error_free release
 *    them. Optional inputs and outputs are NULL.
 *  - Every function launches asynchronously on `stream` and returns 0 on success
 *    or a negative status (-1 invalid argument, -2 unsupported, -3 launch error);
 *    gsb_last_error() returns the message of the calling thread's last error.
 *  - Functions hold no state between calls and may be called from several
 *    threads, with these exceptions: gsb_isect_bucket_sort runs its larger
 *    bucket classes on one internal side stream per device (created on first
 *    use, forked from and joined back to `stream` with events; calls on one
 *    device are serialised on it by a mutex); gsb_inclusive_scan_i32_noalloc
 *    keeps its tile sums in one static device array per device (documented
 *    there). Call every function with the device that owns the pointers current.
 *  - Outputs documented as "zero-initialised by the caller" are accumulated into
 *    with atomics, matching the reference's at::zeros allocations.
 *
 * Each entry point names the reference interface it replaces (paths relative to
 * the mc8max/gsplat source tree).
 */
#ifndef GSPLAT_B200_H_
#define GSPLAT_B200_H_

#include <stddef.h>
#include <stdint.h>
#include <stdbool.h>
#include <cuda_runtime.h>

#if defined(_WIN32)
#define GSB_API __declspec(dllexport)
#else
#define GSB_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

GSB_API const char *gsb_last_error(void);
GSB_API int gsb_version(void);

/* --- Projection -----------------------------------------------------------
 * Replaces torch op gsplat::projection_ewa_3dgs_fused_fwd
 * (gsplat/cuda/ext.cpp:716; gsplat/cuda/csrc/Projection.cpp:129-214).
 * means [B,N,3]; covars [B,N,6] or quats [B,N,4] + scales [B,N,3];
 * opacities [B,N] (optional: opacity-aware radius); viewmats [B,C,4,4];
 * Ks [B,C,3,3]. Outputs [B,C,N,...]: radii int32 x2, means2d x2, depths,
 * conics x3, compensations (only when calc_compensations). Culled entries are
 * written as zeros. camera_model: 0 pinhole, 1 ortho, 2 fisheye. */
GSB_API int gsb_projection_fused_fwd(int B, int C, int N, const float *means, const float *covars,
                             const float *quats, const float *scales, const float *opacities,
                             const float *viewmats, const float *Ks, int width, int height,
                             float eps2d, float near_plane, float far_plane, float radius_clip,
                             int calc_compensations, int camera_model, int32_t *radii,
                             float *means2d, float *depths, float *conics, float *compensations,
                             cudaStream_t stream);

/* Replaces gsplat::projection_ewa_3dgs_fused_bwd (Projection.cpp:216-306).
 * Writes v_means [B,N,3], v_quats [B,N,4] + v_scales [B,N,3] (or v_covars
 * [B,N,6]) completely (no pre-zeroing needed). v_viewmats [B,C,4,4] is
 * accumulated and must be zero-initialised by the caller (NULL to skip). */
GSB_API int gsb_projection_fused_bwd(int B, int C, int N, const float *means, const float *covars,
                             const float *quats, const float *scales, const float *viewmats,
                             const float *Ks, int width, int height, float eps2d, int camera_model,
                             const int32_t *radii, const float *conics, const float *compensations,
                             const float *v_means2d, const float *v_depths, const float *v_conics,
                             const float *v_compensations, float *v_means, float *v_covars,
                             float *v_quats, float *v_scales, float *v_viewmats,
                             cudaStream_t stream);

/* Packed (COO) projection, replaces gsplat::projection_ewa_3dgs_packed_fwd
 * (Projection.cpp:308-460), as a two-call protocol equal to the reference's
 * count pass + cumsum + .item() + write pass:
 *   1. gsb_projection_packed_count -> block_cnts int32 [B*C*blocks] and the
 *      visibility ballots vis_bits uint32 [B*C*blocks*8], blocks =
 *      gsb_projection_packed_blocks(N);
 *   2. gsb_inclusive_scan_i32(block_cnts) -> block_accum int64; nnz = last entry;
 *   3. gsb_projection_packed_write with the same vis_bits, nnz, outputs of
 *      length nnz and indptr [B*C+1]. Pass 2 places exactly the pairs pass 1
 *      marked, so the two passes cannot disagree.
 * Pairs are ordered by (batch, camera) then Gaussian id. */
GSB_API int gsb_projection_packed_blocks(int N);
GSB_API int gsb_projection_packed_count(int B, int C, int N, const float *means, const float *covars,
                                const float *quats, const float *scales, const float *opacities,
                                const float *viewmats, const float *Ks, int width, int height,
                                float eps2d, float near_plane, float far_plane, float radius_clip,
                                int calc_compensations, int camera_model, int32_t *block_cnts,
                                uint32_t *vis_bits, cudaStream_t stream);
GSB_API int gsb_projection_packed_write(int B, int C, int N, const float *means, const float *covars,
                                const float *quats, const float *scales, const float *opacities,
                                const float *viewmats, const float *Ks, int width, int height,
                                float eps2d, float near_plane, float far_plane, float radius_clip,
                                int calc_compensations, int camera_model,
                                const uint32_t *vis_bits, const int64_t *block_accum,
                                long long nnz, int32_t *indptr,
                                int64_t *batch_ids,
                                int64_t *camera_ids, int64_t *gaussian_ids, int32_t *radii,
                                float *means2d, float *depths, float *conics,
                                float *compensations, cudaStream_t stream);

/* Replaces gsplat::projection_ewa_3dgs_packed_bwd (Projection.cpp:462-575).
 * sparse_grad = 0: v_means/v_quats/v_scales/v_covars are dense [B,N,...] and
 * must be zero-initialised (accumulated with atomics); sparse_grad = 1: they are
 * [nnz,...] and written per pair. v_viewmats as in gsb_projection_fused_bwd. */
GSB_API int gsb_projection_packed_bwd(int B, int C, int N, int nnz, const float *means,
                              const float *covars, const float *quats, const float *scales,
                              const float *viewmats, const float *Ks, int width, int height,
                              float eps2d, int camera_model, const int64_t *batch_ids,
                              const int64_t *camera_ids, const int64_t *gaussian_ids,
                              const float *conics, const float *compensations,
                              const float *v_means2d, const float *v_depths,
                              const float *v_conics, const float *v_compensations,
                              int sparse_grad, float *v_means, float *v_covars, float *v_quats,
                              float *v_scales, float *v_viewmats, cudaStream_t stream);

/* --- Covariances and simple projection -----------------------------------
 * gsb_quat_scale_to_covar_preci_fwd / _bwd replace the torch ops
 * gsplat::quat_scale_to_covar_preci_fwd / _bwd (gsplat/cuda/ext.cpp:712-713;
 * gsplat/cuda/csrc/QuatScaleToCovar.cpp:39-106). quats [n,4] (any norm),
 * scales [n,3]; covars / precis [n,6] (triu: xx xy xz yy yz zz) or [n,3,3], each
 * optional (NULL = not computed). Backward: v_covars / v_precis optional
 * upstream gradients in the same layout (triu off-diagonals count once, as the
 * reference halves them); writes v_quats [n,4], v_scales [n,3].
 *
 * gsb_proj_fwd / _bwd replace gsplat::projection_ewa_simple_fwd / _bwd
 * (ext.cpp:726-727; Projection.cpp:41-127): camera-space means [B,C,N,3],
 * covars [B,C,N,3,3], Ks [B,C,3,3] -> means2d [B,C,N,2], covars2d [B,C,N,2,2]
 * (row-major); backward: v_means2d, v_covars2d -> v_means [B,C,N,3],
 * v_covars [B,C,N,3,3]. camera_model: 0 pinhole, 1 ortho, 2 fisheye. */
GSB_API int gsb_quat_scale_to_covar_preci_fwd(long long n, const float *quats, const float *scales, int triu,
                                              float *covars, float *precis, cudaStream_t stream);
GSB_API int gsb_quat_scale_to_covar_preci_bwd(long long n, const float *quats, const float *scales, int triu,
                                              const float *v_covars, const float *v_precis, float *v_quats,
                                              float *v_scales, cudaStream_t stream);
GSB_API int gsb_proj_fwd(int B, int C, int N, const float *means, const float *covars, const float *Ks,
                         int width, int height, int camera_model, float *means2d, float *covars2d,
                         cudaStream_t stream);
GSB_API int gsb_proj_bwd(int B, int C, int N, const float *means, const float *covars, const float *Ks,
                         int width, int height, int camera_model, const float *v_means2d,
                         const float *v_covars2d, float *v_means, float *v_covars, cudaStream_t stream);

/* --- Fused projection + SH (no reference counterpart as one op) -----------
 * The reference's rasterization() runs projection, view directions, SH and the
 * colour clamp as separate ops (gsplat/rendering.py:749-872). These entry points
 * do all of it per (camera, Gaussian): besides the projection outputs they write
 * colors = max(SH(normalize(mean - campos)) + 0.5, 0) [.,3] and opacities_out =
 * opacities * compensations (antialiased) or opacities [.]. sh is the
 * per-Gaussian coefficient tensor [B,N,K,3] (K <= 64, degree <= 4).
 * Packed: pass 1 is gsb_projection_packed_count; pair_index int32 [B*C*N]
 * (optional) receives each pair's packed position or -1 for the backward. */
GSB_API int gsb_projection_sh_dense_fwd(int B, int C, int N, const float *means,
                                        const float *quats, const float *scales,
                                        const float *opacities, const float *sh, int K,
                                        int sh_degree, const float *viewmats, const float *Ks,
                                        int width, int height, float eps2d, float near_plane,
                                        float far_plane, float radius_clip, int calc_compensations,
                                        int camera_model, int32_t *radii, float *means2d,
                                        float *depths, float *conics, float *compensations,
                                        float *colors, float *opacities_out, cudaStream_t stream);
GSB_API int gsb_projection_sh_packed_write(
    int B, int C, int N, const float *means, const float *quats, const float *scales,
    const float *opacities, const float *sh, int K, int sh_degree, const float *viewmats,
    const float *Ks, int width, int height, float eps2d, float near_plane, float far_plane,
    float radius_clip, int calc_compensations, int camera_model, const uint32_t *vis_bits,
    const int64_t *block_accum, long long nnz, int32_t *indptr, int64_t *batch_ids,
    int64_t *camera_ids, int64_t *gaussian_ids, int32_t *radii, float *means2d, float *depths,
    float *conics, float *compensations, float *colors, float *opacities_out, int32_t *pair_index,
    cudaStream_t stream);
/* Backward of both layouts. Writes every row of v_means [B,N,3], v_quats
 * [B,N,4], v_scales [B,N,3], v_opacities [B,N] and v_sh [B,N,K,3] (no
 * pre-zeroing). packed: pair_index from the forward; dense: radii [B,C,N,2].
 * Upstream gradients are indexed like the forward outputs; v_depths and
 * v_compensations may be NULL (no gradient). */
GSB_API int gsb_projection_sh_bwd(
    int B, int C, int N, int packed, const float *means, const float *quats, const float *scales,
    const float *opacities, const float *sh, int K, int sh_degree, const float *viewmats,
    const float *Ks, int width, int height, float eps2d, int calc_compensations, int camera_model,
    const int32_t *pair_index, const int32_t *radii, const float *conics,
    const float *compensations, const float *v_means2d, const float *v_depths,
    const float *v_conics, const float *v_compensations, const float *v_colors,
    const float *v_opacities_out, float *v_means, float *v_quats, float *v_scales,
    float *v_opacities, float *v_sh, cudaStream_t stream);

/* --- Spherical harmonics --------------------------------------------------
 * Replaces gsplat::spherical_harmonics_fwd / _bwd
 * (gsplat/cuda/csrc/SphericalHarmonics.cpp:32-93). dirs [n,3] (normalised
 * inside), coeffs [n,K,3], masks [n] (optional) -> colors [n,3]; masked
 * elements get 0. Backward writes v_coeffs [n,K,3] completely and, when
 * v_dirs != NULL, v_dirs [n,3]. degree in [0,4], K <= 64. */
GSB_API int gsb_spherical_harmonics_fwd(int degree, long long n, int K, const float *dirs,
                                const float *coeffs, const bool *masks, float *colors,
                                cudaStream_t stream);
GSB_API int gsb_spherical_harmonics_bwd(int degree, long long n, int K, const float *dirs,
                                const float *coeffs, const bool *masks, const float *v_colors,
                                float *v_coeffs, float *v_dirs, cudaStream_t stream);

/* --- Prefix sum -----------------------------------------------------------
 * Inclusive int32 -> int64 scan (replaces the at::cumsum of Intersect.cpp:100).
 * scratch: device buffer of gsb_scan_scratch_bytes(n) bytes. */
GSB_API size_t gsb_scan_scratch_bytes(long long n);
GSB_API int gsb_inclusive_scan_i32(const int32_t *in, int64_t *out, long long n, void *scratch,
                           size_t scratch_bytes, cudaStream_t stream);

/* Allocation-free inclusive scan. No counterpart in the reference: it exists for
 * callers that may not allocate device memory where they need the scan, e.g.
 * code running inside a host application that owns all device memory itself, or
 * inside an allocator's callbacks. Same result as gsb_inclusive_scan_i32, but the
 * scratch is a static 512 KiB device array inside this library (held on every
 * GPU that loads it), so n is limited to 2^27 values; larger n returns -1 with a
 * message. The library itself calls no cudaMalloc/cudaFree here. The first call
 * on a device looks the array's device address up (cudaGetSymbolAddress), so make
 * that first call before any stream capture. All calls on a device share the
 * array: calls that overlap on the GPU (unordered streams) race on it. */
GSB_API int gsb_inclusive_scan_i32_noalloc(const int32_t *in, int64_t *out, long long n,
                                           cudaStream_t stream);

/* --- Tile intersection ----------------------------------------------------
 * Replaces gsplat::intersect_tile (Intersect.cpp:33-176) as count -> scan ->
 * emit -> sort. Dense: means2d [I,N,2], radii [I,N,2], depths [I,N] (packed=0).
 * Packed: [nnz,...] plus image_ids int64 [nnz]. conics [.,3] + opacities [.]
 * select the AccuTile ellipse test, else the AABB of radii is used.
 * tiles_per_gauss int32 [I*N or nnz]. Keys: image << (32+tile_bits) |
 * tile << 32 | float_bits(depth); gsb_isect_key_bits() = 32+tile_bits+image_bits. */
GSB_API int gsb_isect_key_bits(int I, int tile_width, int tile_height);
GSB_API int gsb_isect_count(int packed, int I, int N, int nnz, const int64_t *image_ids,
                    const float *means2d, const int32_t *radii, const float *depths,
                    const float *conics, const float *opacities, int tile_size, int tile_width,
                    int tile_height, int32_t *tiles_per_gauss, cudaStream_t stream);
GSB_API int gsb_isect_emit(int packed, int I, int N, int nnz, const int64_t *image_ids,
                   const float *means2d, const int32_t *radii, const float *depths,
                   const float *conics, const float *opacities, int tile_size, int tile_width,
                   int tile_height, const int64_t *cum_tiles_per_gauss, int64_t *isect_ids,
                   int32_t *flatten_ids, cudaStream_t stream);

/* Stable radix sort of (int64 key, int32 value) pairs on bits [0, end_bit);
 * replaces cub::DeviceRadixSort::SortPairs (IntersectTile.cu:478-521). Keys must
 * be non-negative. Ping-pongs between (keys, vals) and (keys_alt, vals_alt);
 * returns 0 if the result is in (keys, vals), 1 if in the alternates, <0 on
 * error. scratch: gsb_radix_sort_scratch_bytes(n) bytes. */
GSB_API size_t gsb_radix_sort_scratch_bytes(long long n);
GSB_API int gsb_radix_sort_pairs(int64_t *keys, int32_t *vals, int64_t *keys_alt, int32_t *vals_alt,
                         long long n, int end_bit, void *scratch, size_t scratch_bytes,
                         cudaStream_t stream);

/* Replaces gsplat::intersect_offset (Intersect.cpp:320-337): offsets int32
 * [I, tile_height, tile_width] = index of the first sorted key of each tile
 * (n_isects for tiles after the last key, 0 everywhere when n_isects == 0). */
GSB_API int gsb_isect_offset_encode(const int64_t *isect_ids, long long n_isects, int I, int tile_width,
                            int tile_height, int32_t *offsets, cudaStream_t stream);

/* --- Tile-bucket path for the sorted intersection list --------------------
 * Produces the same (isect_ids, flatten_ids, offsets) as gsb_isect_count +
 * gsb_inclusive_scan_i32 + gsb_isect_emit + gsb_radix_sort_pairs +
 * gsb_isect_offset_encode -- the reference's intersect_tile(sort=true) followed
 * by intersect_offset (Intersect.cpp:33-176, 320-337) -- bit for bit, without a
 * global sort: entries are scattered into their (image, tile) bucket and each
 * bucket is sorted by (depth bits, splat index) on chip. Buckets are numbered
 * image * tile_width * tile_height + tile; each bucket has S =
 * gsb_isect_bucket_shards(I, tile_width, tile_height) counters, one per shard
 * of splats (contiguous splat ranges handled by one CTA each when the buckets
 * fit in shared memory, else GSB_ISECT_BUCKET_SHARDS shards idx % 16 in
 * global memory).
 *
 * 1. gsb_isect_count_tiles: tiles_per_gauss as gsb_isect_count, plus
 *    shard_counts int32 [n_buckets * S] (all written by the call). Packed
 *    only: with nnz_device (device int64, may be NULL) the splat count is read
 *    on the device and nnz is the capacity of the arrays, so the caller need
 *    not read the count back after the projection. */
#define GSB_ISECT_BUCKET_SHARDS 16
GSB_API int gsb_isect_bucket_shards(int I, int tile_width, int tile_height);
GSB_API int gsb_isect_count_tiles(int packed, int I, int N, int nnz, const int64_t *image_ids,
                                  const float *means2d, const int32_t *radii, const float *depths,
                                  const float *conics, const float *opacities, int tile_size,
                                  int tile_width, int tile_height, const int64_t *nnz_device,
                                  int32_t *tiles_per_gauss, int32_t *shard_counts, cudaStream_t stream);
/* 2. offsets int32 [n_buckets] (= gsb_isect_offset_encode's output),
 *    bucket_sizes int32 [n_buckets], the emit cursor int32 [n_buckets * S],
 *    totals int32 [5] = {n_isects (-1 if above 2^31 - 1), largest bucket,
 *    *nnz_device (0 when nnz_device is NULL), buckets with 1024 < size <= 4096,
 *    buckets with size > 4096}, all device memory, so one copy brings every
 *    size the host needs, and class_list int32 [n_buckets]: the ids of the
 *    buckets with 1024 < size <= 4096 in its first totals[3] entries, of those
 *    above 4096 in its last totals[4] entries (in no particular order); scratch
 *    of gsb_isect_bucket_offsets_scratch_bytes(n_buckets, S). */
GSB_API size_t gsb_isect_bucket_offsets_scratch_bytes(long long n_buckets, int shards);
GSB_API int gsb_isect_bucket_offsets(const int32_t *shard_counts, long long n_buckets, int shards,
                                     int32_t *offsets, int32_t *bucket_sizes, int32_t *cursor,
                                     const int64_t *nnz_device, int32_t *totals, int32_t *class_list,
                                     void *scratch, size_t scratch_bytes, cudaStream_t stream);
/* 3. Scatter every intersection into its bucket as one entry uint64
 *    (depth bits << 32 | splat index) of bucket_entries [n_isects] (unordered
 *    inside the bucket); n_isects = totals[0] of step 2. */
GSB_API int gsb_isect_bucket_emit(int packed, int I, int N, int nnz, const int64_t *image_ids,
                                  const float *means2d, const int32_t *radii, const float *depths,
                                  const float *conics, const float *opacities, int tile_size,
                                  int tile_width, int tile_height, long long n_isects, int32_t *cursor,
                                  uint64_t *bucket_entries, cudaStream_t stream);
/* 4. Sort every bucket and write isect_ids int64 / flatten_ids int32
 *    [n_isects]. max_count (totals[1] of step 2) must not exceed
 *    gsb_isect_bucket_sort_max(); larger buckets take gsb_isect_bucket_sort_ex.
 *    mid_buckets / large_buckets / class_list: totals[3] / totals[4] and the
 *    class list of step 2 (every bucket is sorted by a radix sort in shared
 *    memory, one CTA per bucket; buckets above 1024 entries by larger CTAs
 *    walking the list). */
GSB_API int gsb_isect_bucket_sort_max(void);
GSB_API int gsb_isect_bucket_sort(int I, int tile_width, int tile_height, const int32_t *offsets,
                                  const int32_t *bucket_sizes, int max_count, int mid_buckets,
                                  int large_buckets, const int32_t *class_list, const uint64_t *bucket_entries,
                                  int64_t *isect_ids, int32_t *flatten_ids, cudaStream_t stream);
/* Same as gsb_isect_bucket_sort, also for buckets above gsb_isect_bucket_sort_max()
 * entries: each is split on the device into sub-buckets of its leading (depth,
 * splat index) bits, which then take the on-chip sorts. scratch:
 * gsb_isect_bucket_sort_scratch_bytes(n_isects) bytes (used only when
 * max_count is above the on-chip maximum). overflow (device int32, written on
 * that path only) is set to 1 when a sub-bucket is still above the on-chip
 * maximum (more entries with the same depth than fit on chip): the outputs are
 * then incomplete and the caller sorts with the global path (gsb_isect_emit +
 * gsb_radix_sort_pairs). Together they replace the cub radix sort of
 * IntersectTile.cu:478-521 for such buckets. */
GSB_API size_t gsb_isect_bucket_sort_scratch_bytes(long long n_isects);
GSB_API int gsb_isect_bucket_sort_ex(int I, int tile_width, int tile_height, const int32_t *offsets,
                                     const int32_t *bucket_sizes, int max_count, int mid_buckets,
                                     int large_buckets, const int32_t *class_list,
                                     const uint64_t *bucket_entries, long long n_isects, void *scratch,
                                     size_t scratch_bytes, int *overflow, int64_t *isect_ids,
                                     int32_t *flatten_ids, cudaStream_t stream);

/* --- Rasterization --------------------------------------------------------
 * Replaces gsplat::rasterize_to_pixels_3dgs_fwd (Rasterization.cpp:42-119).
 * means2d [.,2], conics [.,3], colors [.,channels], opacities [.] indexed by
 * flatten_ids; backgrounds [I,channels] and masks [I,th,tw] optional.
 * Outputs renders [I,H,W,channels], alphas [I,H,W], last_ids int32 [I,H,W].
 * Any channel count >= 1 is accepted; tile_size in [1,16]. */
GSB_API int gsb_rasterize_fwd(int I, int channels, const float *means2d, const float *conics,
                      const float *colors, const float *opacities, const float *backgrounds,
                      const bool *masks, int width, int height, int tile_size, int tile_width,
                      int tile_height, const int32_t *tile_offsets, const int32_t *flatten_ids,
                      long long n_isects, float *renders, float *alphas, int32_t *last_ids,
                      cudaStream_t stream);

/* Same as gsb_rasterize_fwd and additionally writes pair_counts int32 [I,H,W], the
 * number of splats that contributed to each pixel (alpha >= 1/255 before the
 * transmittance cut-off). No reference counterpart; used to count the
 * algorithmic work of the rasterizer for its roofline. */
GSB_API int gsb_rasterize_fwd_counted(int I, int channels, const float *means2d,
                                      const float *conics, const float *colors,
                                      const float *opacities, const float *backgrounds,
                                      const bool *masks, int width, int height, int tile_size,
                                      int tile_width, int tile_height, const int32_t *tile_offsets,
                                      const int32_t *flatten_ids, long long n_isects,
                                      float *renders, float *alphas, int32_t *last_ids,
                                      int32_t *pair_counts, cudaStream_t stream);

/* Replaces gsplat::rasterize_to_pixels_3dgs_bwd (Rasterization.cpp:121-214).
 * v_means2d, v_conics, v_colors, v_opacities and v_means2d_abs (optional,
 * absgrad) are accumulated: zero-initialise them. */
GSB_API int gsb_rasterize_bwd(int I, int channels, const float *means2d, const float *conics,
                      const float *colors, const float *opacities, const float *backgrounds,
                      const bool *masks, int width, int height, int tile_size, int tile_width,
                      int tile_height, const int32_t *tile_offsets, const int32_t *flatten_ids,
                      long long n_isects, const float *render_alphas, const int32_t *last_ids,
                      const float *v_render_colors, const float *v_render_alphas,
                      float *v_means2d_abs, float *v_means2d, float *v_conics, float *v_colors,
                      float *v_opacities, cudaStream_t stream);

/* Same as gsb_rasterize_fwd, and optionally writes final_Ts float [I,H,W], the
 * final transmittance of each pixel as the forward computed it (render_alphas is
 * 1 - final_Ts rounded once), and pair_counts int32 [I,H,W] (see
 * gsb_rasterize_fwd_counted). Either may be NULL. The forward half of the pair
 * behind gsplat::rasterize_to_pixels_3dgs_fwd (Rasterization.cpp:42-119) that
 * keeps the transmittance for the backward. */
GSB_API int gsb_rasterize_fwd_ex(int I, int channels, const float *means2d, const float *conics,
                                 const float *colors, const float *opacities,
                                 const float *backgrounds, const bool *masks, int width, int height,
                                 int tile_size, int tile_width, int tile_height,
                                 const int32_t *tile_offsets, const int32_t *flatten_ids,
                                 long long n_isects, float *renders, float *alphas,
                                 int32_t *last_ids, float *final_Ts, int32_t *pair_counts,
                                 cudaStream_t stream);

/* Same as gsb_rasterize_bwd (gsplat::rasterize_to_pixels_3dgs_bwd,
 * Rasterization.cpp:121-214) with the final transmittances of the forward
 * (gsb_rasterize_fwd_ex) as an input: the backward then starts from the
 * forward's own T instead of 1 - render_alphas, whose float32 rounding leaves
 * nearly opaque pixels (alpha ~ 0.9999) with a relative error of up to ~3e-4 in
 * T. final_Ts may be NULL (then 1 - render_alphas, the reference's form). */
GSB_API int gsb_rasterize_bwd_ex(int I, int channels, const float *means2d, const float *conics,
                                 const float *colors, const float *opacities,
                                 const float *backgrounds, const bool *masks, int width, int height,
                                 int tile_size, int tile_width, int tile_height,
                                 const int32_t *tile_offsets, const int32_t *flatten_ids,
                                 long long n_isects, const float *render_alphas,
                                 const float *final_Ts, const int32_t *last_ids,
                                 const float *v_render_colors, const float *v_render_alphas,
                                 float *v_means2d_abs, float *v_means2d, float *v_conics,
                                 float *v_colors, float *v_opacities, cudaStream_t stream);

/* --- Rasterize to indices -------------------------------------------------
 * Replaces torch op gsplat::rasterize_to_indices_3dgs (gsplat/cuda/ext.cpp:737;
 * gsplat/cuda/csrc/Rasterization.cpp:216-300, kernel RasterizeToIndices3DGS.cu).
 * Dense layout: means2d [I,N,2], conics [I,N,3], opacities [I,N],
 * transmittances [I,H,W]; tile_offsets / flatten_ids of the sorted intersections.
 * Batches [range_start, range_end) of tile_size^2 tile-list entries are walked
 * front to back. Two calls: with chunk_ends NULL it writes chunk_cnts int32
 * [I*H*W] (pairs per pixel); with chunk_ends = inclusive prefix sum of those
 * counts (int64) it writes gaussian_ids (flatten id % N) and pixel_ids
 * (image*H*W + row*W + col), int64 [total], grouped by pixel in (image, row,
 * column) order and front to back inside a pixel. tile_size 1..32. */
GSB_API int gsb_rasterize_to_indices(int range_start, int range_end, int I, int N, long long n_isects,
                                     const float *means2d, const float *conics, const float *opacities,
                                     int width, int height, int tile_size, int tile_width, int tile_height,
                                     const int32_t *tile_offsets, const int32_t *flatten_ids,
                                     const float *transmittances, const int64_t *chunk_ends,
                                     int32_t *chunk_cnts, int64_t *gaussian_ids, int64_t *pixel_ids,
                                     cudaStream_t stream);

/* --- Densification statistics ----------------------------------------------
 * The per-step state update of the reference's DefaultStrategy._update_state
 * (gsplat/strategy/default.py:218-276), which has no kernel there (torch ops).
 * grads [n,2] (means2d.grad or .absgrad), radii int32 [n,2]; packed: n = nnz
 * pairs with gaussian_ids [n]; dense (gaussian_ids NULL): n = C*N pairs of
 * Gaussian index % N, counted when both radii are positive. Adds
 * |grad * (W/2*n_cameras, H/2*n_cameras)| to grad2d [N] and 1 to count [N];
 * with max_radii [N] (optional) keeps the largest max(radii)/max(W, H). */
GSB_API int gsb_densify_accumulate(long long n, int N, const int64_t *gaussian_ids, const float *grads,
                                   const int32_t *radii, int width, int height, int n_cameras, float *grad2d,
                                   float *count, float *max_radii, cudaStream_t stream);

/* --- Selective Adam -------------------------------------------------------
 * Replaces gsplat::adam (gsplat/cuda/csrc/Adam.cpp:37-65, AdamCUDA.cu:34-69):
 * masked Adam without bias correction on param/grad/exp_avg/exp_avg_sq of
 * N rows x D elements; valid [N] optional. gsb_adam_multi updates several
 * groups (one SelectiveAdam.step, gsplat/optimizers/selective_adam.py:63-101)
 * sharing the same visibility mask in one launch per 8 groups. */
typedef struct GsbAdamGroup {
    float *param;
    const float *grad;
    float *exp_avg;
    float *exp_avg_sq;
    long long numel; /* N * D */
    int D;
    float lr;
    float eps;
} GsbAdamGroup;

GSB_API int gsb_adam(float *param, const float *grad, float *exp_avg, float *exp_avg_sq,
             const bool *valid, long long N, long long D, float lr, float b1, float b2,
             float eps, cudaStream_t stream);
GSB_API int gsb_adam_multi(int n_groups, const GsbAdamGroup *groups, const bool *valid, float b1,
                   float b2, cudaStream_t stream);

/* --- Gaussian-sharded exchange (multi-GPU) ---------------------------------
 * Replace the column concatenation, split and id arithmetic around the
 * all-to-all of the reference's distributed rasterization
 * (gsplat/rendering.py:907-975, gsplat/distributed.py:182-272).
 * gsb_pack_rows: buf [rows, sum(words)] (4-byte words) gets the columns of the
 * n_arrays row-major arrays srcs[j] [rows, words[j]] side by side; a NULL
 * source packs zeros; with rows_device (device int64, may be NULL) only the
 * first min(rows, *rows_device) rows are packed, so a count that is still on
 * the device can bound the work. gsb_unpack_rows: the inverse (rows_device
 * likewise), from rows of
 * row_words words (the first sum(words) of each row are read); a NULL
 * destination skips its columns. At most 16 arrays. int64 columns count as 2
 * words. */
GSB_API int gsb_pack_rows(long long rows, const int64_t *rows_device, int n_arrays, void *const *srcs,
                          const int *words, uint32_t *buf, cudaStream_t stream);
GSB_API int gsb_unpack_rows(long long rows, const int64_t *rows_device, int row_words, const uint32_t *buf,
                            int n_arrays, void *const *dsts, const int *words, cudaStream_t stream);
/* Camera c goes to rank d = c / cams_per_rank: cam_out = c mod cams_per_rank,
 * gid_out = gaussian_ids + gauss_counts[0] + ... + gauss_counts[d - 1] (the
 * reference's id remap, rendering.py:944-959), for the first
 * min(n, *n_device) entries (n_device may be NULL). All int64, device memory. */
GSB_API int gsb_exchange_ids(long long n, const int64_t *n_device, const int64_t *camera_ids,
                             const int64_t *gaussian_ids, int cams_per_rank, const int64_t *gauss_counts,
                             int64_t *cam_out, int64_t *gid_out, cudaStream_t stream);

/* --- Peer-memory exchange (multi-GPU, GPUs of one node) --------------------
 * The same exchange as the all-to-all above, done by kernels that store the
 * rows straight into the other GPUs' memory (CUDA IPC mappings, NVLink) and
 * hand over with flags (release / acquire at system scope), so no split size
 * reaches the host and no row is copied twice. Every rank owns one arena
 * (gsb_peer_alloc; its IPC handle, 64 bytes, goes to the other ranks, which
 * map it with gsb_peer_open): a mailbox of gsb_peer_mailbox_bytes() at offset
 * 0, two receive buffers of cap_recv rows (exchanges alternate), and a
 * gradient buffer with one row per local packed row. Rows from source rank r
 * sit at rows cams_per_rank * (n_world[0] + ... + n_world[r - 1]) of a receive
 * buffer. Exchange numbers (epoch) start at 1 and grow by one per exchange,
 * the same on every rank. Every wait is bounded (a few seconds): a wait that
 * runs out writes 1 (previous exchange not consumed), 2 (rows) or 3
 * (gradients) to the group's error word, a host-mapped int
 * (gsb_peer_error_alloc), and the kernel finishes without the data.
 *
 * gsb_peer_send_rows: local packed rows [0, *nnz_device) of the row-major
 * source arrays (as gsb_pack_rows), rows bounds[d] .. bounds[d + 1] to rank d.
 * gsb_peer_recv_rows: waits for every source, writes route int64
 * [2*world + 1] (prefix of the counts by source, then each source's first
 * local row), *nnz_recv, and the received rows in source order into the
 * separate arrays (capacity cap_rows rows). gsb_peer_send_grads: the gradient
 * rows of the received rows (separate arrays, route of that exchange) to their
 * sources' gradient buffers, at the rows they came from.
 * gsb_peer_recv_grads: waits for them and unpacks the first *nnz_device rows
 * of this rank's gradient buffer into separate arrays. */
typedef struct {
    void *arena[8];          /* every rank's arena mapped in this process (own one at [rank]) */
    long long recv_offset;   /* byte offset of receive buffer 0 in an arena */
    long long recv_stride;   /* bytes from receive buffer 0 to 1 */
    long long grad_offset;   /* byte offset of the gradient buffer */
    int rank, world;
    int *error;              /* device address of the host-mapped error word */
} GsbPeerGroup;
GSB_API size_t gsb_peer_mailbox_bytes(void);
/* Number of polls a wait of the peer exchange makes before it gives up
 * (records its kind in the group's error word and lets its kernel finish);
 * applies to the exchange calls made after it, process-wide. polls <= 0
 * restores the default (a few seconds). Returns the previous limit. No
 * reference counterpart: the reference's NCCL collectives have no bounded wait. */
GSB_API long long gsb_peer_set_wait_limit(long long polls);
GSB_API int gsb_peer_alloc(size_t bytes, void **ptr, void *ipc_handle);
GSB_API int gsb_peer_open(const void *ipc_handle, void **ptr);
GSB_API int gsb_peer_close(void *ptr);
GSB_API int gsb_peer_free(void *ptr);
GSB_API int gsb_peer_error_alloc(int **host_ptr, int **device_ptr);
GSB_API int gsb_peer_error_free(int *host_ptr);
GSB_API int gsb_peer_send_rows(const GsbPeerGroup *g, unsigned long long epoch, long long cap_rows,
                               const int64_t *nnz_device, const int64_t *bounds, const int64_t *n_world,
                               int cams_per_rank, long long cap_recv, int n_arrays, void *const *srcs,
                               const int *words, cudaStream_t stream);
GSB_API int gsb_peer_recv_rows(const GsbPeerGroup *g, unsigned long long epoch, long long cap_rows, int64_t *route,
                               int64_t *nnz_recv, const int64_t *n_world, int cams_per_rank, long long cap_recv,
                               int n_arrays, void *const *dsts, const int *words, cudaStream_t stream);
GSB_API int gsb_peer_send_grads(const GsbPeerGroup *g, unsigned long long epoch, long long cap_rows,
                                const int64_t *nnz_recv, const int64_t *route, long long cap_grad, int n_arrays,
                                void *const *srcs, const int *words, cudaStream_t stream);
GSB_API int gsb_peer_recv_grads(const GsbPeerGroup *g, unsigned long long epoch, long long cap_rows,
                                const int64_t *nnz_device, int n_arrays, void *const *dsts, const int *words,
                                cudaStream_t stream);

/* --- Measurement ----------------------------------------------------------
 * FP32 FMA throughput probe (no reference counterpart): blocks x threads threads
 * each run 8 independent FMA chains of iters steps and write one float to out
 * [blocks*threads]; FLOPs = blocks * threads * iters * 16. Time it with events. */
GSB_API int gsb_fp32_fma_probe(float *out, int blocks, int threads, int iters, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* GSPLAT_B200_H_ */
