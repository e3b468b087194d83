"""CPU oracle bindings -- TEST INFRASTRUCTURE ONLY.

numpy front-end over ``oracle/gsb_oracle.c`` (a restatement of the reference
gsplat CUDA semantics, see the header of that file for the file:line of each
function). Only ``tests/``, ``__graft_entry__.smoke`` and ``bench.py``'s CPU
baseline import this module; the gsplat_b200 package never does.

Parity pins: projection, SH, covariance, AABB tile intersection and offset
encoding are checked against golden vectors produced by the reference's own
PyTorch implementation (``tests/golden/make_golden.py``). The rasterizer forward
and backward are checked against the reference's PyTorch rasterizer
(``_rasterize_to_pixels`` / ``accumulate`` with autograd), run with nerfacc's two
compositing functions restated and with this oracle's index pass standing in
for its CUDA op; and the whole training-step pipeline (projection to rasterizer,
forward and backward to the Gaussian parameters) against the reference's
pure-PyTorch ``_rasterization``. The index pass itself, the AccuTile sweep and Adam have no
executable CPU path in the reference; they are restated from the CUDA source.
"""

import ctypes

import numpy as np

from . import build as _build

_lib = None

P = ctypes.c_void_p
I32 = ctypes.c_int
I64 = ctypes.c_longlong
F32 = ctypes.c_float

_SIG = {
    "ora_projection_fwd": [I32, I32, I32, P, P, P, P, P, P, P, I32, I32, F32, F32, F32, F32, I32,
                           I32, P, P, P, P, P],
    "ora_projection_bwd": [I32, I32, I32, P, P, P, P, P, P, I32, I32, F32, I32, P, P, P, P, P, P,
                           P, P, P, P, P, P],
    "ora_sh_fwd": [I32, I64, I32, P, P, P, P],
    "ora_sh_bwd": [I32, I64, I32, P, P, P, P, P, P],
    "ora_isect_count": [I64, P, P, P, P, I32, I32, I32, P],
    "ora_isect_emit": [I64, I32, P, I32, P, P, P, P, P, I32, I32, I32, P, P, P],
    "ora_sort_pairs": [I64, P, P],
    "ora_isect_offsets": [I64, P, I32, I32, I32, P],
    "ora_raster_fwd": [I32, I32, P, P, P, P, P, P, I32, I32, I32, I32, I32, P, P, I64, P, P, P],
    "ora_raster_bwd": [I32, I32, P, P, P, P, P, P, I32, I32, I32, I32, I32, P, P, I64, P, I32, P, P, P,
                       I64, P, P, P, P, P],
    "ora_adam": [I64, I64, P, P, P, P, P, F32, F32, F32, F32],
    "ora_covar_preci_fwd": [I64, P, P, I32, P, P],
    "ora_covar_preci_bwd": [I64, P, P, I32, P, P, P, P],
    "ora_proj_fwd": [I32, I32, I32, P, P, P, I32, I32, I32, P, P],
    "ora_proj_bwd": [I32, I32, I32, P, P, P, I32, I32, I32, P, P, P, P],
    "ora_raster_indices": [I32, I32, I32, I32, I64, P, P, P, I32, I32, I32, I32, I32, P, P, P, P, P, P, P],
}


def lib():
    global _lib
    if _lib is None:
        path = _build.build()
        l = ctypes.CDLL(path)
        for name, args in _SIG.items():
            fn = getattr(l, name)
            fn.argtypes = args
            fn.restype = None
        _lib = l
    return _lib


def _f(a):
    return None if a is None else np.ascontiguousarray(a, dtype=np.float32)


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def projection_fwd(means, covars, quats, scales, opacities, viewmats, Ks, W, H, eps2d=0.3,
                   near_plane=0.01, far_plane=1e10, radius_clip=0.0, calc_compensations=False,
                   camera_model=0):
    means, covars, quats, scales, opacities = map(_f, (means, covars, quats, scales, opacities))
    viewmats, Ks = _f(viewmats), _f(Ks)
    bdims = means.shape[:-2]
    N = means.shape[-2]
    C = viewmats.shape[-3]
    B = int(np.prod(bdims)) if bdims else 1
    radii = np.zeros(bdims + (C, N, 2), np.int32)
    means2d = np.zeros(bdims + (C, N, 2), np.float32)
    depths = np.zeros(bdims + (C, N), np.float32)
    conics = np.zeros(bdims + (C, N, 3), np.float32)
    comps = np.zeros(bdims + (C, N), np.float32) if calc_compensations else None
    lib().ora_projection_fwd(B, C, N, _p(means), _p(covars), _p(quats), _p(scales), _p(opacities),
                             _p(viewmats), _p(Ks), W, H, eps2d, near_plane, far_plane, radius_clip,
                             int(calc_compensations), camera_model, _p(radii), _p(means2d),
                             _p(depths), _p(conics), _p(comps))
    return radii, means2d, depths, conics, comps


def projection_bwd(means, covars, quats, scales, viewmats, Ks, W, H, eps2d, radii, conics, comps,
                   v_means2d, v_depths, v_conics, v_comps, camera_model=0, viewmats_grad=True):
    means, covars, quats, scales = map(_f, (means, covars, quats, scales))
    viewmats, Ks, conics, comps = _f(viewmats), _f(Ks), _f(conics), _f(comps)
    v_means2d, v_depths, v_conics, v_comps = map(_f, (v_means2d, v_depths, v_conics, v_comps))
    radii = np.ascontiguousarray(radii, np.int32)
    bdims = means.shape[:-2]
    N = means.shape[-2]
    C = viewmats.shape[-3]
    B = int(np.prod(bdims)) if bdims else 1
    v_means = np.zeros_like(means)
    v_covars = np.zeros_like(covars) if covars is not None else None
    v_quats = np.zeros_like(quats) if covars is None else None
    v_scales = np.zeros_like(scales) if covars is None else None
    v_viewmats = np.zeros_like(viewmats) if viewmats_grad else None
    lib().ora_projection_bwd(B, C, N, _p(means), _p(covars), _p(quats), _p(scales), _p(viewmats),
                             _p(Ks), W, H, eps2d, camera_model, _p(radii), _p(conics), _p(comps),
                             _p(v_means2d), _p(v_depths), _p(v_conics), _p(v_comps), _p(v_means),
                             _p(v_covars), _p(v_quats), _p(v_scales), _p(v_viewmats))
    return v_means, v_covars, v_quats, v_scales, v_viewmats


def sh_fwd(degree, dirs, coeffs, masks=None):
    dirs, coeffs = _f(dirs), _f(coeffs)
    n = dirs.size // 3
    K = coeffs.shape[-2]
    m = None if masks is None else np.ascontiguousarray(masks, np.uint8)
    out = np.zeros(dirs.shape, np.float32)
    lib().ora_sh_fwd(degree, n, K, _p(dirs), _p(coeffs), _p(m), _p(out))
    return out


def sh_bwd(degree, dirs, coeffs, v_colors, masks=None):
    dirs, coeffs, v_colors = _f(dirs), _f(coeffs), _f(v_colors)
    n = dirs.size // 3
    K = coeffs.shape[-2]
    m = None if masks is None else np.ascontiguousarray(masks, np.uint8)
    v_coeffs = np.zeros(coeffs.shape, np.float32)
    v_dirs = np.zeros(dirs.shape, np.float32)
    lib().ora_sh_bwd(degree, n, K, _p(dirs), _p(coeffs), _p(m), _p(v_colors), _p(v_coeffs),
                     _p(v_dirs))
    return v_coeffs, v_dirs


def isect_tiles(means2d, radii, depths, tile_size, tile_width, tile_height, conics=None,
                opacities=None, image_ids=None, n_images=None, sort=True):
    """Dense when image_ids is None (images = leading dims), else packed."""
    means2d, depths, conics, opacities = _f(means2d), _f(depths), _f(conics), _f(opacities)
    radii = np.ascontiguousarray(radii, np.int32)
    if image_ids is None:
        N = means2d.shape[-2]
        I = int(np.prod(means2d.shape[:-2]))
        n = I * N
        iid = None
    else:
        N = 0
        I = int(n_images)
        n = means2d.shape[0]
        iid = np.ascontiguousarray(image_ids, np.int64)
    if (conics is None) != (opacities is None):
        conics, opacities = None, None
    assert means2d.size == 2 * n and radii.size == 2 * n and depths.size == n
    if conics is not None:
        assert conics.size == 3 * n and opacities.size == n, (conics.shape, opacities.shape)
    tpg = np.zeros(depths.shape, np.int32)
    lib().ora_isect_count(n, _p(means2d), _p(radii), _p(conics), _p(opacities), tile_size,
                          tile_width, tile_height, _p(tpg))
    cum = np.cumsum(tpg.reshape(-1).astype(np.int64))
    n_isects = int(cum[-1]) if n > 0 else 0
    keys = np.zeros(n_isects, np.int64)
    ids = np.zeros(n_isects, np.int32)
    if n_isects:
        lib().ora_isect_emit(n, max(N, 1), _p(iid), I, _p(means2d), _p(radii), _p(depths),
                             _p(conics), _p(opacities), tile_size, tile_width, tile_height,
                             _p(cum), _p(keys), _p(ids))
        if sort:
            lib().ora_sort_pairs(n_isects, _p(keys), _p(ids))
    return tpg, keys, ids


def isect_offset_encode(isect_ids, n_images, tile_width, tile_height):
    keys = np.ascontiguousarray(isect_ids, np.int64)
    out = np.zeros((n_images, tile_height, tile_width), np.int32)
    lib().ora_isect_offsets(keys.size, _p(keys), n_images, tile_width, tile_height, _p(out))
    return out


def _check_splats(means2d, conics, colors, opacities, fids):
    n = means2d.size // 2
    assert conics.size == 3 * n and opacities.size == n and colors.size == n * colors.shape[-1], (
        means2d.shape, conics.shape, colors.shape, opacities.shape)
    assert fids.size == 0 or (0 <= fids.min() and fids.max() < n)


def raster_fwd(means2d, conics, colors, opacities, W, H, tile_size, offsets, flatten_ids,
               backgrounds=None, masks=None):
    means2d, conics, colors, opacities, backgrounds = map(
        _f, (means2d, conics, colors, opacities, backgrounds))
    offsets = np.ascontiguousarray(offsets, np.int32)
    fids = np.ascontiguousarray(flatten_ids, np.int32)
    m = None if masks is None else np.ascontiguousarray(masks, np.uint8)
    idims = offsets.shape[:-2]
    I = int(np.prod(idims)) if idims else 1
    th, tw = offsets.shape[-2:]
    CH = colors.shape[-1]
    _check_splats(means2d, conics, colors, opacities, fids)
    renders = np.zeros(idims + (H, W, CH), np.float32)
    alphas = np.zeros(idims + (H, W, 1), np.float32)
    last = np.zeros(idims + (H, W), np.int32)
    lib().ora_raster_fwd(I, CH, _p(means2d), _p(conics), _p(colors), _p(opacities), _p(backgrounds),
                         _p(m), W, H, tile_size, tw, th, _p(offsets), _p(fids), fids.size,
                         _p(renders), _p(alphas), _p(last))
    return renders, alphas, last


def raster_bwd(means2d, conics, colors, opacities, W, H, tile_size, offsets, flatten_ids,
               render_alphas, last_ids, v_renders, v_alphas, backgrounds=None, masks=None,
               absgrad=False, t_from_alphas=False):
    """Rasterizer backward in float64 (RasterizeToPixels3DGSBwd.cu:99-299). The
    final transmittance of each pixel is recomputed in float64 over the pairs up
    to ``last_ids`` (the exact value the PyTorch path differentiates);
    ``t_from_alphas`` uses 1 - render_alphas instead (the CUDA reference's form)."""
    means2d, conics, colors, opacities, backgrounds = map(
        _f, (means2d, conics, colors, opacities, backgrounds))
    render_alphas, v_renders, v_alphas = _f(render_alphas), _f(v_renders), _f(v_alphas)
    offsets = np.ascontiguousarray(offsets, np.int32)
    fids = np.ascontiguousarray(flatten_ids, np.int32)
    last_ids = np.ascontiguousarray(last_ids, np.int32)
    m = None if masks is None else np.ascontiguousarray(masks, np.uint8)
    idims = offsets.shape[:-2]
    I = int(np.prod(idims)) if idims else 1
    th, tw = offsets.shape[-2:]
    CH = colors.shape[-1]
    _check_splats(means2d, conics, colors, opacities, fids)
    n_splats = opacities.size
    v_m2d = np.zeros(means2d.shape, np.float32)
    v_abs = np.zeros(means2d.shape, np.float32) if absgrad else None
    v_con = np.zeros(conics.shape, np.float32)
    v_col = np.zeros(colors.shape, np.float32)
    v_op = np.zeros(opacities.shape, np.float32)
    lib().ora_raster_bwd(I, CH, _p(means2d), _p(conics), _p(colors), _p(opacities),
                         _p(backgrounds), _p(m), W, H, tile_size, tw, th, _p(offsets), _p(fids),
                         fids.size, _p(render_alphas), int(bool(t_from_alphas)), _p(last_ids),
                         _p(v_renders), _p(v_alphas),
                         n_splats, _p(v_abs), _p(v_m2d), _p(v_con), _p(v_col), _p(v_op))
    return v_m2d, v_con, v_col, v_op, v_abs


def adam(param, grad, exp_avg, exp_avg_sq, valid, lr, b1, b2, eps):
    """In-place on float32 numpy arrays."""
    N = param.shape[0]
    D = param.size // N
    v = None if valid is None else np.ascontiguousarray(valid, np.uint8)
    lib().ora_adam(N, D, _p(param), _p(_f(grad)), _p(exp_avg), _p(exp_avg_sq), _p(v), lr, b1, b2,
                   eps)


def covar_preci_fwd(quats, scales, triu=False, compute_covar=True, compute_preci=True):
    """quat_scale_to_covar_preci forward (QuatScaleToCovarCUDA.cu:36-122)."""
    quats, scales = _f(quats), _f(scales)
    n = quats.size // 4
    shape = quats.shape[:-1] + ((6,) if triu else (3, 3))
    covars = np.zeros(shape, np.float32) if compute_covar else None
    precis = np.zeros(shape, np.float32) if compute_preci else None
    lib().ora_covar_preci_fwd(n, _p(quats), _p(scales), int(triu), _p(covars), _p(precis))
    return covars, precis


def covar_preci_bwd(quats, scales, triu, v_covars, v_precis):
    """quat_scale_to_covar_preci backward (QuatScaleToCovarCUDA.cu:124-292)."""
    quats, scales = _f(quats), _f(scales)
    n = quats.size // 4
    v_quats = np.zeros(quats.shape, np.float32)
    v_scales = np.zeros(scales.shape, np.float32)
    lib().ora_covar_preci_bwd(n, _p(quats), _p(scales), int(triu), _p(_f(v_covars)), _p(_f(v_precis)),
                              _p(v_quats), _p(v_scales))
    return v_quats, v_scales


def proj_fwd(means, covars, Ks, W, H, camera_model=0):
    """proj forward (ProjectionEWASimple.cu:36-161): camera-space [..., C, N, 3] / [..., C, N, 3, 3]."""
    means, covars, Ks = _f(means), _f(covars), _f(Ks)
    C, N = means.shape[-3], means.shape[-2]
    B = means.size // max(1, C * N * 3)
    means2d = np.zeros(means.shape[:-1] + (2,), np.float32)
    covars2d = np.zeros(means.shape[:-1] + (2, 2), np.float32)
    lib().ora_proj_fwd(B, C, N, _p(means), _p(covars), _p(Ks), W, H, camera_model, _p(means2d), _p(covars2d))
    return means2d, covars2d


def proj_bwd(means, covars, Ks, W, H, camera_model, v_means2d, v_covars2d):
    """proj backward (ProjectionEWASimple.cu:163-317)."""
    means, covars, Ks = _f(means), _f(covars), _f(Ks)
    C, N = means.shape[-3], means.shape[-2]
    B = means.size // max(1, C * N * 3)
    v_means = np.zeros(means.shape, np.float32)
    v_covars = np.zeros(covars.shape, np.float32)
    lib().ora_proj_bwd(B, C, N, _p(means), _p(covars), _p(Ks), W, H, camera_model, _p(_f(v_means2d)),
                       _p(_f(v_covars2d)), _p(v_means), _p(v_covars))
    return v_means, v_covars


def raster_indices(range_start, range_end, transmittances, means2d, conics, opacities, W, H, tile_size,
                   offsets, flatten_ids):
    """rasterize_to_indices_in_range (RasterizeToIndices3DGS.cu:36-200): returns
    gaussian_ids, pixel_ids, image_ids (int64) and the per-pixel counts."""
    means2d, conics, opacities, trans = _f(means2d), _f(conics), _f(opacities), _f(transmittances)
    offsets = np.ascontiguousarray(offsets, np.int32)
    fids = np.ascontiguousarray(flatten_ids, np.int32)
    N = means2d.shape[-2]
    I = means2d.size // (2 * N)
    th, tw = offsets.shape[-2:]
    counts = np.zeros(I * H * W, np.int32)
    args = (range_start, range_end, I, N, fids.size, _p(means2d), _p(conics), _p(opacities), W, H, tile_size,
            tw, th, _p(offsets), _p(fids), _p(trans))
    lib().ora_raster_indices(*args, _p(counts), None, None, None)
    ends = np.cumsum(counts, dtype=np.int64)
    starts = np.ascontiguousarray(ends - counts)
    total = int(ends[-1]) if ends.size else 0
    gids = np.zeros(total, np.int64)
    pids = np.zeros(total, np.int64)
    lib().ora_raster_indices(*args, None, _p(starts), _p(gids), _p(pids))
    return gids, pids % (W * H), pids // (W * H), counts
