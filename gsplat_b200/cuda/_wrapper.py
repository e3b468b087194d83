"""Python operators of the splatting hot path, backed by the gsplat_b200 C ABI.

Names, argument order, defaults, return tuples and assertion behaviour follow the
reference's ``gsplat/cuda/_wrapper.py`` (fully_fused_projection 479-631,
spherical_harmonics 342-372, quat_scale_to_covar_preci 375-407, proj 410-476,
isect_tiles 634-730, isect_offset_encode 806-826,
rasterize_to_pixels 829-961, rasterize_to_indices_in_range 1274-1353, adam 326-339
and the autograd Functions
_FullyFusedProjection 1464-1594, _RasterizeToPixels 1709-1836,
_FullyFusedProjectionPacked 2107-2326, _SphericalHarmonics 2329-2364), so code and
tests written against the reference run unchanged. Every op launches the
hand-written sm_100a kernels of ``gsplat_b200/csrc``; there is no CPU path.
"""

import math
import warnings
from typing import Optional, Tuple

import torch
from torch import Tensor
from typing_extensions import Literal

from . import _backend as _B
from ._backend import call, check_cuda, device_guard, ptr, stream_of

CameraModel = Literal["pinhole", "ortho", "fisheye", "ftheta", "lidar"]
_CAMERA_IDS = {"pinhole": 0, "ortho": 1, "fisheye": 2}


def _camera_id(camera_model: str) -> int:
    assert (
        camera_model != "ftheta"
    ), "ftheta camera is only supported via UT, please set with_ut=True in the rasterization()"
    if camera_model not in _CAMERA_IDS:
        raise NotImplementedError(
            f"camera_model={camera_model!r} is not implemented by gsplat_b200 (pinhole, ortho, fisheye)"
        )
    return _CAMERA_IDS[camera_model]


def has_3dgs() -> bool:
    return _B.is_available()


def has_adam() -> bool:
    return _B.is_available()


def has_2dgs() -> bool:
    return False


def has_3dgut() -> bool:
    return False


def has_reloc() -> bool:
    return False


def has_camera_wrappers() -> bool:
    return False


# ---------------------------------------------------------------------------
# Selective Adam
# ---------------------------------------------------------------------------
def adam(
    param: Tensor,
    param_grad: Tensor,
    exp_avg: Tensor,
    exp_avg_sq: Tensor,
    valid: Tensor,
    lr: float,
    b1: float,
    b2: float,
    eps: float,
) -> None:
    for name, t in (("param", param), ("param_grad", param_grad), ("exp_avg", exp_avg),
                    ("exp_avg_sq", exp_avg_sq), ("valid", valid)):
        check_cuda(name, t)
    N = param.size(0)
    D = param.numel() // N if N > 0 else 0
    with device_guard(param.device):
        call("gsb_adam", ptr(param), ptr(param_grad), ptr(exp_avg), ptr(exp_avg_sq), ptr(valid),
             N, D, lr, b1, b2, eps, stream_of(param))


def adam_multi(groups, valid: Optional[Tensor], b1: float, b2: float) -> None:
    """One launch for several (param, grad, exp_avg, exp_avg_sq, lr, eps) groups
    that share the row visibility mask ``valid``."""
    if not groups:
        return
    arr = (_B.GsbAdamGroup * len(groups))()
    dev = groups[0][0].device
    for i, (p, g, m, v, lr, eps) in enumerate(groups):
        for name, t in (("param", p), ("grad", g), ("exp_avg", m), ("exp_avg_sq", v)):
            check_cuda(name, t)
        N = p.size(0)
        arr[i] = _B.GsbAdamGroup(p.data_ptr(), g.data_ptr(), m.data_ptr(), v.data_ptr(), p.numel(),
                                 p.numel() // N if N > 0 else 1, lr, eps)
    check_cuda("valid", valid)
    with device_guard(dev):
        call("gsb_adam_multi", len(groups), arr, ptr(valid), b1, b2, stream_of(groups[0][0]))


# ---------------------------------------------------------------------------
# Spherical harmonics
# ---------------------------------------------------------------------------
def spherical_harmonics(
    degrees_to_use: int,
    dirs: Tensor,  # [..., 3]
    coeffs: Tensor,  # [..., K, 3]
    masks: Optional[Tensor] = None,  # [...,]
) -> Tensor:
    """Computes spherical harmonics colours (reference _wrapper.py:342-372)."""
    assert (degrees_to_use + 1) ** 2 <= coeffs.shape[-2], coeffs.shape
    batch_dims = dirs.shape[:-1]
    assert dirs.shape == batch_dims + (3,), dirs.shape
    assert (
        (len(coeffs.shape) == len(batch_dims) + 2)
        and coeffs.shape[:-2] == batch_dims
        and coeffs.shape[-1] == 3
    ), coeffs.shape
    if masks is not None:
        assert masks.shape == batch_dims, masks.shape
        masks = masks.contiguous()
    return _SphericalHarmonics.apply(degrees_to_use, dirs.contiguous(), coeffs.contiguous(), masks)


class _SphericalHarmonics(torch.autograd.Function):
    @staticmethod
    def forward(ctx, sh_degree: int, dirs: Tensor, coeffs: Tensor, masks: Optional[Tensor]) -> Tensor:
        for name, t in (("dirs", dirs), ("coeffs", coeffs), ("masks", masks)):
            check_cuda(name, t)
        n = dirs.numel() // 3
        K = coeffs.shape[-2]
        colors = torch.empty(dirs.shape, dtype=dirs.dtype, device=dirs.device)
        with device_guard(dirs.device):
            call("gsb_spherical_harmonics_fwd", sh_degree, n, K, ptr(dirs), ptr(coeffs), ptr(masks),
                 ptr(colors), stream_of(dirs))
        ctx.save_for_backward(dirs, coeffs, masks)
        ctx.sh_degree = sh_degree
        return colors

    @staticmethod
    def backward(ctx, v_colors: Tensor):
        dirs, coeffs, masks = ctx.saved_tensors
        compute_v_dirs = ctx.needs_input_grad[1]
        v_colors = v_colors.contiguous()
        n = dirs.numel() // 3
        K = coeffs.shape[-2]
        v_coeffs = torch.empty_like(coeffs)
        v_dirs = torch.empty_like(dirs) if compute_v_dirs else None
        with device_guard(dirs.device):
            call("gsb_spherical_harmonics_bwd", ctx.sh_degree, n, K, ptr(dirs), ptr(coeffs),
                 ptr(masks), ptr(v_colors), ptr(v_coeffs), ptr(v_dirs), stream_of(dirs))
        return None, v_dirs, v_coeffs, None


# ---------------------------------------------------------------------------
# Covariances and the simple projection
# ---------------------------------------------------------------------------
def world_to_cam(
    means: Tensor,  # [..., N, 3]
    covars: Tensor,  # [..., N, 3, 3]
    viewmats: Tensor,  # [..., C, 4, 4]
) -> Tuple[Tensor, Tensor]:
    """Transforms Gaussians to camera space (reference _wrapper.py:288-323, which
    has no kernel for it either and evaluates it with tensor ops): returns means
    [..., C, N, 3] and covariances [..., C, N, 3, 3]."""
    warnings.warn(
        "world_to_cam() has no kernel; it is evaluated with tensor ops and will be removed in a "
        "future release.",
        DeprecationWarning,
    )
    batch_dims = means.shape[:-2]
    N = means.shape[-2]
    C = viewmats.shape[-3]
    assert means.shape == batch_dims + (N, 3), means.shape
    assert covars.shape == batch_dims + (N, 3, 3), covars.shape
    assert viewmats.shape == batch_dims + (C, 4, 4), viewmats.shape
    R = viewmats[..., :3, :3]  # [..., C, 3, 3]
    t = viewmats[..., :3, 3]  # [..., C, 3]
    means_c = torch.einsum("...cij,...nj->...cni", R, means) + t[..., None, :]
    covars_c = torch.einsum("...cij,...njk,...clk->...cnil", R, covars, R)
    return means_c, covars_c


def quat_scale_to_covar_preci(
    quats: Tensor,  # [..., 4]
    scales: Tensor,  # [..., 3]
    compute_covar: bool = True,
    compute_preci: bool = True,
    triu: bool = False,
) -> Tuple[Optional[Tensor], Optional[Tensor]]:
    """Covariance R S S R^T and precision R S^-1 S^-1 R^T matrices from
    quaternions (any norm) and scales (reference _wrapper.py:375-407): [..., 3, 3],
    or [..., 6] upper triangles with triu; None where not requested."""
    batch_dims = quats.shape[:-1]
    assert quats.shape == batch_dims + (4,), quats.shape
    assert scales.shape == batch_dims + (3,), scales.shape
    covars, precis = _QuatScaleToCovarPreci.apply(quats.contiguous(), scales.contiguous(), compute_covar,
                                                  compute_preci, triu)
    return covars if compute_covar else None, precis if compute_preci else None


class _QuatScaleToCovarPreci(torch.autograd.Function):
    """Reference _wrapper.py:1356-1400."""

    @staticmethod
    def forward(ctx, quats: Tensor, scales: Tensor, compute_covar: bool, compute_preci: bool, triu: bool):
        for name, t in (("quats", quats), ("scales", scales)):
            check_cuda(name, t)
        batch_dims = quats.shape[:-1]
        n = quats.numel() // 4
        shape = batch_dims + ((6,) if triu else (3, 3))
        covars = torch.empty(shape, dtype=quats.dtype, device=quats.device) if compute_covar else None
        precis = torch.empty(shape, dtype=quats.dtype, device=quats.device) if compute_preci else None
        with device_guard(quats.device):
            call("gsb_quat_scale_to_covar_preci_fwd", n, ptr(quats), ptr(scales), int(triu), ptr(covars),
                 ptr(precis), stream_of(quats))
        ctx.save_for_backward(quats, scales)
        ctx.compute_covar = compute_covar
        ctx.compute_preci = compute_preci
        ctx.triu = triu
        if covars is None:
            covars = torch.empty(shape, dtype=quats.dtype, device=quats.device)
            ctx.mark_non_differentiable(covars)
        if precis is None:
            precis = torch.empty(shape, dtype=quats.dtype, device=quats.device)
            ctx.mark_non_differentiable(precis)
        return covars, precis

    @staticmethod
    def backward(ctx, v_covars: Tensor, v_precis: Tensor):
        quats, scales = ctx.saved_tensors
        if ctx.compute_covar and v_covars is not None and v_covars.is_sparse:
            v_covars = v_covars.to_dense()
        if ctx.compute_preci and v_precis is not None and v_precis.is_sparse:
            v_precis = v_precis.to_dense()
        v_covars = v_covars.contiguous() if (ctx.compute_covar and v_covars is not None) else None
        v_precis = v_precis.contiguous() if (ctx.compute_preci and v_precis is not None) else None
        n = quats.numel() // 4
        v_quats = torch.empty_like(quats)
        v_scales = torch.empty_like(scales)
        with device_guard(quats.device):
            call("gsb_quat_scale_to_covar_preci_bwd", n, ptr(quats), ptr(scales), int(ctx.triu), ptr(v_covars),
                 ptr(v_precis), ptr(v_quats), ptr(v_scales), stream_of(quats))
        return v_quats, v_scales, None, None, None


def persp_proj(means: Tensor, covars: Tensor, Ks: Tensor, width: int, height: int) -> Tuple[Tensor, Tensor]:
    """Perspective projection (reference _wrapper.py:410-438); deprecated there in
    favour of ``proj(..., camera_model="pinhole")``."""
    warnings.warn(
        "persp_proj is deprecated and will be removed in a future release. "
        "Use proj with ortho=False instead.",
        DeprecationWarning,
    )
    return proj(means, covars, Ks, width, height, camera_model="pinhole")


def proj(
    means: Tensor,  # [..., C, N, 3]
    covars: Tensor,  # [..., C, N, 3, 3]
    Ks: Tensor,  # [..., C, 3, 3]
    width: int,
    height: int,
    camera_model: CameraModel = "pinhole",
) -> Tuple[Tensor, Tensor]:
    """Projects camera-space Gaussians (reference _wrapper.py:441-476): returns
    means2d [..., C, N, 2] and covariances [..., C, N, 2, 2]."""
    model = _camera_id(camera_model)
    batch_dims = means.shape[:-3]
    C, N = means.shape[-3:-1]
    assert means.shape == batch_dims + (C, N, 3), means.shape
    assert covars.shape == batch_dims + (C, N, 3, 3), covars.shape
    assert Ks.shape == batch_dims + (C, 3, 3), Ks.shape
    return _Proj.apply(means.contiguous(), covars.contiguous(), Ks.contiguous(), width, height, model)


class _Proj(torch.autograd.Function):
    """Reference _wrapper.py:1403-1461."""

    @staticmethod
    def forward(ctx, means: Tensor, covars: Tensor, Ks: Tensor, width: int, height: int, model: int):
        for name, t in (("means", means), ("covars", covars), ("Ks", Ks)):
            check_cuda(name, t)
        C, N = means.shape[-3:-1]
        B = means.numel() // max(1, C * N * 3)
        means2d = torch.empty(means.shape[:-1] + (2,), dtype=means.dtype, device=means.device)
        covars2d = torch.empty(means.shape[:-1] + (2, 2), dtype=means.dtype, device=means.device)
        with device_guard(means.device):
            call("gsb_proj_fwd", B, C, N, ptr(means), ptr(covars), ptr(Ks), width, height, model,
                 ptr(means2d), ptr(covars2d), stream_of(means))
        ctx.save_for_backward(means, covars, Ks)
        ctx.width, ctx.height, ctx.model = width, height, model
        return means2d, covars2d

    @staticmethod
    def backward(ctx, v_means2d: Tensor, v_covars2d: Tensor):
        means, covars, Ks = ctx.saved_tensors
        C, N = means.shape[-3:-1]
        B = means.numel() // max(1, C * N * 3)
        v_means2d = (v_means2d if v_means2d is not None else torch.zeros(
            means.shape[:-1] + (2,), dtype=means.dtype, device=means.device)).contiguous()
        v_covars2d = (v_covars2d if v_covars2d is not None else torch.zeros(
            means.shape[:-1] + (2, 2), dtype=means.dtype, device=means.device)).contiguous()
        v_means = torch.empty_like(means)
        v_covars = torch.empty_like(covars)
        with device_guard(means.device):
            call("gsb_proj_bwd", B, C, N, ptr(means), ptr(covars), ptr(Ks), ctx.width, ctx.height, ctx.model,
                 ptr(v_means2d), ptr(v_covars2d), ptr(v_means), ptr(v_covars), stream_of(means))
        return v_means, v_covars, None, None, None, None


# ---------------------------------------------------------------------------
# Projection
# ---------------------------------------------------------------------------
def fully_fused_projection(
    means: Tensor,  # [..., N, 3]
    covars: Optional[Tensor],  # [..., N, 6] or None
    quats: Optional[Tensor],  # [..., N, 4] or None
    scales: Optional[Tensor],  # [..., N, 3] or None
    viewmats: Tensor,  # [..., C, 4, 4]
    Ks: Tensor,  # [..., C, 3, 3]
    width: int,
    height: int,
    eps2d: float = 0.3,
    near_plane: float = 0.01,
    far_plane: float = 1e10,
    radius_clip: float = 0.0,
    packed: bool = False,
    sparse_grad: bool = False,
    calc_compensations: bool = False,
    camera_model: CameraModel = "pinhole",
    opacities: Optional[Tensor] = None,  # [..., N] or None
) -> Tuple[Tensor, ...]:
    """Projects Gaussians to 2D (reference _wrapper.py:479-631).

    Returns (radii, means2d, depths, conics, compensations) when packed is False,
    else (batch_ids, camera_ids, gaussian_ids, indptr, radii, means2d, depths,
    conics, compensations) with the pairs in COO order.
    """
    batch_dims = means.shape[:-2]
    N = means.shape[-2]
    C = viewmats.shape[-3]
    assert means.shape == batch_dims + (N, 3), means.shape
    assert viewmats.shape == batch_dims + (C, 4, 4), viewmats.shape
    assert Ks.shape == batch_dims + (C, 3, 3), Ks.shape
    means = means.contiguous()
    if covars is not None:
        assert covars.shape == batch_dims + (N, 6), covars.shape
        covars = covars.contiguous()
    else:
        assert quats is not None, "covars or quats is required"
        assert scales is not None, "covars or scales is required"
        assert quats.shape == batch_dims + (N, 4), quats.shape
        assert scales.shape == batch_dims + (N, 3), scales.shape
        quats = quats.contiguous()
        scales = scales.contiguous()
    if sparse_grad:
        assert packed, "sparse_grad is only supported when packed is True"
        assert batch_dims == (), "sparse_grad does not support batch dimensions"
    if opacities is not None:
        assert opacities.shape == batch_dims + (N,), opacities.shape
        opacities = opacities.contiguous()
    cam = _camera_id(camera_model)
    viewmats = viewmats.contiguous()
    Ks = Ks.contiguous()
    if packed:
        return _FullyFusedProjectionPacked.apply(
            means, covars, quats, scales, viewmats, Ks, width, height, eps2d, near_plane,
            far_plane, radius_clip, sparse_grad, calc_compensations, cam, opacities)
    return _FullyFusedProjection.apply(
        means, covars, quats, scales, viewmats, Ks, width, height, eps2d, near_plane, far_plane,
        radius_clip, calc_compensations, cam, opacities)


def _check_proj_inputs(means, covars, quats, scales, viewmats, Ks, opacities):
    for name, t in (("means", means), ("covars", covars), ("quats", quats), ("scales", scales),
                    ("viewmats", viewmats), ("Ks", Ks), ("opacities", opacities)):
        check_cuda(name, t)
        if t is not None and t.dtype != torch.float32:
            raise RuntimeError(f"{name} must be float32")


class _FullyFusedProjection(torch.autograd.Function):
    @staticmethod
    def forward(ctx, means, covars, quats, scales, viewmats, Ks, width, height, eps2d, near_plane,
                far_plane, radius_clip, calc_compensations, camera_model, opacities):
        _check_proj_inputs(means, covars, quats, scales, viewmats, Ks, opacities)
        batch_dims = means.shape[:-2]
        N = means.shape[-2]
        C = viewmats.shape[-3]
        B = math.prod(batch_dims)
        dev = means.device
        radii = torch.empty(batch_dims + (C, N, 2), dtype=torch.int32, device=dev)
        means2d = torch.empty(batch_dims + (C, N, 2), dtype=means.dtype, device=dev)
        depths = torch.empty(batch_dims + (C, N), dtype=means.dtype, device=dev)
        conics = torch.empty(batch_dims + (C, N, 3), dtype=means.dtype, device=dev)
        comps = torch.zeros(batch_dims + (C, N), dtype=means.dtype, device=dev) if calc_compensations else None
        with device_guard(dev):
            call("gsb_projection_fused_fwd", B, C, N, ptr(means), ptr(covars), ptr(quats),
                 ptr(scales), ptr(opacities), ptr(viewmats), ptr(Ks), width, height, eps2d,
                 near_plane, far_plane, radius_clip, int(calc_compensations), camera_model,
                 ptr(radii), ptr(means2d), ptr(depths), ptr(conics), ptr(comps), stream_of(means))
        ctx.save_for_backward(means, covars, quats, scales, viewmats, Ks, radii, conics, comps)
        ctx.width = width
        ctx.height = height
        ctx.eps2d = eps2d
        ctx.camera_model = camera_model
        ctx.mark_non_differentiable(radii)
        return radii, means2d, depths, conics, comps

    @staticmethod
    def backward(ctx, v_radii, v_means2d, v_depths, v_conics, v_comps):
        means, covars, quats, scales, viewmats, Ks, radii, conics, comps = ctx.saved_tensors
        batch_dims = means.shape[:-2]
        N = means.shape[-2]
        C = viewmats.shape[-3]
        B = math.prod(batch_dims)
        v_means2d = v_means2d.contiguous()
        v_depths = v_depths.contiguous()
        v_conics = v_conics.contiguous()
        if comps is None:
            v_comps = None
        elif v_comps is not None:
            v_comps = v_comps.contiguous()
        v_means = torch.empty_like(means)
        v_covars = torch.empty_like(covars) if covars is not None else None
        v_quats = torch.empty_like(quats) if covars is None else None
        v_scales = torch.empty_like(scales) if covars is None else None
        v_viewmats = torch.zeros_like(viewmats) if ctx.needs_input_grad[4] else None
        with device_guard(means.device):
            call("gsb_projection_fused_bwd", B, C, N, ptr(means), ptr(covars), ptr(quats),
                 ptr(scales), ptr(viewmats), ptr(Ks), ctx.width, ctx.height, ctx.eps2d,
                 ctx.camera_model, ptr(radii), ptr(conics), ptr(comps), ptr(v_means2d),
                 ptr(v_depths), ptr(v_conics), ptr(v_comps), ptr(v_means), ptr(v_covars),
                 ptr(v_quats), ptr(v_scales), ptr(v_viewmats), stream_of(means))
        return (
            v_means if ctx.needs_input_grad[0] else None,
            v_covars if ctx.needs_input_grad[1] else None,
            v_quats if ctx.needs_input_grad[2] else None,
            v_scales if ctx.needs_input_grad[3] else None,
            v_viewmats,
            None, None, None, None, None, None, None, None, None, None,
        )


def _scan_i32(x: Tensor) -> Tensor:
    """Inclusive int32 -> int64 prefix sum on the device (gsb_inclusive_scan_i32)."""
    n = x.numel()
    out = torch.empty(n, dtype=torch.int64, device=x.device)
    if n == 0:
        return out
    nbytes = _B.lib().gsb_scan_scratch_bytes(n)
    scratch = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
    call("gsb_inclusive_scan_i32", ptr(x), ptr(out), n, ptr(scratch), nbytes, stream_of(x))
    return out


class _FullyFusedProjectionPacked(torch.autograd.Function):
    @staticmethod
    def forward(ctx, means, covars, quats, scales, viewmats, Ks, width, height, eps2d, near_plane,
                far_plane, radius_clip, sparse_grad, calc_compensations, camera_model, opacities):
        _check_proj_inputs(means, covars, quats, scales, viewmats, Ks, opacities)
        batch_dims = means.shape[:-2]
        N = means.shape[-2]
        C = viewmats.shape[-3]
        B = math.prod(batch_dims)
        dev = means.device
        common = (B, C, N, ptr(means), ptr(covars), ptr(quats), ptr(scales), ptr(opacities),
                  ptr(viewmats), ptr(Ks), width, height, eps2d, near_plane, far_plane, radius_clip,
                  int(calc_compensations), camera_model)
        with device_guard(dev):
            stream = stream_of(means)
            nblocks = _B.lib().gsb_projection_packed_blocks(N)
            block_cnts = torch.empty(B * C * nblocks, dtype=torch.int32, device=dev)
            vis_bits = torch.empty(B * C * nblocks * 8, dtype=torch.int32, device=dev)
            call("gsb_projection_packed_count", *common, ptr(block_cnts), ptr(vis_bits), stream)
            block_accum = _scan_i32(block_cnts)
            nnz = int(block_accum[-1].item()) if block_accum.numel() > 0 else 0
            indptr = torch.zeros(B * C + 1, dtype=torch.int32, device=dev)
            batch_ids = torch.empty(nnz, dtype=torch.int64, device=dev)
            camera_ids = torch.empty(nnz, dtype=torch.int64, device=dev)
            gaussian_ids = torch.empty(nnz, dtype=torch.int64, device=dev)
            radii = torch.empty((nnz, 2), dtype=torch.int32, device=dev)
            means2d = torch.empty((nnz, 2), dtype=means.dtype, device=dev)
            depths = torch.empty(nnz, dtype=means.dtype, device=dev)
            conics = torch.empty((nnz, 3), dtype=means.dtype, device=dev)
            comps = torch.zeros(nnz, dtype=means.dtype, device=dev) if calc_compensations else None
            if block_accum.numel() > 0:
                call("gsb_projection_packed_write", *common, ptr(vis_bits), ptr(block_accum), nnz,
                     ptr(indptr),
                     ptr(batch_ids), ptr(camera_ids), ptr(gaussian_ids), ptr(radii), ptr(means2d),
                     ptr(depths), ptr(conics), ptr(comps), stream)
        ctx.save_for_backward(batch_ids, camera_ids, gaussian_ids, means, covars, quats, scales,
                              viewmats, Ks, conics, comps)
        ctx.width = width
        ctx.height = height
        ctx.eps2d = eps2d
        ctx.sparse_grad = sparse_grad
        ctx.camera_model = camera_model
        ctx.mark_non_differentiable(batch_ids, camera_ids, gaussian_ids, indptr, radii)
        return batch_ids, camera_ids, gaussian_ids, indptr, radii, means2d, depths, conics, comps

    @staticmethod
    def backward(ctx, v_batch_ids, v_camera_ids, v_gaussian_ids, v_indptr, v_radii, v_means2d,
                 v_depths, v_conics, v_comps):
        (batch_ids, camera_ids, gaussian_ids, means, covars, quats, scales, viewmats, Ks, conics,
         comps) = ctx.saved_tensors
        batch_dims = means.shape[:-2]
        N = means.shape[-2]
        C = viewmats.shape[-3]
        B = math.prod(batch_dims)
        nnz = batch_ids.numel()
        sparse = ctx.sparse_grad
        v_means2d = v_means2d.contiguous()
        v_depths = v_depths.contiguous()
        v_conics = v_conics.contiguous()
        if comps is None:
            v_comps = None
        elif v_comps is not None:
            v_comps = v_comps.contiguous()

        def grad_buf(t, width_):
            if t is None:
                return None
            return torch.zeros((nnz, width_) if sparse else t.shape, dtype=t.dtype, device=t.device)

        v_means = grad_buf(means, 3)
        v_covars = grad_buf(covars, 6)
        v_quats = grad_buf(quats, 4) if covars is None else None
        v_scales = grad_buf(scales, 3) if covars is None else None
        v_viewmats = torch.zeros_like(viewmats) if ctx.needs_input_grad[4] else None
        with device_guard(means.device):
            call("gsb_projection_packed_bwd", B, C, N, nnz, ptr(means), ptr(covars), ptr(quats),
                 ptr(scales), ptr(viewmats), ptr(Ks), ctx.width, ctx.height, ctx.eps2d,
                 ctx.camera_model, ptr(batch_ids), ptr(camera_ids), ptr(gaussian_ids), ptr(conics),
                 ptr(comps), ptr(v_means2d), ptr(v_depths), ptr(v_conics), ptr(v_comps),
                 int(sparse), ptr(v_means), ptr(v_covars), ptr(v_quats), ptr(v_scales),
                 ptr(v_viewmats), stream_of(means))

        def finish(v, t, idx):
            if not ctx.needs_input_grad[idx] or v is None:
                return None
            if sparse:
                return torch.sparse_coo_tensor(indices=gaussian_ids[None], values=v, size=t.shape,
                                               is_coalesced=len(viewmats) == 1)
            return v

        return (
            finish(v_means, means, 0),
            finish(v_covars, covars, 1),
            finish(v_quats, quats, 2),
            finish(v_scales, scales, 3),
            v_viewmats,
            None, None, None, None, None, None, None, None, None, None, None,
        )


# ---------------------------------------------------------------------------
# Tile intersection
# ---------------------------------------------------------------------------
@torch.no_grad()
def isect_tiles(
    means2d: Tensor,  # [..., N, 2] or [nnz, 2]
    radii: Tensor,  # [..., N, 2] or [nnz, 2]
    depths: Tensor,  # [..., N] or [nnz]
    tile_size: int,
    tile_width: int,
    tile_height: int,
    sort: bool = True,
    segmented: bool = False,
    packed: bool = False,
    n_images: Optional[int] = None,
    image_ids: Optional[Tensor] = None,
    gaussian_ids: Optional[Tensor] = None,
    conics: Optional[Tensor] = None,
    opacities: Optional[Tensor] = None,
) -> Tuple[Tensor, Tensor, Tensor]:
    """Maps projected Gaussians to intersecting tiles (reference _wrapper.py:634-730).

    Returns (tiles_per_gauss int32, isect_ids int64 [n_isects], flatten_ids int32
    [n_isects]); with ``sort`` the pairs are ordered exactly like a stable sort of
    isect_ids. ``segmented`` gives the same result (the keys of each image are
    already contiguous), so one code path serves both.
    """
    if packed:
        assert gaussian_ids is not None, "gaussian_ids is required if packed is True"
    tiles_per_gauss, isect_ids, flatten_ids, _ = _isect_tiles(
        means2d, radii, depths, tile_size, tile_width, tile_height, sort, packed, n_images, image_ids,
        conics, opacities)
    return tiles_per_gauss, isect_ids, flatten_ids


@torch.no_grad()
def isect_tiles_with_offsets(means2d, radii, depths, tile_size, tile_width, tile_height, packed=False,
                             n_images=None, image_ids=None, gaussian_ids=None, conics=None, opacities=None,
                             nnz_device=None):
    """isect_tiles(sort=True) followed by isect_offset_encode, as used by
    rasterization(): returns (tiles_per_gauss, isect_ids, flatten_ids, offsets
    [I, th, tw]). The tile-bucket sort produces the offsets on the way. With
    ``nnz_device`` (packed; a device int64 count) only that many leading rows of
    the capacity-sized splat arrays are intersected."""
    if packed:
        assert gaussian_ids is not None, "gaussian_ids is required if packed is True"
    tiles_per_gauss, isect_ids, flatten_ids, offsets = _isect_tiles(
        means2d, radii, depths, tile_size, tile_width, tile_height, True, packed, n_images, image_ids,
        conics, opacities, nnz_device)
    I = n_images if packed else math.prod(means2d.shape[:-2])
    if offsets is None:
        offsets = isect_offset_encode(isect_ids, I, tile_width, tile_height)
    else:
        offsets = offsets.view(I, tile_height, tile_width)
    return tiles_per_gauss, isect_ids, flatten_ids, offsets


def _isect_tiles(means2d, radii, depths, tile_size, tile_width, tile_height, sort, packed, n_images,
                 image_ids, conics, opacities, nnz_device=None):
    if packed:
        nnz = means2d.size(0)
        assert means2d.shape == (nnz, 2), means2d.shape
        assert radii.shape == (nnz, 2), radii.shape
        assert depths.shape == (nnz,), depths.shape
        if conics is not None:
            assert conics.shape == (nnz, 3), conics.shape
        if opacities is not None:
            assert opacities.shape == (nnz,), opacities.shape
        assert image_ids is not None, "image_ids is required if packed is True"
        assert n_images is not None, "n_images is required if packed is True"
        image_ids = image_ids.contiguous()
        I = n_images
        N = 0
        n = nnz
    else:
        image_dims = means2d.shape[:-2]
        I = math.prod(image_dims)
        N = means2d.shape[-2]
        nnz = 0
        assert means2d.shape == image_dims + (N, 2), means2d.shape
        assert radii.shape == image_dims + (N, 2), radii.shape
        assert depths.shape == image_dims + (N,), depths.shape
        if conics is not None:
            assert conics.shape == image_dims + (N, 3), conics.shape
        if opacities is not None:
            assert opacities.shape == image_dims + (N,), opacities.shape
        n = I * N
    means2d = means2d.contiguous()
    radii = radii.contiguous()
    depths = depths.contiguous()
    conics = conics.contiguous() if conics is not None else None
    opacities = opacities.contiguous() if opacities is not None else None
    if image_ids is not None and image_ids.dtype != torch.int64:
        image_ids = image_ids.long()
    for name, t in (("means2d", means2d), ("radii", radii), ("depths", depths), ("conics", conics),
                    ("opacities", opacities), ("image_ids", image_ids)):
        check_cuda(name, t)
    dev = means2d.device
    tiles_per_gauss = torch.empty(depths.shape, dtype=torch.int32, device=dev)
    if (conics is None) != (opacities is None):
        conics, opacities = None, None  # AccuTile needs both; AABB otherwise
    n_buckets = I * tile_width * tile_height
    with device_guard(dev):
        stream = stream_of(means2d)
        args = (int(packed), I, N, nnz, ptr(image_ids), ptr(means2d), ptr(radii), ptr(depths),
                ptr(conics), ptr(opacities), tile_size, tile_width, tile_height)
        if n == 0:
            empty = torch.empty(0, dtype=torch.int64, device=dev)
            return tiles_per_gauss, empty, torch.empty(0, dtype=torch.int32, device=dev), None
        if not sort:
            call("gsb_isect_count", *args, ptr(tiles_per_gauss), stream)
            cum = _scan_i32(tiles_per_gauss.view(-1))
            n_isects = int(cum[-1].item())
            isect_ids = torch.empty(n_isects, dtype=torch.int64, device=dev)
            flatten_ids = torch.empty(n_isects, dtype=torch.int32, device=dev)
            if n_isects:
                call("gsb_isect_emit", *args, ptr(cum), ptr(isect_ids), ptr(flatten_ids), stream)
            return tiles_per_gauss, isect_ids, flatten_ids, None

        if nnz_device is not None:
            assert packed and sort, "a device splat count needs packed, sorted intersections"
            check_cuda("nnz_device", nnz_device)
        isect_ids, flatten_ids, offsets, _ = _bucket_isect(args, I, tile_width, tile_height,
                                                          tiles_per_gauss, dev, stream, nnz_device=nnz_device)
        return tiles_per_gauss, isect_ids, flatten_ids, offsets


def _sized(n: int, dtype, dev) -> Tensor:
    """An uninitialised 1-D tensor of n elements whose allocation is rounded up
    to the next multiple of 1/16 of n's power of two (at most ~6% more). Buffers
    sized by data-dependent counts (intersections, splats) change size a little
    from step to step; rounded, successive steps request the same sizes and the
    caching allocator serves them from its cache instead of new device
    allocations (which synchronise the device, at multi-GB sizes for many ms)."""
    if n <= 4096:
        return torch.empty(n, dtype=dtype, device=dev)
    step = 1 << max(0, n.bit_length() - 5)
    return torch.empty((n + step - 1) // step * step, dtype=dtype, device=dev)[:n]


def _bucket_isect(args, I, tile_width, tile_height, tiles_per_gauss, dev, stream, nnz_device=None):
    """Sorted intersections through the tile-bucket path: per-splat and
    per-(image, tile) counts, bucket offsets, one host read of (n_isects, largest
    bucket, nnz), bucket emit and on-chip bucket sort. ``args`` are the leading
    arguments of the isect entry points (packed, I, N, nnz, image_ids, means2d,
    radii, depths, conics, opacities, tile_size, tile_width, tile_height). With
    ``nnz_device`` (packed, a device int64 count) the splat arrays have ``nnz``
    rows of capacity and the actual count is read back with the other sizes.
    Returns (isect_ids, flatten_ids, offsets int32 [I * th * tw], nnz or None)."""
    n_buckets = I * tile_width * tile_height
    shards = _B.lib().gsb_isect_bucket_shards(I, tile_width, tile_height)
    shard_counts = torch.empty(n_buckets * shards, dtype=torch.int32, device=dev)
    call("gsb_isect_count_tiles", *args, ptr(nnz_device), ptr(tiles_per_gauss), ptr(shard_counts), stream)
    offsets = torch.empty(n_buckets, dtype=torch.int32, device=dev)
    bucket_sizes = torch.empty(n_buckets, dtype=torch.int32, device=dev)
    cursor = torch.empty(n_buckets * shards, dtype=torch.int32, device=dev)
    totals = torch.empty(5, dtype=torch.int32, device=dev)
    class_list = torch.empty(n_buckets, dtype=torch.int32, device=dev)
    nbytes = _B.lib().gsb_isect_bucket_offsets_scratch_bytes(n_buckets, shards)
    scratch = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    call("gsb_isect_bucket_offsets", ptr(shard_counts), n_buckets, shards, ptr(offsets), ptr(bucket_sizes),
         ptr(cursor), ptr(nnz_device), ptr(totals), ptr(class_list), ptr(scratch), nbytes, stream)
    n_isects, largest, nnz, mid_buckets, large_buckets = (int(v) for v in _B.read_back(totals))
    if n_isects < 0 or nnz < 0:
        raise RuntimeError("isect_tiles: more than 2^31 - 1 tile intersections or splats")
    if nnz_device is None:
        nnz = None
    else:
        args = args[:3] + (nnz,) + args[4:]
    isect_ids = _sized(n_isects, torch.int64, dev)
    flatten_ids = _sized(n_isects, torch.int32, dev)
    if n_isects == 0:
        return isect_ids, flatten_ids, offsets, nnz
    bucket_entries = _sized(n_isects, torch.int64, dev)
    call("gsb_isect_bucket_emit", *args, n_isects, ptr(cursor), ptr(bucket_entries), stream)
    if largest <= _B.lib().gsb_isect_bucket_sort_max():
        call("gsb_isect_bucket_sort", I, tile_width, tile_height, ptr(offsets), ptr(bucket_sizes), largest,
             mid_buckets, large_buckets, ptr(class_list), ptr(bucket_entries), ptr(isect_ids),
             ptr(flatten_ids), stream)
        return isect_ids, flatten_ids, offsets, nnz
    # buckets above the on-chip maximum: split on the device into sub-buckets
    # by their leading (depth, index) bits, each sorted on chip; one more host
    # read tells whether a sub-bucket was still too large (many equal depths)
    nbytes = _B.lib().gsb_isect_bucket_sort_scratch_bytes(n_isects)
    split_scratch = _sized(nbytes, torch.uint8, dev)
    overflow = torch.zeros(1, dtype=torch.int32, device=dev)
    call("gsb_isect_bucket_sort_ex", I, tile_width, tile_height, ptr(offsets), ptr(bucket_sizes), largest,
         mid_buckets, large_buckets, ptr(class_list), ptr(bucket_entries), n_isects, ptr(split_scratch), nbytes,
         ptr(overflow), ptr(isect_ids), ptr(flatten_ids), stream)
    del bucket_entries, split_scratch
    if not int(_B.read_back(overflow)[0]):
        return isect_ids, flatten_ids, offsets, nnz
    # a run of equal depths too large for the on-chip sort: emit in splat order
    # and sort globally (stable LSD radix sort)
    n_live = tiles_per_gauss.numel() if nnz is None else nnz
    cum = _scan_i32(tiles_per_gauss.view(-1)[:n_live])
    call("gsb_isect_emit", *args, ptr(cum), ptr(isect_ids), ptr(flatten_ids), stream)
    isect_ids, flatten_ids = _radix_sort(isect_ids, flatten_ids,
                                         _B.lib().gsb_isect_key_bits(I, tile_width, tile_height))
    return isect_ids, flatten_ids, offsets, nnz


def _radix_sort(keys: Tensor, vals: Tensor, end_bit: int) -> Tuple[Tensor, Tensor]:
    n = keys.numel()
    keys_alt = torch.empty_like(keys)
    vals_alt = torch.empty_like(vals)
    nbytes = _B.lib().gsb_radix_sort_scratch_bytes(n)
    scratch = torch.empty(nbytes, dtype=torch.uint8, device=keys.device)
    which = call("gsb_radix_sort_pairs", ptr(keys), ptr(vals), ptr(keys_alt), ptr(vals_alt), n,
                 end_bit, ptr(scratch), nbytes, stream_of(keys))
    return (keys_alt, vals_alt) if which == 1 else (keys, vals)


@torch.no_grad()
def isect_offset_encode(isect_ids: Tensor, n_images: int, tile_width: int, tile_height: int) -> Tensor:
    """Encodes sorted intersection ids to per-tile offsets [I, th, tw]
    (reference _wrapper.py:806-826)."""
    isect_ids = isect_ids.contiguous()
    check_cuda("isect_ids", isect_ids)
    offsets = torch.empty((n_images, tile_height, tile_width), dtype=torch.int32,
                          device=isect_ids.device)
    with device_guard(isect_ids.device):
        call("gsb_isect_offset_encode", ptr(isect_ids), isect_ids.numel(), n_images, tile_width,
             tile_height, ptr(offsets), stream_of(isect_ids))
    return offsets


# ---------------------------------------------------------------------------
# Rasterization
# ---------------------------------------------------------------------------
def rasterize_to_pixels(
    means2d: Tensor,  # [..., N, 2] or [nnz, 2]
    conics: Tensor,  # [..., N, 3] or [nnz, 3]
    colors: Tensor,  # [..., N, channels] or [nnz, channels]
    opacities: Tensor,  # [..., N] or [nnz]
    image_width: int,
    image_height: int,
    tile_size: int,
    isect_offsets: Tensor,  # [..., tile_height, tile_width]
    flatten_ids: Tensor,  # [n_isects]
    backgrounds: Optional[Tensor] = None,  # [..., channels]
    masks: Optional[Tensor] = None,  # [..., tile_height, tile_width]
    packed: bool = False,
    absgrad: bool = False,
) -> Tuple[Tensor, Tensor]:
    """Rasterizes Gaussians to pixels (reference _wrapper.py:829-961).

    Returns (render_colors [..., H, W, channels], render_alphas [..., H, W, 1]).
    Any channel count >= 1 is rendered directly (no zero padding).
    """
    image_dims = means2d.shape[:-2]
    channels = colors.shape[-1]
    if packed:
        nnz = means2d.size(0)
        assert means2d.shape == (nnz, 2), means2d.shape
        assert conics.shape == (nnz, 3), conics.shape
        assert colors.shape[0] == nnz, colors.shape
        assert opacities.shape == (nnz,), opacities.shape
    else:
        N = means2d.size(-2)
        assert means2d.shape == image_dims + (N, 2), means2d.shape
        assert conics.shape == image_dims + (N, 3), conics.shape
        assert colors.shape == image_dims + (N, channels), colors.shape
        assert opacities.shape == image_dims + (N,), opacities.shape
    if backgrounds is not None:
        if packed:
            # one background per image (isect_offsets' leading dims), or one
            # shared by all images as in the reference's packed check
            img_dims = isect_offsets.shape[:-2]
            if backgrounds.shape == (channels,):
                backgrounds = backgrounds.expand(img_dims + (channels,))
            assert backgrounds.shape == img_dims + (channels,), backgrounds.shape
        else:
            assert backgrounds.shape == image_dims + (channels,), backgrounds.shape
        backgrounds = backgrounds.contiguous()
    if masks is not None:
        assert masks.shape == isect_offsets.shape, masks.shape
        masks = masks.contiguous()
    if channels == 0:
        raise ValueError(f"Unsupported number of color channels: {channels}")
    tile_height, tile_width = isect_offsets.shape[-2:]
    assert (
        tile_height * tile_size >= image_height
    ), f"Assert Failed: {tile_height} * {tile_size} >= {image_height}"
    assert (
        tile_width * tile_size >= image_width
    ), f"Assert Failed: {tile_width} * {tile_size} >= {image_width}"
    return _RasterizeToPixels.apply(
        means2d.contiguous(), conics.contiguous(), colors.contiguous(), opacities.contiguous(),
        backgrounds, masks, image_width, image_height, tile_size, isect_offsets.contiguous(),
        flatten_ids.contiguous(), absgrad)


def rasterize_to_indices_in_range(
    range_start: int,
    range_end: int,
    transmittances: Tensor,  # [..., image_height, image_width]
    means2d: Tensor,  # [..., N, 2]
    conics: Tensor,  # [..., N, 3]
    opacities: Tensor,  # [..., N]
    image_width: int,
    image_height: int,
    tile_size: int,
    isect_offsets: Tensor,  # [..., tile_height, tile_width]
    flatten_ids: Tensor,  # [n_isects]
) -> Tuple[Tensor, Tensor, Tensor]:
    """The (Gaussian, pixel, image) index triples that splat batches
    [range_start, range_end) (front to back, tile_size^2 tile-list entries per
    batch) contribute to each pixel given its current transmittance (reference
    _wrapper.py:1274-1353). Returns gaussian_ids, pixel_ids (row-major) and
    image_ids, int64 [M], grouped by pixel in (image, row, column) order."""
    image_dims = means2d.shape[:-2]
    tile_height, tile_width = isect_offsets.shape[-2:]
    N = means2d.shape[-2]
    assert transmittances.shape == image_dims + (image_height, image_width), transmittances.shape
    assert means2d.shape == image_dims + (N, 2), means2d.shape
    assert conics.shape == image_dims + (N, 3), conics.shape
    assert opacities.shape == image_dims + (N,), opacities.shape
    assert isect_offsets.shape == image_dims + (tile_height, tile_width), isect_offsets.shape
    assert tile_height * tile_size >= image_height, f"Assert Failed: {tile_height} * {tile_size} >= {image_height}"
    assert tile_width * tile_size >= image_width, f"Assert Failed: {tile_width} * {tile_size} >= {image_width}"
    tensors = (transmittances.contiguous(), means2d.contiguous(), conics.contiguous(), opacities.contiguous(),
               isect_offsets.contiguous(), flatten_ids.contiguous())
    for name, t in zip(("transmittances", "means2d", "conics", "opacities", "isect_offsets", "flatten_ids"),
                       tensors):
        check_cuda(name, t)
    trans, m2, con, op, offsets, fids = tensors
    I = math.prod(image_dims)
    dev = means2d.device
    n_isects = fids.numel()
    lo = int(max(0, min(range_start, 2**31 - 1)))
    hi = int(max(0, min(range_end, 2**31 - 1)))
    empty = torch.empty(0, dtype=torch.int64, device=dev)
    if n_isects == 0 or I == 0 or hi <= lo:
        return empty, empty.clone(), empty.clone()
    args = (lo, hi, I, N, n_isects, ptr(m2), ptr(con), ptr(op), image_width, image_height, tile_size,
            tile_width, tile_height, ptr(offsets), ptr(fids), ptr(trans))
    with device_guard(dev):
        stream = stream_of(m2)
        cnts = torch.zeros(I * image_height * image_width, dtype=torch.int32, device=dev)
        call("gsb_rasterize_to_indices", *args, None, ptr(cnts), None, None, stream)
        ends = _scan_i32(cnts)
        total = int(ends[-1].item())
        gaussian_ids = torch.empty(total, dtype=torch.int64, device=dev)
        indices = torch.empty(total, dtype=torch.int64, device=dev)
        if total:
            call("gsb_rasterize_to_indices", *args, ptr(ends), None, ptr(gaussian_ids), ptr(indices), stream)
    hw = image_width * image_height
    return gaussian_ids, indices % hw, torch.div(indices, hw, rounding_mode="floor")


class _RasterizeToPixels(torch.autograd.Function):
    @staticmethod
    def forward(ctx, means2d, conics, colors, opacities, backgrounds, masks, width, height,
                tile_size, isect_offsets, flatten_ids, absgrad):
        for name, t in (("means2d", means2d), ("conics", conics), ("colors", colors),
                        ("opacities", opacities), ("backgrounds", backgrounds), ("masks", masks),
                        ("isect_offsets", isect_offsets), ("flatten_ids", flatten_ids)):
            check_cuda(name, t)
        image_dims = isect_offsets.shape[:-2]
        I = math.prod(image_dims)
        th, tw = isect_offsets.shape[-2:]
        channels = colors.shape[-1]
        dev = means2d.device
        renders = torch.empty(image_dims + (height, width, channels), dtype=torch.float32, device=dev)
        alphas = torch.empty(image_dims + (height, width, 1), dtype=torch.float32, device=dev)
        last_ids = torch.empty(image_dims + (height, width), dtype=torch.int32, device=dev)
        # the forward's final transmittances, kept for the backward (1 - alphas
        # loses the low bits of T in nearly opaque pixels)
        final_Ts = torch.empty(image_dims + (height, width), dtype=torch.float32, device=dev)
        with device_guard(dev):
            call("gsb_rasterize_fwd_ex", I, channels, ptr(means2d), ptr(conics), ptr(colors),
                 ptr(opacities), ptr(backgrounds), ptr(masks), width, height, tile_size, tw, th,
                 ptr(isect_offsets), ptr(flatten_ids), flatten_ids.numel(), ptr(renders),
                 ptr(alphas), ptr(last_ids), ptr(final_Ts), None, stream_of(means2d))
        ctx.save_for_backward(means2d, conics, colors, opacities, backgrounds, masks,
                              isect_offsets, flatten_ids, alphas, last_ids, final_Ts)
        ctx.width = width
        ctx.height = height
        ctx.tile_size = tile_size
        ctx.absgrad = absgrad
        return renders, alphas

    @staticmethod
    def backward(ctx, v_render_colors, v_render_alphas):
        (means2d, conics, colors, opacities, backgrounds, masks, isect_offsets, flatten_ids,
         render_alphas, last_ids, final_Ts) = ctx.saved_tensors
        image_dims = isect_offsets.shape[:-2]
        I = math.prod(image_dims)
        th, tw = isect_offsets.shape[-2:]
        channels = colors.shape[-1]
        v_render_colors = v_render_colors.contiguous()
        v_render_alphas = v_render_alphas.contiguous()
        # the kernel accumulates with atomics: all gradients live in one zeroed
        # buffer (a single fill)
        likes = [means2d, conics, colors, opacities] + ([means2d] if ctx.absgrad else [])
        flat = _sized(sum(t.numel() for t in likes), means2d.dtype, means2d.device).zero_()
        views, off = [], 0
        for t in likes:
            views.append(flat[off:off + t.numel()].view(t.shape))
            off += t.numel()
        v_means2d, v_conics, v_colors, v_opacities = views[:4]
        v_means2d_abs = views[4] if ctx.absgrad else None
        with device_guard(means2d.device):
            call("gsb_rasterize_bwd_ex", I, channels, ptr(means2d), ptr(conics), ptr(colors),
                 ptr(opacities), ptr(backgrounds), ptr(masks), ctx.width, ctx.height,
                 ctx.tile_size, tw, th, ptr(isect_offsets), ptr(flatten_ids), flatten_ids.numel(),
                 ptr(render_alphas), ptr(final_Ts), ptr(last_ids), ptr(v_render_colors),
                 ptr(v_render_alphas),
                 ptr(v_means2d_abs), ptr(v_means2d), ptr(v_conics), ptr(v_colors),
                 ptr(v_opacities), stream_of(means2d))
        if ctx.absgrad:
            means2d.absgrad = v_means2d_abs
        v_backgrounds = None
        if ctx.needs_input_grad[4]:
            v_backgrounds = (v_render_colors * final_Ts[..., None]).sum(dim=(-3, -2))
        return (v_means2d, v_conics, v_colors, v_opacities, v_backgrounds,
                None, None, None, None, None, None, None)


# ---------------------------------------------------------------------------
# Fused projection + SH (used by rasterization())
# ---------------------------------------------------------------------------
def fully_fused_projection_sh(
    means: Tensor,  # [..., N, 3]
    quats: Tensor,  # [..., N, 4]
    scales: Tensor,  # [..., N, 3]
    opacities: Tensor,  # [..., N]
    sh_coeffs: Tensor,  # [..., N, K, 3]
    sh_degree: int,
    viewmats: Tensor,  # [..., C, 4, 4]
    Ks: Tensor,  # [..., C, 3, 3]
    width: int,
    height: int,
    eps2d: float = 0.3,
    near_plane: float = 0.01,
    far_plane: float = 1e10,
    radius_clip: float = 0.0,
    packed: bool = False,
    calc_compensations: bool = False,
    camera_model: CameraModel = "pinhole",
    isect_tiling: Optional[Tuple[int, int, int]] = None,
    defer_count: bool = False,
) -> Tuple[Tensor, ...]:
    """Projection, view-dependent SH colour and opacity compensation in one op.

    Equivalent to fully_fused_projection(..., opacities=opacities) followed by
    colors = clamp_min(spherical_harmonics(sh_degree, normalize(means - campos),
    coeffs) + 0.5, 0) and opacities * compensations, as the reference's
    rasterization() computes them (gsplat/rendering.py:749-872). Returns the
    projection outputs followed by (colors, opacities): dense
    (radii, means2d, depths, conics, compensations, colors, opacities) or packed
    (batch_ids, camera_ids, gaussian_ids, indptr, radii, means2d, depths, conics,
    compensations, colors, opacities). Gradients flow to means, quats, scales,
    opacities and sh_coeffs (not to viewmats).

    With ``packed`` and ``isect_tiling = (tile_size, tile_width, tile_height)``
    the op also runs isect_tiles (AccuTile with the conics and the output
    opacities, sorted) and isect_offset_encode on the projected splats, and
    appends (tiles_per_gauss, isect_ids, flatten_ids, isect_offsets [B*C, th,
    tw]). The splat count then travels to the host together with the
    intersection sizes in one read instead of two.

    With ``packed`` and ``defer_count`` (and no ``isect_tiling``) the packed
    outputs keep B*C*N rows of capacity, their first nnz rows valid, and the
    device-side count ``nnz`` (int64 [1]) is appended: the caller reads it
    together with whatever else it needs from the device.
    """
    batch_dims = means.shape[:-2]
    N = means.shape[-2]
    C = viewmats.shape[-3]
    assert means.shape == batch_dims + (N, 3), means.shape
    assert quats.shape == batch_dims + (N, 4), quats.shape
    assert scales.shape == batch_dims + (N, 3), scales.shape
    assert opacities.shape == batch_dims + (N,), opacities.shape
    assert sh_coeffs.shape[:-2] == batch_dims + (N,) and sh_coeffs.shape[-1] == 3, sh_coeffs.shape
    assert (sh_degree + 1) ** 2 <= sh_coeffs.shape[-2], sh_coeffs.shape
    assert viewmats.shape == batch_dims + (C, 4, 4), viewmats.shape
    assert Ks.shape == batch_dims + (C, 3, 3), Ks.shape
    cam = _camera_id(camera_model)
    return _FullyFusedProjectionSH.apply(
        means.contiguous(), quats.contiguous(), scales.contiguous(), opacities.contiguous(),
        sh_coeffs.contiguous(), sh_degree, viewmats.contiguous(), Ks.contiguous(), width, height,
        eps2d, near_plane, far_plane, radius_clip, packed, calc_compensations, cam,
        isect_tiling if packed else None, bool(packed and defer_count and isect_tiling is None))


class _FullyFusedProjectionSH(torch.autograd.Function):
    @staticmethod
    def forward(ctx, means, quats, scales, opacities, sh, sh_degree, viewmats, Ks, width, height,
                eps2d, near_plane, far_plane, radius_clip, packed, calc_compensations, camera_model,
                isect_tiling, defer_count):
        # outputs without a gradient (ids, radii, depths, intersections) reach the
        # backward as None instead of zero-filled tensors
        ctx.set_materialize_grads(False)
        for name, t in (("means", means), ("quats", quats), ("scales", scales),
                        ("opacities", opacities), ("sh_coeffs", sh), ("viewmats", viewmats),
                        ("Ks", Ks)):
            check_cuda(name, t)
        batch_dims = means.shape[:-2]
        N = means.shape[-2]
        C = viewmats.shape[-3]
        B = math.prod(batch_dims)
        K = sh.shape[-2]
        dev = means.device
        f32 = means.dtype
        shared = (B, C, N, ptr(means), ptr(quats), ptr(scales), ptr(opacities), ptr(sh), K,
                  sh_degree, ptr(viewmats), ptr(Ks), width, height, eps2d, near_plane, far_plane,
                  radius_clip, int(calc_compensations), camera_model)
        with device_guard(dev):
            stream = stream_of(means)
            if not packed:
                radii = torch.empty(batch_dims + (C, N, 2), dtype=torch.int32, device=dev)
                means2d = torch.empty(batch_dims + (C, N, 2), dtype=f32, device=dev)
                depths = torch.empty(batch_dims + (C, N), dtype=f32, device=dev)
                conics = torch.empty(batch_dims + (C, N, 3), dtype=f32, device=dev)
                comps = torch.empty(batch_dims + (C, N), dtype=f32, device=dev) if calc_compensations else None
                colors = torch.empty(batch_dims + (C, N, 3), dtype=f32, device=dev)
                opac_out = torch.empty(batch_dims + (C, N), dtype=f32, device=dev)
                call("gsb_projection_sh_dense_fwd", *shared, ptr(radii), ptr(means2d), ptr(depths),
                     ptr(conics), ptr(comps), ptr(colors), ptr(opac_out), stream)
                pair_index = None
                outs = (radii, means2d, depths, conics, comps, colors, opac_out)
            else:
                nblocks = _B.lib().gsb_projection_packed_blocks(N)
                block_cnts = torch.empty(B * C * nblocks, dtype=torch.int32, device=dev)
                vis_bits = torch.empty(B * C * nblocks * 8, dtype=torch.int32, device=dev)
                call("gsb_projection_packed_count", B, C, N, ptr(means), None, ptr(quats),
                     ptr(scales), ptr(opacities), ptr(viewmats), ptr(Ks), width, height, eps2d,
                     near_plane, far_plane, radius_clip, int(calc_compensations), camera_model,
                     ptr(block_cnts), ptr(vis_bits), stream)
                block_accum = _scan_i32(block_cnts)
                deferred = (isect_tiling is not None or defer_count) and block_accum.numel() > 0
                if deferred:
                    # capacity rows; the count stays on the device until the
                    # intersection sizes are read
                    nnz = B * C * N
                else:
                    nnz = int(block_accum[-1].item()) if block_accum.numel() > 0 else 0
                indptr = torch.zeros(B * C + 1, dtype=torch.int32, device=dev)
                batch_ids = torch.empty(nnz, dtype=torch.int64, device=dev)
                camera_ids = torch.empty(nnz, dtype=torch.int64, device=dev)
                gaussian_ids = torch.empty(nnz, dtype=torch.int64, device=dev)
                radii = torch.empty((nnz, 2), dtype=torch.int32, device=dev)
                means2d = torch.empty((nnz, 2), dtype=f32, device=dev)
                depths = torch.empty(nnz, dtype=f32, device=dev)
                conics = torch.empty((nnz, 3), dtype=f32, device=dev)
                comps = torch.empty(nnz, dtype=f32, device=dev) if calc_compensations else None
                colors = torch.empty((nnz, 3), dtype=f32, device=dev)
                opac_out = torch.empty(nnz, dtype=f32, device=dev)
                pair_index = torch.empty(B * C * N, dtype=torch.int32, device=dev)
                if block_accum.numel() > 0:
                    call("gsb_projection_sh_packed_write", *shared, ptr(vis_bits), ptr(block_accum),
                         nnz, ptr(indptr), ptr(batch_ids), ptr(camera_ids), ptr(gaussian_ids),
                         ptr(radii), ptr(means2d), ptr(depths), ptr(conics), ptr(comps),
                         ptr(colors), ptr(opac_out), ptr(pair_index), stream)
                outs = (batch_ids, camera_ids, gaussian_ids, indptr, radii, means2d, depths, conics,
                        comps, colors, opac_out)
                if isect_tiling is not None:
                    tile_size, tile_width, tile_height = isect_tiling
                    I = B * C
                    tiles_per_gauss = torch.empty(nnz, dtype=torch.int32, device=dev)
                    if nnz == 0:
                        isect = (torch.empty(0, dtype=torch.int64, device=dev),
                                 torch.empty(0, dtype=torch.int32, device=dev),
                                 torch.zeros(I * tile_width * tile_height, dtype=torch.int32, device=dev))
                    else:
                        image_ids = camera_ids if B == 1 else batch_ids * C + camera_ids
                        args = (1, I, 0, nnz, ptr(image_ids), ptr(means2d), ptr(radii), ptr(depths),
                                ptr(conics), ptr(opac_out), tile_size, tile_width, tile_height)
                        *isect, nnz = _bucket_isect(args, I, tile_width, tile_height, tiles_per_gauss,
                                                    dev, stream, nnz_device=block_accum[-1:])
                        outs = tuple(t[:nnz] if t is not None and t is not indptr else t for t in outs)
                        tiles_per_gauss = tiles_per_gauss[:nnz]
                    isect_offsets = isect[2].view(I, tile_height, tile_width)
                    outs = outs + (tiles_per_gauss, isect[0], isect[1], isect_offsets)
                elif defer_count:
                    nnz_dev = block_accum[-1:] if deferred else torch.zeros(1, dtype=torch.int64, device=dev)
                    outs = outs + (nnz_dev,)
                (batch_ids, camera_ids, gaussian_ids, indptr, radii, means2d, depths, conics, comps,
                 colors, opac_out) = outs[:11]
                ctx.mark_non_differentiable(batch_ids, camera_ids, gaussian_ids, indptr, radii, *outs[11:])
        if not packed:
            ctx.mark_non_differentiable(radii)
        ctx.save_for_backward(means, quats, scales, opacities, sh, viewmats, Ks, pair_index,
                              None if packed else radii, conics, comps)
        ctx.meta = (B, C, N, K, sh_degree, width, height, eps2d, calc_compensations, camera_model,
                    packed)
        return outs

    @staticmethod
    def backward(ctx, *grads):
        means, quats, scales, opacities, sh, viewmats, Ks, pair_index, radii, conics, comps = ctx.saved_tensors
        B, C, N, K, deg, width, height, eps2d, calc, cam, packed = ctx.meta
        if packed:
            _, _, _, _, _, v_means2d, v_depths, v_conics, v_comps, v_colors, v_opac = grads[:11]
        else:
            _, v_means2d, v_depths, v_conics, v_comps, v_colors, v_opac = grads

        def c(t, like):
            return torch.zeros_like(like) if t is None else t.contiguous()

        v_means2d = c(v_means2d, conics[..., :2])
        v_depths = v_depths.contiguous() if v_depths is not None else None  # the kernel reads None as 0
        v_conics = c(v_conics, conics)
        v_colors = c(v_colors, conics)
        v_opac = c(v_opac, conics[..., 0])
        v_comps = v_comps.contiguous() if (calc and v_comps is not None) else None
        v_means = torch.empty_like(means)
        v_quats = torch.empty_like(quats)
        v_scales = torch.empty_like(scales)
        v_opacities = torch.empty_like(opacities)
        v_sh = torch.empty_like(sh)
        with device_guard(means.device):
            call("gsb_projection_sh_bwd", B, C, N, int(packed), ptr(means), ptr(quats), ptr(scales),
                 ptr(opacities), ptr(sh), K, deg, ptr(viewmats), ptr(Ks), width, height, eps2d,
                 int(calc), cam, ptr(pair_index), ptr(radii), ptr(conics), ptr(comps),
                 ptr(v_means2d), ptr(v_depths), ptr(v_conics), ptr(v_comps), ptr(v_colors),
                 ptr(v_opac), ptr(v_means), ptr(v_quats), ptr(v_scales), ptr(v_opacities),
                 ptr(v_sh), stream_of(means))
        return (v_means, v_quats, v_scales, v_opacities, v_sh, None, None, None, None, None, None,
                None, None, None, None, None, None, None, None)
