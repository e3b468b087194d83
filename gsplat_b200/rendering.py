"""``rasterization()``: the 3D Gaussian splatting render call, forward + backward.

Drop-in for the reference's ``gsplat/rendering.py:256-1273`` for the 3DGS pinhole /
orthographic / fisheye path: same keyword arguments and defaults, same return value
``(render_colors, render_alphas, meta)`` and the same ``meta`` keys, so
densification strategies that read ``meta["means2d"].grad`` / ``.absgrad`` work
unchanged. The stages are the ops of ``gsplat_b200.cuda._wrapper`` (projection,
SH, tile intersection + sort + offsets, rasterization); the multi-GPU mode shards
Gaussians and sends projected splats to the rank that owns their camera, like the
reference (``rendering.py:689-706, 907-1022``), through peer memory on one node
(or an NCCL all-to-all).

Options that belong to other pipelines of the reference (3DGUT ``with_ut``,
``with_eval3d``, lidar, distortion, rolling shutter) raise ``NotImplementedError``.
"""

import math
from typing import Dict, Optional, Tuple

import torch
import torch.nn.functional as F
from torch import Tensor
from typing_extensions import Literal

from .cuda._wrapper import (
    fully_fused_projection,
    fully_fused_projection_sh,
    isect_tiles_with_offsets,
    rasterize_to_pixels,
    spherical_harmonics,
)
from .cuda import _backend as _B
from .cuda._backend import call, device_guard, ptr, stream_of
from .distributed import (
    PeerExchange,
    peer_exchange_available,
    peer_exchange_rows,
    all_gather_tensor_list,
    all_to_all_int32,
    all_to_all_tensor_list,
    exchange_rows,
    pack_rows,
)

RenderMode = Literal["RGB", "d", "Ed", "D", "ED", "RGB-d", "RGB-Ed", "RGB+D", "RGB+ED"]
RasterizeMode = Literal["classic", "antialiased"]


def render_mode_has_color(mode) -> bool:
    return mode in {"RGB", "RGB-d", "RGB-Ed", "RGB+D", "RGB+ED"}


def render_mode_has_hit_distance(mode) -> bool:
    return mode in {"d", "Ed", "RGB-d", "RGB-Ed"}


def render_mode_has_depth(mode) -> bool:
    return mode in {"D", "ED", "RGB+D", "RGB+ED"}


def render_mode_has_expected_depth(mode) -> bool:
    return mode in {"Ed", "ED", "RGB-Ed", "RGB+ED"}


def render_mode_has_depth_channel(mode) -> bool:
    return render_mode_has_depth(mode) or render_mode_has_hit_distance(mode)


def viewmat_to_camera_position(viewmats: Tensor) -> Tensor:
    """Camera centre -R^T t of a world-to-camera matrix (reference rendering.py:214-224)."""
    R = viewmats[..., :3, :3]
    t = viewmats[..., :3, 3]
    return -(R.mT @ t.unsqueeze(-1)).squeeze(-1)


def compute_directions(batch_dims, means, viewmats, batch_ids=None, camera_ids=None,
                       gaussian_ids=None, indptr=None) -> Tensor:
    """Unit view directions from each camera to each Gaussian
    (reference rendering.py:95-167, 227-253)."""
    campos = viewmat_to_camera_position(viewmats)
    if gaussian_ids is None:
        dirs = means[..., None, :, :] - campos[..., None, :]
    else:
        B = math.prod(batch_dims)
        N = means.shape[-2]
        C = campos.shape[-2]
        means_flat = means.reshape(B, N, 3)
        campos_flat = campos.reshape(B, C, 3)
        if B * C == 1:
            dirs = means_flat[0, gaussian_ids] - campos_flat[0, 0]
        else:
            dirs = means_flat[batch_ids, gaussian_ids] - campos_flat[batch_ids, camera_ids]
    return F.normalize(dirs, p=2, dim=-1)


def normalize_features_layout(features, batch_dims, C, trailing_dims, batch_ids=None,
                              camera_ids=None, feature_ids=None) -> Tensor:
    """Per-view or per-Gaussian features to [nnz, *t] (packed) or [..., C, N, *t]
    (reference rendering.py:170-213)."""
    B = math.prod(batch_dims)
    N = features.shape[-(len(trailing_dims) + 1)]
    if features.shape == batch_dims + (C, N) + tuple(trailing_dims):
        if feature_ids is not None:
            return features.reshape(B, C, N, *trailing_dims)[batch_ids, camera_ids, feature_ids]
        return features
    assert features.shape == (*batch_dims, N, *trailing_dims)
    if feature_ids is not None:
        return features.reshape(B, N, *trailing_dims)[batch_ids, feature_ids]
    return torch.broadcast_to(features.unsqueeze(len(batch_dims)), batch_dims + (C, N, *trailing_dims))


def _trim_local_meta(meta: Dict, n: int) -> None:
    """Distributed packed mode: the local projection outputs in ``meta`` have
    the projection's capacity rows, of which the first ``n`` (the local splat
    count, known on the host once the sizes are read) are set; keep those, like
    the reference's exact-size outputs. ``means2d`` enters the exchange at full
    capacity, so ``meta["means2d"]`` becomes a leaf view of its first ``n`` rows
    whose ``.grad`` is filled from the capacity tensor's gradient when the
    backward reaches it: what a densification strategy reads after
    ``retain_grad()`` and ``backward()``."""
    for k in ("batch_ids", "camera_ids", "gaussian_ids", "radii", "depths", "conics", "opacities"):
        t = meta.get(k)
        if t is not None:
            meta[k] = t[:n]
    m = meta.get("means2d")
    if m is None:
        return
    view = m.detach()[:n]
    if m.requires_grad:
        view.requires_grad_(True)

        def tap(grad):
            piece = grad[:n].clone()
            view.grad = piece if view.grad is None else view.grad + piece

        m.register_hook(tap)
    meta["means2d"] = view


def _camera_major(C: int, rows: Tensor, N_world) -> Tensor:
    """Rows received from every rank, in rank order, each rank r sending a
    camera-major block of C x N_r rows, rearranged into [C, sum_r N_r, ...]: camera
    c holds rank 0's Gaussians, then rank 1's, ... (one gather)."""
    counts = torch.as_tensor([int(n) for n in N_world], dtype=torch.int64, device=rows.device)
    first = torch.cumsum(counts, 0) - counts  # first global Gaussian of each rank
    block = first * C  # first received row of each rank's block
    owner = torch.repeat_interleave(torch.arange(len(N_world), device=rows.device), counts)
    local = torch.arange(owner.numel(), device=rows.device) - first[owner]
    cam = torch.arange(C, device=rows.device)[:, None]
    src = block[owner][None] + cam * counts[owner][None] + local[None]  # [C, sum_r N_r]
    return rows[src.reshape(-1)].reshape((C, owner.numel()) + rows.shape[1:])


def rasterization(
    means: Tensor,  # [..., N, 3]
    quats: Tensor,  # [..., N, 4]
    scales: Tensor,  # [..., N, 3]
    opacities: Tensor,  # [..., N]
    colors: Optional[Tensor],  # [..., (C,) N, D] or [..., (C,) N, K, 3]
    viewmats: Tensor,  # [..., C, 4, 4]
    Ks: Tensor,  # [..., C, 3, 3]
    width: int,
    height: int,
    near_plane: float = 0.01,
    far_plane: float = 1e10,
    radius_clip: float = 0.0,
    eps2d: float = 0.3,
    sh_degree: Optional[int] = None,
    packed: bool = True,
    tile_size: int = 16,
    backgrounds: Optional[Tensor] = None,
    render_mode: RenderMode = "RGB",
    sparse_grad: bool = False,
    absgrad: bool = False,
    rasterize_mode: RasterizeMode = "classic",
    channel_chunk: int = 32,
    distributed: bool = False,
    camera_model: str = "pinhole",
    segmented: bool = False,
    covars: Optional[Tensor] = None,
    with_ut: bool = False,
    with_eval3d: bool = False,
    return_normals: bool = False,
    global_z_order: bool = True,
    rays: Optional[Tensor] = None,
    radial_coeffs: Optional[Tensor] = None,
    tangential_coeffs: Optional[Tensor] = None,
    thin_prism_coeffs: Optional[Tensor] = None,
    ftheta_coeffs=None,
    lidar_coeffs=None,
    external_distortion_coeffs=None,
    rolling_shutter=None,
    viewmats_rs: Optional[Tensor] = None,
    ut_params=None,
    extra_signals: Optional[Tensor] = None,
    extra_signals_sh_degree: Optional[int] = None,
) -> Tuple[Tensor, Tensor, Dict]:
    """Rasterizes N 3D Gaussians into C images (reference rendering.py:256-1273).

    Returns ``(render_colors [..., C, H, W, X], render_alphas [..., C, H, W, 1],
    meta)`` where X is D for "RGB", 1 for "D"/"ED", D+1 for "RGB+D"/"RGB+ED".
    """
    unsupported = {
        "with_ut": with_ut,
        "with_eval3d": with_eval3d,
        "return_normals": return_normals,
        "rays": rays is not None,
        "radial_coeffs": radial_coeffs is not None,
        "tangential_coeffs": tangential_coeffs is not None,
        "thin_prism_coeffs": thin_prism_coeffs is not None,
        "ftheta_coeffs": ftheta_coeffs is not None,
        "lidar_coeffs": lidar_coeffs is not None,
        "external_distortion_coeffs": external_distortion_coeffs is not None,
        "viewmats_rs": viewmats_rs is not None,
        "ut_params": ut_params is not None,
        "global_z_order=False": not global_z_order,
        "hit-distance render modes": render_mode_has_hit_distance(render_mode),
    }
    if rolling_shutter is not None and int(rolling_shutter) != 4:  # 4 = GLOBAL
        unsupported["rolling_shutter"] = True
    bad = [k for k, v in unsupported.items() if v]
    if bad:
        raise NotImplementedError(f"gsplat_b200.rasterization does not implement: {', '.join(bad)}")

    meta: Dict = {}
    has_color = render_mode_has_color(render_mode)
    if colors is None and has_color:
        raise ValueError(
            f"colors must be provided when render_mode='{render_mode}' includes RGB. "
            f"Pass colors=None only for depth-only render modes (D, d, Ed, ED)."
        )
    if colors is None and sh_degree is not None:
        raise ValueError(f"sh_degree must be None when colors is None, got sh_degree={sh_degree}.")

    batch_dims = means.shape[:-2]
    num_batch_dims = len(batch_dims)
    B = math.prod(batch_dims)
    N = means.shape[-2]
    C = viewmats.shape[-3]
    D = colors.shape[-1] if has_color else 0
    I = B * C
    device = means.device
    assert means.shape == batch_dims + (N, 3), means.shape
    if covars is None:
        assert quats.shape == batch_dims + (N, 4), quats.shape
        assert scales.shape == batch_dims + (N, 3), scales.shape
    else:
        assert covars.shape == batch_dims + (N, 3, 3), covars.shape
        quats, scales = None, None
        tri = ([0, 0, 0, 1, 1, 2], [0, 1, 2, 1, 2, 2])
        covars = covars[..., tri[0], tri[1]]
    assert opacities.shape == batch_dims + (N,), opacities.shape
    assert viewmats.shape == batch_dims + (C, 4, 4), viewmats.shape
    assert Ks.shape == batch_dims + (C, 3, 3), Ks.shape

    def check_features(features: Tensor, deg: Optional[int], name: str) -> None:
        channels = features.shape[-1]
        if deg is None:
            assert (
                features.dim() == num_batch_dims + 2 and features.shape[:-1] == (*batch_dims, N)
            ) or (
                features.dim() == num_batch_dims + 3 and features.shape[:-1] == (*batch_dims, C, N)
            ), f"{name}'s shape {features.shape=} must be either {(*batch_dims, N, channels)} or {(*batch_dims, C, N, channels)}"
            if distributed:
                assert features.dim() == num_batch_dims + 2, f"Distributed mode only supports per-Gaussian {name}."
        else:
            assert (
                features.dim() == num_batch_dims + 3
                and features.shape[:-2] == batch_dims + (N,)
                and channels == 3
            ) or (
                features.dim() == num_batch_dims + 4
                and features.shape[:-2] == batch_dims + (C, N)
                and channels == 3
            ), f"{name}'s shape {features.shape=} must be either {(*batch_dims, N, 3)} or {(*batch_dims, C, N, 3)}"
            assert (deg + 1) ** 2 <= features.shape[-2], features.shape
            if distributed:
                assert features.dim() == num_batch_dims + 3, f"Distributed mode only supports per-Gaussian {name}."

    if has_color:
        check_features(colors, sh_degree, "colors")
    if extra_signals is not None:
        check_features(extra_signals, extra_signals_sh_degree, "extra signals")
    if absgrad:
        assert not distributed, "AbsGrad is not supported in distributed mode."

    n_world_event = None  # pinned copy of the gathered Gaussian counts (peer exchange)
    if distributed:
        assert batch_dims == (), "Distributed mode does not support batch dimensions"
        world_rank = torch.distributed.get_rank()
        world_size = torch.distributed.get_world_size()
        # Gaussian counts of all ranks, kept on the device (read only by the
        # paths that need host split sizes)
        C_world = [C] * world_size
        if viewmats.requires_grad or Ks.requires_grad:
            N_world_dev = torch.empty(world_size, dtype=torch.int64, device=device)
            torch.distributed.all_gather_into_tensor(
                N_world_dev, torch.full((1,), N, dtype=torch.int64, device=device))
            viewmats, Ks = all_gather_tensor_list(world_size, [viewmats, Ks])
        else:
            # one all-gather for the cameras and the Gaussian count of every rank
            # (the int64 count travels bit-cast in the first two float32 slots of
            # each row; copied out before the bit-cast, since a one-row slice
            # already counts as contiguous but keeps the odd row stride)
            n_bits = torch.full((C, 1), N, dtype=torch.int64, device=viewmats.device).view(torch.float32)
            row = torch.cat([n_bits, viewmats.reshape(C, 16).float(), Ks.reshape(C, 9).float()],
                            dim=1).contiguous()
            gathered = torch.empty((world_size * C, 27), dtype=row.dtype, device=row.device)
            torch.distributed.all_gather_into_tensor(gathered, row)
            viewmats = gathered[:, 2:18].reshape(world_size * C, 4, 4).to(viewmats.dtype)
            Ks = gathered[:, 18:27].reshape(world_size * C, 3, 3).to(Ks.dtype)
            N_world_dev = gathered[::C, 0:2].clone(memory_format=torch.contiguous_format).view(
                torch.int64).reshape(world_size)
        C = len(viewmats)
        if packed and peer_exchange_available(device):
            # the Gaussian counts size the peer exchange: copied to pinned host
            # memory now and waited for only at the exchange, so the projection
            # kernels queued meanwhile keep the GPU busy
            n_world_pinned = torch.empty(world_size, dtype=torch.int64, pin_memory=True)
            n_world_pinned.copy_(N_world_dev, non_blocking=True)
            n_world_event = torch.cuda.Event()
            n_world_event.record()

    # One fused kernel for projection + view-dependent SH colour + opacity
    # compensation when the colours are per-Gaussian SH coefficients; the general
    # op-by-op path otherwise (per-view colours, covariances, extra signals,
    # pose gradients).
    use_fused = (
        has_color
        and sh_degree is not None
        and covars is None
        and extra_signals is None
        and colors.dim() == num_batch_dims + 3
        and colors.shape[-2] <= 64
        and sh_degree <= 4
        and camera_model in ("pinhole", "ortho", "fisheye")
        and not viewmats.requires_grad
    )
    compensations = None
    nnz_device = None  # device splat count of capacity-sized packed outputs (distributed)
    peer_nnz = None  # device count of the rows received by the peer exchange (capacity-sized tensors)
    tile_width = math.ceil(width / float(tile_size))
    tile_height = math.ceil(height / float(tile_size))
    isect = None  # (tiles_per_gauss, isect_ids, flatten_ids, isect_offsets) when done by the projection
    if use_fused:
        # packed and not distributed: the projection op also intersects the tiles,
        # so the splat count and the intersection sizes reach the host in one read
        # distributed + packed: the splat count stays on the device until it is read
        # together with the exchange counts
        fuse_isect = packed and not distributed
        defer_count = packed and distributed
        proj = fully_fused_projection_sh(
            means, quats, scales, opacities, colors, sh_degree, viewmats, Ks, width, height,
            eps2d=eps2d, near_plane=near_plane, far_plane=far_plane, radius_clip=radius_clip,
            packed=packed, calc_compensations=(rasterize_mode == "antialiased"),
            camera_model=camera_model,
            isect_tiling=(tile_size, tile_width, tile_height) if fuse_isect else None,
            defer_count=defer_count)
        if packed:
            (batch_ids, camera_ids, gaussian_ids, indptr, radii, means2d, depths, conics,
             _, proj_features, opacities) = proj[:11]
            if fuse_isect:
                isect = proj[11:]
            if defer_count:
                nnz_device = proj[11]
            image_ids = camera_ids if B == 1 else batch_ids * C + camera_ids
        else:
            radii, means2d, depths, conics, _, proj_features, opacities = proj
            indptr, batch_ids, camera_ids, gaussian_ids = None, None, None, None
            image_ids = None
    else:
        proj = fully_fused_projection(
            means, covars, quats, scales, viewmats, Ks, width, height, eps2d=eps2d, packed=packed,
            near_plane=near_plane, far_plane=far_plane, radius_clip=radius_clip,
            sparse_grad=sparse_grad, calc_compensations=(rasterize_mode == "antialiased"),
            camera_model=camera_model, opacities=opacities)
        if packed:
            (batch_ids, camera_ids, gaussian_ids, indptr, radii, means2d, depths, conics,
             compensations) = proj
            opacities = opacities.reshape(B, N)[batch_ids, gaussian_ids]
            image_ids = batch_ids * C + camera_ids
        else:
            radii, means2d, depths, conics, compensations = proj
            opacities = torch.broadcast_to(opacities[..., None, :], batch_dims + (C, N))
            indptr, batch_ids, camera_ids, gaussian_ids = None, None, None, None
            image_ids = None
        if compensations is not None:
            opacities = opacities * compensations

    meta.update(
        {
            "batch_ids": batch_ids,
            "camera_ids": camera_ids,
            "gaussian_ids": gaussian_ids,
            "radii": radii,
            "means2d": means2d,
            "depths": depths,
            "conics": conics,
            "opacities": opacities,
        }
    )

    if use_fused:
        pass
    elif sh_degree is None and extra_signals_sh_degree is None:
        feature_list = []
        if has_color:
            feature_list.append(colors)
        if extra_signals is not None:
            feature_list.append(extra_signals)
        proj_features = None
        if feature_list:
            proj_features = torch.cat(feature_list, dim=-1) if len(feature_list) > 1 else feature_list[0]
            proj_features = normalize_features_layout(
                proj_features, batch_dims, C, proj_features.shape[-1:], batch_ids, camera_ids,
                gaussian_ids)
    else:
        colors_sh_degree = sh_degree if has_color else None
        dirs = compute_directions(batch_dims, means, viewmats, batch_ids, camera_ids, gaussian_ids,
                                  indptr)
        feature_list = []
        if has_color:
            tail = colors.shape[-2:] if colors_sh_degree is not None else colors.shape[-1:]
            colors = normalize_features_layout(colors, batch_dims, C, tail, batch_ids, camera_ids,
                                               gaussian_ids)
            if colors_sh_degree is not None:
                colors = spherical_harmonics(colors_sh_degree, dirs, colors,
                                             masks=(radii > 0).all(dim=-1))
                colors = torch.clamp_min(colors + 0.5, 0.0)
            feature_list.append(colors)
        if extra_signals is not None:
            tail = (extra_signals.shape[-2:] if extra_signals_sh_degree is not None
                    else extra_signals.shape[-1:])
            extra_signals = normalize_features_layout(extra_signals, batch_dims, C, tail, batch_ids,
                                                      camera_ids, gaussian_ids)
            if extra_signals_sh_degree is not None:
                extra_signals = spherical_harmonics(extra_signals_sh_degree, dirs, extra_signals,
                                                    masks=(radii > 0).all(dim=-1))
                extra_signals = extra_signals + 0.5
            feature_list.append(extra_signals)
        proj_features = None
        if feature_list:
            proj_features = torch.cat(feature_list, dim=-1) if len(feature_list) > 1 else feature_list[0]

    if distributed and packed and nnz_device is not None:
        # Same exchange as the reference (below), through peer memory or with one
        # host read and one all-to-all: packed rows are ordered by camera, so
        # the rows for rank r are indptr[cstart[r]] .. indptr[cstart[r + 1]].
        # every rank holds C_world[0] cameras (the same count is gathered above)
        bounds = indptr[::C_world[0]].to(torch.int64)
        if n_world_event is None:
            send_cnt = bounds[1:] - bounds[:-1]
            recv_cnt = torch.empty_like(send_cnt)
            torch.distributed.all_to_all_single(recv_cnt, send_cnt)
        # Before the sizes reach the host: camera ids local to the destination
        # rank, gaussian ids shifted by the destination's Gaussian offset
        # (reference rendering.py:944-959), and the send buffer, all bounded by
        # the splat count still on the device. The projection outputs keep their
        # spare rows: only the first nnz are sent, and the projection's backward
        # reads no gradient row past them.
        cap = camera_ids.shape[0]
        cam_local = torch.empty_like(camera_ids)
        gid_global = torch.empty_like(gaussian_ids)
        with device_guard(device):
            call("gsb_exchange_ids", cap, ptr(nnz_device), ptr(camera_ids), ptr(gaussian_ids), C_world[0],
                 ptr(N_world_dev), ptr(cam_local), ptr(gid_global), stream_of(camera_ids))
        floats = [means2d, depths, conics, opacities] + ([proj_features] if proj_features is not None else [])
        ints = [radii, cam_local, gid_global]
    peer_out = None
    if distributed and packed and nnz_device is not None and n_world_event is not None:
        # peer-memory exchange: rows stored straight into the other GPUs'
        # buffers; the received count stays on the device and reaches the host
        # with the intersection sizes
        _B.wait_event(n_world_event)
        # the local splat count, for meta: read with the intersection sizes
        local_nnz = torch.empty(1, dtype=torch.int64, pin_memory=True)
        local_nnz.copy_(nnz_device.reshape(1), non_blocking=True)
        peer_out = peer_exchange_rows(floats, ints, nnz_device, bounds, N_world_dev, n_world_pinned.tolist(),
                                      C_world[0])
        if peer_out is None:  # peer memory unavailable on some rank: the all-to-all below
            send_cnt = bounds[1:] - bounds[:-1]
            recv_cnt = torch.empty_like(send_cnt)
            torch.distributed.all_to_all_single(recv_cnt, send_cnt)
    if peer_out is not None:
        floats, ints, peer_nnz = peer_out
        means2d, depths, conics, opacities = floats[:4]
        if proj_features is not None:
            proj_features = floats[4]
        radii, camera_ids, gaussian_ids = ints
        batch_ids = torch.zeros_like(camera_ids)
        C = C_world[world_rank]
        image_ids = camera_ids
        I = B * C
    elif distributed and packed and nnz_device is not None:
        send_buf = pack_rows(floats, ints, cap, rows_device=nnz_device)
        sizes = _B.read_back(torch.cat([send_cnt, recv_cnt, nnz_device.to(torch.int64)]))
        send_splits, recv_splits, nnz = sizes[:world_size], sizes[world_size:2 * world_size], sizes[-1]
        batch_ids, camera_ids, gaussian_ids = batch_ids[:nnz], camera_ids[:nnz], gaussian_ids[:nnz]
        _trim_local_meta(meta, nnz)
        floats, ints = exchange_rows(world_size, floats, ints, send_splits, recv_splits, packed=send_buf)
        means2d, depths, conics, opacities = floats[:4]
        if proj_features is not None:
            proj_features = floats[4]
        radii, camera_ids, gaussian_ids = ints
        C = C_world[world_rank]
        image_ids = camera_ids
        I = B * C
    elif distributed:
        N_world = _B.read_back(N_world_dev)
        if packed:
            cnts = torch.bincount(camera_ids, minlength=C)
            cnts = cnts.split(C_world, dim=0)
            cnts = [c.sum() for c in cnts]
            collected_splits = all_to_all_int32(world_size, cnts, device=device)
            (radii,) = all_to_all_tensor_list(world_size, [radii], cnts, output_splits=collected_splits)
            tensors = [means2d, depths, conics, opacities]
            if proj_features is not None:
                tensors.append(proj_features)
            out = all_to_all_tensor_list(world_size, tensors, cnts, output_splits=collected_splits)
            means2d, depths, conics, opacities = out[:4]
            if proj_features is not None:
                proj_features = out[4]
            offsets = torch.tensor([0] + C_world[:-1], device=device, dtype=camera_ids.dtype)
            offsets = torch.cumsum(offsets, dim=0).repeat_interleave(torch.stack(cnts))
            camera_ids = camera_ids - offsets
            offsets = torch.tensor([0] + N_world[:-1], device=device, dtype=gaussian_ids.dtype)
            offsets = torch.cumsum(offsets, dim=0).repeat_interleave(torch.stack(cnts))
            gaussian_ids = gaussian_ids + offsets
            camera_ids, gaussian_ids = all_to_all_tensor_list(
                world_size, [camera_ids, gaussian_ids], cnts, output_splits=collected_splits)
            C = C_world[world_rank]
            image_ids = camera_ids
        else:
            C = C_world[world_rank]
            splits = [C_i * N for C_i in C_world]
            out_splits = [C * N_i for N_i in N_world]
            (radii,) = all_to_all_tensor_list(world_size, [radii.flatten(0, 1)], splits=splits,
                                              output_splits=out_splits)
            radii = _camera_major(C, radii, N_world)
            tensors = [means2d.flatten(0, 1), depths.flatten(0, 1), conics.flatten(0, 1),
                       opacities.flatten(0, 1)]
            if proj_features is not None:
                tensors.append(proj_features.flatten(0, 1))
            out = all_to_all_tensor_list(world_size, tensors, splits=splits, output_splits=out_splits)
            means2d, depths, conics, opacities = [_camera_major(C, t, N_world) for t in out[:4]]
            if proj_features is not None:
                proj_features = _camera_major(C, out[4], N_world)
        I = B * C

    if render_mode_has_depth_channel(render_mode):
        depth_channel = depths[..., None]
        if proj_features is not None:
            proj_features = torch.cat((proj_features, depth_channel), dim=-1)
            if backgrounds is not None:
                backgrounds = torch.cat(
                    [backgrounds, torch.zeros((*batch_dims, C, 1), device=backgrounds.device)], dim=-1)
        else:
            proj_features = depth_channel
            if backgrounds is not None:
                backgrounds = torch.zeros((*batch_dims, C, 1), device=backgrounds.device)
    assert proj_features is not None

    if isect is not None:
        tiles_per_gauss, isect_ids, flatten_ids, isect_offsets = isect
    elif peer_nnz is not None:
        tiles_per_gauss, isect_ids, flatten_ids, isect_offsets = isect_tiles_with_offsets(
            means2d, radii, depths, tile_size, tile_width, tile_height, packed=True, n_images=I,
            image_ids=image_ids, gaussian_ids=gaussian_ids, conics=conics, opacities=opacities,
            nnz_device=peer_nnz)
        PeerExchange.get(device).check()
        _trim_local_meta(meta, int(local_nnz[0]))  # the copy is ordered before the size read
    else:
        # isect_tiles(sort=True, segmented) + isect_offset_encode in one pass
        tiles_per_gauss, isect_ids, flatten_ids, isect_offsets = isect_tiles_with_offsets(
            means2d, radii, depths, tile_size, tile_width, tile_height, packed=packed, n_images=I,
            image_ids=image_ids, gaussian_ids=gaussian_ids, conics=conics, opacities=opacities)
    isect_offsets = isect_offsets.reshape(batch_dims + (C, tile_height, tile_width))

    meta.update(
        {
            "tile_width": tile_width,
            "tile_height": tile_height,
            "tiles_per_gauss": tiles_per_gauss,
            "isect_ids": isect_ids,
            "flatten_ids": flatten_ids,
            "isect_offsets": isect_offsets,
            "width": width,
            "height": height,
            "tile_size": tile_size,
            "n_batches": B,
            "n_cameras": C,
        }
    )

    if proj_features.shape[-1] > channel_chunk:
        n_chunks = (proj_features.shape[-1] + channel_chunk - 1) // channel_chunk
        render_colors, render_alphas = [], []
        for i in range(n_chunks):
            chunk = proj_features[..., i * channel_chunk:(i + 1) * channel_chunk]
            bg_chunk = (backgrounds[..., i * channel_chunk:(i + 1) * channel_chunk]
                        if backgrounds is not None else None)
            rc, ra = rasterize_to_pixels(means2d, conics, chunk, opacities, width, height, tile_size,
                                         isect_offsets, flatten_ids, backgrounds=bg_chunk,
                                         packed=packed, absgrad=absgrad)
            render_colors.append(rc)
            render_alphas.append(ra)
        render_colors = torch.cat(render_colors, dim=-1)
        render_alphas = render_alphas[0]
    else:
        render_colors, render_alphas = rasterize_to_pixels(
            means2d, conics, proj_features, opacities, width, height, tile_size, isect_offsets,
            flatten_ids, backgrounds=backgrounds, packed=packed, absgrad=absgrad)

    if extra_signals is not None:
        E = extra_signals.shape[-1]
        meta["render_extra_signals"] = render_colors[..., D:D + E]
        if render_mode_has_depth_channel(render_mode):
            render_depth = render_colors[..., -1:]
            if render_mode_has_expected_depth(render_mode):
                render_depth = render_depth / render_alphas.clamp(min=1e-10)
            render_colors = torch.cat([render_colors[..., 0:D], render_depth], dim=-1)
        else:
            render_colors = render_colors[..., 0:D]
    elif render_mode_has_expected_depth(render_mode):
        render_colors = torch.cat(
            [render_colors[..., :-1], render_colors[..., -1:] / render_alphas.clamp(min=1e-10)],
            dim=-1)
    return render_colors, render_alphas, meta
