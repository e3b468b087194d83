"""Generates the golden vectors in tests/golden/ from the reference gsplat itself.

Run in the build container, where the read-only reference checkout is available:

    python tests/golden/make_golden.py /path/to/reference

The reference's pure-PyTorch path (gsplat/cuda/_torch_impl.py, gsplat/cuda/_math.py)
is imported on CPU -- its CUDA extension cannot be built there, so the JIT loader is
told that no CUDA toolkit exists and gsplat falls back to ``_C = None``. Inputs follow
the reference tests: a seeded subset of the reference fixture assets/test_garden.npz
with its three real cameras (tests/test_basic.py:85-110, gsplat/_helper.py:48-100),
the random intersection case of tests/test_basic.py:698-736, the SH case of
tests/test_basic.py:2903-2939, the rasterizer case of tests/test_basic.py:1954-2063 and
the end-to-end case of tests/test_rasterization.py (the reference's pure-PyTorch
``_rasterization`` with autograd). Outputs are stored as small .npz files which the
CPU tests (tests/test_oracle_golden.py, tests/test_oracle_raster_golden.py,
tests/test_oracle_rasterization_golden.py) compare with the oracle and the GPU tests
compare with the kernels; nothing reads the reference at test time.

    python tests/golden/make_golden.py /path/to/reference raster   # one fixture
"""

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def import_reference(ref_root: str):
    import torch.utils.cpp_extension as ext

    ext._find_cuda_home = lambda: None
    sys.path.insert(0, ref_root)
    import gsplat  # noqa: F401
    from gsplat.cuda import _math, _torch_impl

    return _torch_impl, _math


def garden_subset(ref_root: str, n: int, seed: int):
    d = np.load(os.path.join(ref_root, "assets", "test_garden.npz"))
    means = d["means3d"].astype(np.float32)
    sel = np.all((means >= -2) & (means <= 2), axis=-1)
    means = means[sel]
    rng = np.random.default_rng(seed)
    means = means[rng.choice(len(means), n, replace=False)]
    g = torch.Generator().manual_seed(seed)
    scales = torch.rand((n, 3), generator=g) * (0.02 - 1e-4) + 1e-4
    quats = torch.nn.functional.normalize(torch.randn((n, 4), generator=g), dim=-1)
    opacities = torch.rand((n,), generator=g)
    return (torch.from_numpy(means), quats, scales, opacities, torch.from_numpy(d["viewmats"]),
            torch.from_numpy(d["Ks"]), int(d["width"]), int(d["height"]))


def make_projection(ti, tm, ref_root):
    means, quats, scales, opacities, viewmats, Ks, W, H = garden_subset(ref_root, 800, 7)
    out = {}
    for calc in (False, True):
        m = means.clone().requires_grad_(True)
        q = quats.clone().requires_grad_(True)
        s = scales.clone().requires_grad_(True)
        v = viewmats.clone().requires_grad_(True)
        covars, _ = tm._quat_scale_to_covar_preci(q, s, compute_preci=False, triu=False)
        radii, means2d, depths, conics, comps = ti._fully_fused_projection(
            m, covars, v, Ks, W, H, eps2d=0.3, calc_compensations=calc)
        valid = (radii > 0).all(dim=-1)
        g = torch.Generator().manual_seed(11)
        vm2 = torch.randn(means2d.shape, generator=g) * valid[..., None]
        vd = torch.randn(depths.shape, generator=g) * valid
        vc = torch.randn(conics.shape, generator=g) * valid[..., None]
        loss = (means2d * vm2).sum() + (depths * vd).sum() + (conics * vc).sum()
        vcomp = None
        if calc:
            vcomp = torch.randn(comps.shape, generator=g) * valid
            loss = loss + (comps * vcomp).sum()
        gm, gq, gs, gv = torch.autograd.grad(loss, (m, q, s, v))
        tag = "aa" if calc else "classic"
        out.update({
            f"{tag}_radii": radii.numpy(), f"{tag}_means2d": means2d.detach().numpy(),
            f"{tag}_depths": depths.detach().numpy(), f"{tag}_conics": conics.detach().numpy(),
            f"{tag}_v_means2d": vm2.numpy(), f"{tag}_v_depths": vd.numpy(),
            f"{tag}_v_conics": vc.numpy(), f"{tag}_v_means": gm.numpy(),
            f"{tag}_v_quats": gq.numpy(), f"{tag}_v_scales": gs.numpy(),
            f"{tag}_v_viewmats": gv.numpy(),
        })
        if calc:
            out[f"{tag}_comps"] = comps.detach().numpy()
            out[f"{tag}_v_comps"] = vcomp.numpy()
    out.update({"means": means.numpy(), "quats": quats.numpy(), "scales": scales.numpy(),
                "opacities": opacities.numpy(), "viewmats": viewmats.numpy(), "Ks": Ks.numpy(),
                "width": W, "height": H})
    np.savez_compressed(os.path.join(HERE, "projection_garden.npz"), **out)


def make_covar(tm):
    g = torch.Generator().manual_seed(3)
    quats = torch.randn((500, 4), generator=g)
    scales = torch.rand((500, 3), generator=g) * 0.1 + 1e-3
    covars, precis = tm._quat_scale_to_covar_preci(quats, scales, triu=False)
    np.savez_compressed(os.path.join(HERE, "covar.npz"), quats=quats.numpy(), scales=scales.numpy(),
                        covars=covars.numpy(), precis=precis.numpy())


def make_covar_grad(tm):
    """tests/test_basic.py:117-152: gradients of covars and precis (full and triu)."""
    g = torch.Generator().manual_seed(13)
    quats = torch.randn((400, 4), generator=g)
    scales = torch.rand((400, 3), generator=g) * 0.1 + 2e-2
    out = {"quats": quats.numpy(), "scales": scales.numpy()}
    for triu in (False, True):
        q = quats.clone().requires_grad_(True)
        s = scales.clone().requires_grad_(True)
        covars, precis = tm._quat_scale_to_covar_preci(q, s, triu=triu)
        vc = torch.randn(covars.shape, generator=g)
        vp = torch.randn(precis.shape, generator=g) * 0.01
        gq, gs = torch.autograd.grad((covars * vc).sum() + (precis * vp).sum(), (q, s))
        tag = "triu" if triu else "full"
        out.update({f"{tag}_covars": covars.detach().numpy(), f"{tag}_precis": precis.detach().numpy(),
                    f"{tag}_v_covars": vc.numpy(), f"{tag}_v_precis": vp.numpy(),
                    f"{tag}_v_quats": gq.numpy(), f"{tag}_v_scales": gs.numpy()})
    np.savez_compressed(os.path.join(HERE, "covar_grad.npz"), **out)


def make_proj(ti, tm, ref_root):
    """tests/test_basic.py:155-211 (proj of camera-space Gaussians, three camera
    models) and 214-324 (fully fused projection with the fisheye model)."""
    means, quats, scales, opacities, viewmats, Ks, W, H = garden_subset(ref_root, 300, 17)
    covars, _ = tm._quat_scale_to_covar_preci(quats, scales, compute_preci=False, triu=False)
    means_c, covars_c = ti._world_to_cam(means, covars, viewmats)
    out = {"means": means.numpy(), "quats": quats.numpy(), "scales": scales.numpy(),
           "viewmats": viewmats.numpy(), "Ks": Ks.numpy(), "width": W, "height": H,
           "means_c": means_c.numpy(), "covars_c": covars_c.numpy()}
    fns = {"pinhole": ti._persp_proj, "ortho": ti._ortho_proj, "fisheye": ti._fisheye_proj}
    g = torch.Generator().manual_seed(19)
    for name, fn in fns.items():
        m = means_c.clone().requires_grad_(True)
        c = covars_c.clone().requires_grad_(True)
        means2d, covars2d = fn(m, c, Ks, W, H)
        vm = torch.randn(means2d.shape, generator=g)
        vc = torch.randn(covars2d.shape, generator=g)
        gm, gc = torch.autograd.grad((means2d * vm).sum() + (covars2d * vc).sum(), (m, c))
        out.update({f"{name}_means2d": means2d.detach().numpy(), f"{name}_covars2d": covars2d.detach().numpy(),
                    f"{name}_v_means2d": vm.numpy(), f"{name}_v_covars2d": vc.numpy(),
                    f"{name}_v_means": gm.numpy(), f"{name}_v_covars": gc.numpy()})
    # fully fused projection, fisheye
    m = means.clone().requires_grad_(True)
    q = quats.clone().requires_grad_(True)
    s = scales.clone().requires_grad_(True)
    v = viewmats.clone().requires_grad_(True)
    cov, _ = tm._quat_scale_to_covar_preci(q, s, compute_preci=False, triu=False)
    radii, means2d, depths, conics, _ = ti._fully_fused_projection(m, cov, v, Ks, W, H, eps2d=0.3,
                                                                   camera_model="fisheye")
    valid = (radii > 0).all(dim=-1)
    vm2 = torch.randn(means2d.shape, generator=g) * valid[..., None]
    vd = torch.randn(depths.shape, generator=g) * valid
    vcn = torch.randn(conics.shape, generator=g) * valid[..., None]
    loss = (means2d * vm2).sum() + (depths * vd).sum() + (conics * vcn).sum()
    gm, gq, gs, gv = torch.autograd.grad(loss, (m, q, s, v))
    out.update({"fused_radii": radii.numpy(), "fused_means2d": means2d.detach().numpy(),
                "fused_depths": depths.detach().numpy(), "fused_conics": conics.detach().numpy(),
                "fused_v_means2d": vm2.numpy(), "fused_v_depths": vd.numpy(), "fused_v_conics": vcn.numpy(),
                "fused_v_means": gm.numpy(), "fused_v_quats": gq.numpy(), "fused_v_scales": gs.numpy(),
                "fused_v_viewmats": gv.numpy()})
    np.savez_compressed(os.path.join(HERE, "proj_garden.npz"), **out)


def make_projection_variants(ti, tm, ref_root):
    """tests/test_basic.py:214-324 (test_projection) beyond the default camera:
    "ortho": the orthographic model with compensations (quats / scales input);
    "planes": pinhole with near / far planes that cull part of the scene, a batch
    of two scenes and camera sets ([2, N, 3], [2, C, 4, 4]), and the covariance
    input instead of quats / scales (gradients with respect to the full 3x3
    covariances)."""
    means, quats, scales, opacities, viewmats, Ks, W, H = garden_subset(ref_root, 300, 37)
    g = torch.Generator().manual_seed(41)
    out = {"means": means.numpy(), "quats": quats.numpy(), "scales": scales.numpy(),
           "viewmats": viewmats.numpy(), "Ks": Ks.numpy(), "width": W, "height": H}

    def upstream(radii, means2d, depths, conics, comps):
        valid = (radii > 0).all(dim=-1)
        vm2 = torch.randn(means2d.shape, generator=g) * valid[..., None]
        vd = torch.randn(depths.shape, generator=g) * valid
        vcn = torch.randn(conics.shape, generator=g) * valid[..., None]
        vcp = None if comps is None else torch.randn(comps.shape, generator=g) * valid
        loss = (means2d * vm2).sum() + (depths * vd).sum() + (conics * vcn).sum()
        if comps is not None:
            loss = loss + (comps * vcp).sum()
        return loss, vm2, vd, vcn, vcp

    # ortho, compensations
    m = means.clone().requires_grad_(True)
    q = quats.clone().requires_grad_(True)
    s = scales.clone().requires_grad_(True)
    v = viewmats.clone().requires_grad_(True)
    cov, _ = tm._quat_scale_to_covar_preci(q, s, compute_preci=False, triu=False)
    res = ti._fully_fused_projection(m, cov, v, Ks, W, H, eps2d=0.3, calc_compensations=True,
                                     camera_model="ortho")
    loss, vm2, vd, vcn, vcp = upstream(*res)
    gm, gq, gs, gv = torch.autograd.grad(loss, (m, q, s, v))
    radii, means2d, depths, conics, comps = res
    out.update({"ortho_radii": radii.numpy(), "ortho_means2d": means2d.detach().numpy(),
                "ortho_depths": depths.detach().numpy(), "ortho_conics": conics.detach().numpy(),
                "ortho_comps": comps.detach().numpy(), "ortho_v_means2d": vm2.numpy(),
                "ortho_v_depths": vd.numpy(), "ortho_v_conics": vcn.numpy(), "ortho_v_comps": vcp.numpy(),
                "ortho_v_means": gm.numpy(), "ortho_v_quats": gq.numpy(), "ortho_v_scales": gs.numpy(),
                "ortho_v_viewmats": gv.numpy()})

    # near / far planes, batch of two, covariance input
    means_b = torch.stack([means, means + torch.randn(means.shape, generator=g) * 0.05])
    covars_b, _ = tm._quat_scale_to_covar_preci(quats, scales, compute_preci=False, triu=False)
    covars_b = torch.stack([covars_b, covars_b.flip(0)])
    viewmats_b = torch.stack([viewmats, viewmats.clone()])
    viewmats_b[1, :, 0, 3] += 0.1
    Ks_b = torch.stack([Ks, Ks])
    near, far = 0.6, 2.0
    m = means_b.clone().requires_grad_(True)
    c = covars_b.clone().requires_grad_(True)
    v = viewmats_b.clone().requires_grad_(True)
    res = ti._fully_fused_projection(m, c, v, Ks_b, W, H, eps2d=0.3, near_plane=near, far_plane=far)
    loss, vm2, vd, vcn, _ = upstream(*res)
    gm, gc, gv = torch.autograd.grad(loss, (m, c, v))
    radii, means2d, depths, conics, _ = res
    out.update({"planes_near": near, "planes_far": far, "planes_means": means_b.numpy(),
                "planes_covars": covars_b.numpy(), "planes_viewmats": viewmats_b.numpy(), "planes_Ks": Ks_b.numpy(),
                "planes_radii": radii.numpy(), "planes_means2d": means2d.detach().numpy(),
                "planes_depths": depths.detach().numpy(), "planes_conics": conics.detach().numpy(),
                "planes_v_means2d": vm2.numpy(), "planes_v_depths": vd.numpy(), "planes_v_conics": vcn.numpy(),
                "planes_v_means": gm.numpy(), "planes_v_covars": gc.numpy(), "planes_v_viewmats": gv.numpy()})
    np.savez_compressed(os.path.join(HERE, "projection_variants.npz"), **out)


def make_sh(ti):
    out = {}
    g = torch.Generator().manual_seed(42)
    N = 300
    coeffs = torch.randn((N, 25, 3), generator=g)
    dirs = torch.randn((N, 3), generator=g)
    out["coeffs"] = coeffs.numpy()
    out["dirs"] = dirs.numpy()
    for deg in range(5):
        c = coeffs.clone().requires_grad_(True)
        d = dirs.clone().requires_grad_(True)
        colors = ti._spherical_harmonics(deg, d, c)
        vcol = torch.randn(colors.shape, generator=g)
        gc, gd = torch.autograd.grad((colors * vcol).sum(), (c, d), allow_unused=True)
        out[f"deg{deg}_colors"] = colors.detach().numpy()
        out[f"deg{deg}_v_colors"] = vcol.numpy()
        out[f"deg{deg}_v_coeffs"] = gc.numpy()
        out[f"deg{deg}_v_dirs"] = (gd if gd is not None else torch.zeros_like(dirs)).numpy()
    np.savez_compressed(os.path.join(HERE, "sh.npz"), **out)


def make_isect(ti):
    """tests/test_basic.py:698-736: C=3, N=1000, 40x60 image, AABB tiles."""
    import math

    g = torch.Generator().manual_seed(42)
    C, N = 3, 1000
    width, height = 40, 60
    means2d = torch.randn((C, N, 2), generator=g) * width
    radii = torch.randint(0, width, (C, N, 2), generator=g, dtype=torch.int32)
    depths = torch.rand((C, N), generator=g)
    tile_size = 16
    tw = math.ceil(width / tile_size)
    th = math.ceil(height / tile_size)
    tpg, isect_ids, flatten_ids = ti._isect_tiles(means2d, radii, depths, tile_size, tw, th)
    # torch.sort is not guaranteed stable; re-sort stably to pin the order of
    # equal keys like cub's stable radix sort.
    _, unsorted_keys, unsorted_ids = ti._isect_tiles(means2d, radii, depths, tile_size, tw, th, sort=False)
    order = np.argsort(unsorted_keys.numpy(), kind="stable")
    offsets = ti._isect_offset_encode(isect_ids, C, tw, th)
    np.savez_compressed(
        os.path.join(HERE, "isect_aabb.npz"), means2d=means2d.numpy(), radii=radii.numpy(),
        depths=depths.numpy(), tile_size=tile_size, tile_width=tw, tile_height=th,
        tiles_per_gauss=tpg.numpy(), isect_ids=unsorted_keys.numpy()[order],
        flatten_ids=unsorted_ids.numpy()[order], torch_sorted_keys=isect_ids.numpy(),
        isect_offsets=offsets.numpy())


def nerfacc_standin():
    """A module object with the two nerfacc functions that the reference's
    PyTorch compositing imports (gsplat/cuda/_torch_impl.py:522-568). nerfacc is
    a third-party dependency of the reference (setup.py: ``nerfacc>=0.5.3``) and is
    not installed here; this restates its published algorithm (nerfacc 0.5.3,
    ``nerfacc/volrend.py``) for samples given ray by ray, in order along each ray:

    - ``render_weight_from_alpha``: transmittance = exclusive product of
      (1 - alpha) along the ray, weight = transmittance * alpha;
    - ``accumulate_along_rays``: per-ray sum of weight * value (of the weights
      when no values are given).

    Both are differentiable, like nerfacc's."""
    import types

    def render_weight_from_alpha(alphas, packed_info=None, ray_indices=None, n_rays=None, prefix_trans=None):
        assert packed_info is None and prefix_trans is None and ray_indices is not None
        if alphas.numel() == 0:
            return alphas.clone(), alphas.clone()
        if ray_indices.numel() > 1:
            assert bool((ray_indices[1:] >= ray_indices[:-1]).all()), "samples must be grouped by ray"
        _, seg, counts = torch.unique_consecutive(ray_indices, return_inverse=True, return_counts=True)
        starts = torch.cumsum(counts, 0) - counts
        pos = torch.arange(ray_indices.numel()) - starts[seg]
        grid = torch.ones((counts.numel(), int(counts.max())), dtype=alphas.dtype)
        grid = grid.index_put((seg, pos), 1.0 - alphas)
        prod = torch.cumprod(grid, dim=1)
        excl = torch.cat([torch.ones_like(prod[:, :1]), prod[:, :-1]], dim=1)
        trans = excl[seg, pos]
        return trans * alphas, trans

    def accumulate_along_rays(weights, values=None, ray_indices=None, n_rays=None):
        src = weights[..., None] if values is None else weights[..., None] * values
        out = torch.zeros((n_rays, src.shape[-1]), dtype=src.dtype)
        return out.index_add(0, ray_indices, src)

    mod = types.ModuleType("nerfacc")
    mod.render_weight_from_alpha = render_weight_from_alpha
    mod.accumulate_along_rays = accumulate_along_rays
    return mod


def make_raster(ti, tm, ref_root):
    """tests/test_basic.py:1954-2063 (test_rasterize_to_pixels) on the CPU: the
    reference's own PyTorch rasterizer ``_rasterize_to_pixels`` (its batching over
    the tile lists, transmittance carry-over between batches, ``accumulate``,
    background) and autograd through it. Two pieces it calls have no CPU path
    in the reference and are supplied here: nerfacc (``nerfacc_standin``) and the
    CUDA op behind ``rasterize_to_indices_in_range``, replaced by the oracle's
    restatement of RasterizeToIndices3DGS.cu (which pixel/splat pairs a batch
    composites, given the transmittances so far). The golden outputs thus pin
    the oracle rasterizer's forward and backward to the reference's own
    compositing code over the oracle's index pairs. Two cameras of the fixture
    scaled to 80x56 pixels (a partial tile row), AABB tiles from the
    reference's own projection / _isect_tiles / _isect_offset_encode, splats
    large and dense enough that pixels reach the transmittance threshold and
    every third alpha hits the 0.99 clamp; ``batch_per_iter`` 100 (one pass) and
    1 (one 256-entry batch of each tile list per pass); and a "soft" case with
    the opacities scaled by 0.3 (no pixel near the transmittance threshold)."""
    import math

    sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
    from oracle import oracle as O
    import gsplat.cuda._wrapper as ref_wrapper

    def indices_from_oracle(range_start, range_end, transmittances, means2d, conics, opacities, image_width,
                            image_height, tile_size, isect_offsets, flatten_ids):
        n = lambda t: t.detach().numpy()
        gids, pids, iids, _ = O.raster_indices(range_start, range_end, n(transmittances), n(means2d), n(conics),
                                               n(opacities), image_width, image_height, tile_size,
                                               isect_offsets.numpy(), flatten_ids.numpy())
        return torch.from_numpy(gids), torch.from_numpy(pids), torch.from_numpy(iids)

    sys.modules["nerfacc"] = nerfacc_standin()
    ref_wrapper.rasterize_to_indices_in_range = indices_from_oracle
    # the backward of the indexed gathers accumulates in parallel on several
    # threads (order-dependent rounding): one thread keeps the fixture reproducible
    threads = torch.get_num_threads()
    torch.set_num_threads(1)

    means, quats, scales, opacities, viewmats, Ks, W0, H0 = garden_subset(ref_root, 300, 29)
    W, H, ts = 80, 56, 16
    C = 2
    viewmats, Ks = viewmats[:C].contiguous(), Ks[:C].clone()
    Ks[:, 0, :] *= W / W0
    Ks[:, 1, :] *= H / H0
    g = torch.Generator().manual_seed(31)
    N = means.shape[0]
    scales = torch.rand((N, 3), generator=g) * 0.2 + 0.05
    opacities = torch.rand((N,), generator=g)
    opacities[::3] = 0.995
    covars, _ = tm._quat_scale_to_covar_preci(quats, scales, compute_preci=False, triu=False)
    radii, means2d, depths, conics, _ = ti._fully_fused_projection(means, covars, viewmats, Ks, W, H)
    tw, th = math.ceil(W / ts), math.ceil(H / ts)
    _, keys, fids = ti._isect_tiles(means2d, radii, depths, ts, tw, th, sort=False)
    order = np.argsort(keys.numpy(), kind="stable")  # stable, like the CUDA radix sort
    keys, fids = keys[torch.from_numpy(order)], fids[torch.from_numpy(order)]
    offsets = ti._isect_offset_encode(keys, C, tw, th)
    opacities = torch.broadcast_to(opacities[None], (C, N)).contiguous()
    colors = torch.rand((C, N, 3), generator=g)
    backgrounds = torch.rand((C, 3), generator=g)
    v_colors_img = torch.randn((C, H, W, 3), generator=g)
    v_alphas_img = torch.randn((C, H, W, 1), generator=g)
    out = {"width": W, "height": H, "tile_size": ts, "means2d": means2d.numpy(), "conics": conics.numpy(),
           "colors": colors.numpy(), "opacities": opacities.numpy(), "backgrounds": backgrounds.numpy(),
           "isect_offsets": offsets.numpy(), "flatten_ids": fids.numpy(),
           "v_render_colors": v_colors_img.numpy(), "v_render_alphas": v_alphas_img.numpy()}
    out["soft_opacities"] = (opacities * 0.3).numpy()
    for tag, per_iter in (("one", 100), ("iter", 1), ("soft", 100)):
        op_case = opacities * 0.3 if tag == "soft" else opacities
        leaves = [t.clone().requires_grad_(True) for t in (means2d, conics, colors, op_case, backgrounds)]
        m2, con, col, op, bg = leaves
        rc, ra = ti._rasterize_to_pixels(m2, con, col, op, W, H, ts, offsets, fids, backgrounds=bg,
                                         batch_per_iter=per_iter)
        grads = torch.autograd.grad((rc * v_colors_img).sum() + (ra * v_alphas_img).sum(), leaves)
        out.update({f"{tag}_render_colors": rc.detach().numpy(), f"{tag}_render_alphas": ra.detach().numpy()})
        for name, gr in zip(("means2d", "conics", "colors", "opacities", "backgrounds"), grads):
            out[f"{tag}_v_{name}"] = gr.numpy()
    torch.set_num_threads(threads)
    np.savez_compressed(os.path.join(HERE, "raster_garden.npz"), **out)


def make_rasterization(ti, tm, ref_root):
    """tests/test_rasterization.py (rasterization() against _rasterization()) on
    the CPU: the reference's own pure-PyTorch ``gsplat.rendering._rasterization``
    (projection by _fully_fused_projection, SH colours by _maybe_evaluate_sh,
    compositing by _rasterize_to_pixels, expected depth) and autograd through it
    to the Gaussian parameters. The CUDA ops it calls are replaced by the
    reference's own PyTorch counterparts where they exist (isect_tiles ->
    _isect_tiles in AABB mode, sorted stably; isect_offset_encode ->
    _isect_offset_encode; spherical_harmonics -> _spherical_harmonics with the
    visibility mask applied) and otherwise as in ``make_raster`` (the oracle's
    index pass, nerfacc restated). One garden camera scaled to 80x56, 400
    Gaussians with SH degree 3; "classic" RGB and "antialiased" RGB+ED."""
    import math

    sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
    from oracle import oracle as O
    import gsplat.cuda._wrapper as ref_wrapper
    import gsplat.rendering as ref_rendering

    def indices_from_oracle(range_start, range_end, transmittances, means2d, conics, opacities, image_width,
                            image_height, tile_size, isect_offsets, flatten_ids):
        n = lambda t: t.detach().numpy()
        gids, pids, iids, _ = O.raster_indices(range_start, range_end, n(transmittances), n(means2d), n(conics),
                                               n(opacities), image_width, image_height, tile_size,
                                               isect_offsets.numpy(), flatten_ids.numpy())
        return torch.from_numpy(gids), torch.from_numpy(pids), torch.from_numpy(iids)

    def isect_tiles_torch(means2d, radii, depths, tile_size, tile_width, tile_height, **unused):
        tpg, keys, fids = ti._isect_tiles(means2d.detach(), radii, depths.detach(), tile_size, tile_width,
                                          tile_height, sort=False)
        order = torch.from_numpy(np.argsort(keys.numpy(), kind="stable"))
        return tpg, keys[order], fids[order]

    def sh_torch(degrees_to_use, dirs, coeffs, masks=None):
        out = ti._spherical_harmonics(degrees_to_use, dirs, coeffs)
        return out if masks is None else torch.where(masks[..., None], out, torch.zeros_like(out))

    sys.modules["nerfacc"] = nerfacc_standin()
    ref_wrapper.rasterize_to_indices_in_range = indices_from_oracle
    ref_rendering.isect_tiles = isect_tiles_torch
    ref_rendering.isect_offset_encode = lambda ids, n, tw, th: ti._isect_offset_encode(ids, n, tw, th)
    ref_rendering.spherical_harmonics = sh_torch
    threads = torch.get_num_threads()
    torch.set_num_threads(1)  # reproducible accumulation order in the backward

    means, quats, scales, opacities, viewmats, Ks, W0, H0 = garden_subset(ref_root, 400, 43)
    W, H = 80, 56
    viewmats, Ks = viewmats[:1].contiguous(), Ks[:1].clone()
    Ks[:, 0, :] *= W / W0
    Ks[:, 1, :] *= H / H0
    N = means.shape[0]
    g = torch.Generator().manual_seed(47)
    scales = torch.rand((N, 3), generator=g) * 0.2 + 0.05
    opacities = torch.rand((N,), generator=g) * 0.9 + 0.05
    sh = torch.randn((N, 16, 3), generator=g) * 0.05
    sh[:, 0, :] = torch.randn((N, 3), generator=g) * 0.2 + 0.5
    G = torch.randn((1, H, W, 4), generator=g)
    Ga = torch.randn((1, H, W, 1), generator=g)
    out = {"width": W, "height": H, "means": means.numpy(), "quats": quats.numpy(), "scales": scales.numpy(),
           "opacities": opacities.numpy(), "sh": sh.numpy(), "viewmats": viewmats.numpy(), "Ks": Ks.numpy(),
           "G": G.numpy(), "Ga": Ga.numpy()}
    for tag, mode, rmode in (("classic", "RGB", "classic"), ("aa", "RGB+ED", "antialiased")):
        leaves = [t.clone().requires_grad_(True) for t in (means, quats, scales, opacities, sh)]
        rc, ra, _ = ref_rendering._rasterization(*leaves[:4], leaves[4], viewmats, Ks, W, H, sh_degree=3,
                                                 render_mode=mode, rasterize_mode=rmode)
        loss = (rc * G[..., :rc.shape[-1]]).sum() + (ra * Ga).sum()
        grads = torch.autograd.grad(loss, leaves)
        out.update({f"{tag}_render": rc.detach().numpy(), f"{tag}_alpha": ra.detach().numpy()})
        for name, gr in zip(("means", "quats", "scales", "opacities", "sh"), grads):
            out[f"{tag}_v_{name}"] = gr.numpy()
    torch.set_num_threads(threads)
    assert math.isfinite(float(out["classic_render"].sum()))
    np.savez_compressed(os.path.join(HERE, "rasterization_garden.npz"), **out)


def indices_torch(range_start, range_end, transmittances, means2d, conics, opacities, image_width,
                  image_height, tile_size, isect_offsets, flatten_ids):
    """The index pass behind ``rasterize_to_indices_in_range`` written directly in
    PyTorch from its CUDA source (RasterizeToIndices3DGS.cu:100-185), independent
    of the oracle: for every pixel of every tile, walk the tile-list entries of
    batches [range_start, range_end) front to back starting from the pixel's
    transmittance; skip a pair when sigma < 0 or alpha = min(0.99, o exp(-sigma))
    < 1/255; stop (exclusively) at the first kept pair that would take the
    transmittance to <= 1e-4; emit the kept pairs before it. Decisions are taken
    in float32 (the CUDA kernel's arithmetic) whatever the dtype of the inputs.
    Returns gaussian_ids, pixel_ids, image_ids (int64), grouped by pixel."""
    f32 = lambda t: t.detach().to(torch.float32)
    image_dims = means2d.shape[:-2]
    I = int(np.prod(image_dims)) if len(image_dims) else 1
    N = means2d.shape[-2]
    th, tw = isect_offsets.shape[-2:]
    m2 = f32(means2d).reshape(I * N, 2)
    con = f32(conics).reshape(I * N, 3)
    op = f32(opacities).reshape(I * N)
    trans = f32(transmittances).reshape(I, image_height * image_width)
    offs = isect_offsets.reshape(-1).tolist() + [flatten_ids.numel()]
    bs = tile_size * tile_size
    out_g, out_p, out_i = [], [], []
    ly, lx = torch.meshgrid(torch.arange(tile_size), torch.arange(tile_size), indexing="ij")
    ly, lx = ly.reshape(-1), lx.reshape(-1)
    for t in range(I * th * tw):
        img, tile = divmod(t, th * tw)
        ty, tx = divmod(tile, tw)
        lo = offs[t] + bs * range_start
        hi = min(offs[t + 1], offs[t] + bs * range_end)
        if hi <= lo:
            continue
        py, px = ty * tile_size + ly, tx * tile_size + lx
        inside = (py < image_height) & (px < image_width)
        py, px = py[inside], px[inside]
        pix = py * image_width + px
        fid = flatten_ids[lo:hi].to(torch.int64)  # flat index into [I * N]
        dx = m2[fid, 0][None, :] - (px.to(torch.float32) + 0.5)[:, None]
        dy = m2[fid, 1][None, :] - (py.to(torch.float32) + 0.5)[:, None]
        c = con[fid]
        sigma = 0.5 * (c[:, 0][None] * dx * dx + c[:, 2][None] * dy * dy) + c[:, 1][None] * dx * dy
        alpha = torch.clamp_max(op[fid][None] * torch.exp(-sigma), 0.99)
        keep = (sigma >= 0) & (alpha >= 1.0 / 255.0)
        factor = torch.where(keep, 1.0 - alpha, torch.ones_like(alpha))
        T = trans[img, pix][:, None] * torch.cumprod(factor, dim=1)  # after each entry
        stop = keep & (T <= 1e-4)
        # pairs before each pixel's first stopping entry
        before = torch.cumsum(stop.to(torch.int32), dim=1) == 0
        emit = keep & before
        rows, cols = torch.nonzero(emit, as_tuple=True)  # row-major: grouped by pixel, in list order
        out_g.append(fid[cols] % N)
        out_p.append(pix[rows])
        out_i.append(torch.full_like(rows, img))
    if not out_g:
        e = torch.zeros(0, dtype=torch.int64)
        return e, e.clone(), e.clone()
    g, p_, i_ = torch.cat(out_g), torch.cat(out_p), torch.cat(out_i)
    order = torch.argsort(i_ * (image_height * image_width) + p_, stable=True)
    return g[order], p_[order], i_[order]


def make_config0(ti, tm, ref_root):
    """BASELINE config 0 end to end: the reference's own pure-PyTorch
    ``gsplat.rendering._rasterization`` on the seeded config-0 scene of
    tests/_data.py (10k Gaussians, one 256x256 pinhole camera, fx=fy=300, SH
    degree 3, RGB), forward and autograd backward to means, quats, scales,
    opacities and SH with N(0,1) upstream gradients. Run twice: in float64 (the
    golden truth) and in float32 (the reference's own float32 error against that
    truth, stored as per-tensor summaries). The CUDA ops it calls are replaced by
    the reference's PyTorch counterparts (_isect_tiles sorted stably,
    _isect_offset_encode, _spherical_harmonics), the index pass by
    ``indices_torch`` and nerfacc by ``nerfacc_standin``; no oracle code runs."""
    import math

    import importlib.util

    spec = importlib.util.spec_from_file_location("gsb_test_data", os.path.join(os.path.dirname(HERE), "_data.py"))
    _data = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(_data)
    import gsplat.cuda._wrapper as ref_wrapper
    import gsplat.rendering as ref_rendering

    def isect_tiles_torch(means2d, radii, depths, tile_size, tile_width, tile_height, **unused):
        tpg, keys, fids = ti._isect_tiles(means2d.detach().float(), radii, depths.detach().float(), tile_size,
                                          tile_width, tile_height, sort=False)
        order = torch.from_numpy(np.argsort(keys.numpy(), kind="stable"))
        return tpg, keys[order], fids[order]

    def sh_torch(degrees_to_use, dirs, coeffs, masks=None):
        out = ti._spherical_harmonics(degrees_to_use, dirs, coeffs)
        return out if masks is None else torch.where(masks[..., None], out, torch.zeros_like(out))

    sys.modules["nerfacc"] = nerfacc_standin()
    ref_wrapper.rasterize_to_indices_in_range = indices_torch
    ref_rendering.isect_tiles = isect_tiles_torch
    ref_rendering.isect_offset_encode = lambda ids, n, tw, th: ti._isect_offset_encode(ids, n, tw, th)
    ref_rendering.spherical_harmonics = sh_torch

    d = _data.config0()
    W, H = d["width"], d["height"]
    g = torch.Generator().manual_seed(1)  # upstream gradients (seed + 1)
    G = torch.randn((1, H, W, 3), generator=g)
    Ga = torch.randn((1, H, W, 1), generator=g)
    names = ("means", "quats", "scales", "opacities", "sh")
    out = {"width": W, "height": H, "G": G.numpy(), "Ga": Ga.numpy()}
    for k in names:
        out[f"input_{k}"] = d[k].numpy()
    res = {}
    for dt in (torch.float64, torch.float32):
        leaves = [d[k].to(dt).clone().requires_grad_(True) for k in names]
        rc, ra, meta = ref_rendering._rasterization(*leaves, d["viewmats"].to(dt), d["Ks"].to(dt), W, H,
                                                    sh_degree=3, render_mode="RGB")
        loss = (rc * G.to(dt)).sum() + (ra * Ga.to(dt)).sum()
        grads = torch.autograd.grad(loss, leaves)
        res[dt] = {"render": rc.detach(), "alpha": ra.detach(),
                   **{f"v_{k}": gr for k, gr in zip(names, grads)}}
    for k, v in res[torch.float64].items():
        out[k] = v.to(torch.float32).numpy()  # the float64 truth, rounded once
        e = (res[torch.float32][k].double() - v).abs()
        bar = e > 1e-5 + 1e-4 * v.abs()
        out[f"ref32_{k}"] = np.array([float(e.max()), float(e.max() / v.abs().max()), float(bar.double().mean())])
    assert math.isfinite(float(out["render"].sum()))
    np.savez_compressed(os.path.join(HERE, "config0.npz"), **out)


def main():
    ref_root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("GSPLAT_REFERENCE", "")
    if not ref_root or not os.path.isdir(ref_root):
        raise SystemExit("usage: make_golden.py <reference checkout> [fixture ...]")
    ti, tm = import_reference(ref_root)
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    makers = {
        "covar": lambda: make_covar(tm),
        "covar_grad": lambda: make_covar_grad(tm),
        "proj": lambda: make_proj(ti, tm, ref_root),
        "sh": lambda: make_sh(ti),
        "projection": lambda: make_projection(ti, tm, ref_root),
        "projection_variants": lambda: make_projection_variants(ti, tm, ref_root),
        "isect": lambda: make_isect(ti),
        "raster": lambda: make_raster(ti, tm, ref_root),
        "rasterization": lambda: make_rasterization(ti, tm, ref_root),
        "config0": lambda: make_config0(ti, tm, ref_root),
    }
    for name in sys.argv[2:] or list(makers):
        makers[name]()
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
