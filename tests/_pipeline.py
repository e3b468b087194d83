"""The reference training step's forward and backward on the CPU through the
oracle (test infrastructure): projection -> SH -> AccuTile -> sort -> offsets ->
rasterize, then the chain of backward passes to the Gaussian parameters. Shared
by the GPU end-to-end parity test and the CPU pin against the reference's own
PyTorch ``_rasterization``."""

import math

import numpy as np

from oracle import oracle as O


def oracle_pipeline(d, W, H, tile_size, calc, depth_channel, v_fn, camera_model=0):
    """The reference algorithm on the CPU: projection -> SH -> AccuTile -> sort ->
    offsets -> rasterize, then the chain of backward passes to the parameters."""
    n = lambda t: t.detach().cpu().numpy()
    means, quats, scales, opac, sh = n(d["means"]), n(d["quats"]), n(d["scales"]), n(d["opacities"]), n(d["sh"])
    vm, K = n(d["viewmats"]), n(d["Ks"])
    C = vm.shape[0]
    N = means.shape[0]
    radii, m2, dep, con, comp = O.projection_fwd(means, None, quats, scales, opac, vm, K, W, H,
                                                 calc_compensations=calc, camera_model=camera_model)
    valid = (radii > 0).all(-1)
    campos = -np.einsum("cji,cj->ci", vm[:, :3, :3], vm[:, :3, 3])
    dirs = means[None] - campos[:, None]
    coeffs = np.broadcast_to(sh[None], (C,) + sh.shape)
    raw = O.sh_fwd(3, dirs, coeffs, valid)
    colors = np.maximum(raw + 0.5, 0.0)
    op_eff = np.ascontiguousarray(np.broadcast_to(opac[None], (C, N)) * (comp if calc else 1.0))
    feats = np.concatenate([colors, dep[..., None]], -1) if depth_channel else colors
    tw, th = math.ceil(W / tile_size), math.ceil(H / tile_size)
    _, keys, fids = O.isect_tiles(m2, radii, dep, tile_size, tw, th, conics=con, opacities=op_eff)
    offsets = O.isect_offset_encode(keys, C, tw, th)
    rc, ra, last = O.raster_fwd(m2, con, feats, op_eff, W, H, tile_size, offsets, fids)
    vrc, vra = v_fn(rc, ra)
    v_m2, v_con, v_feat, v_op, _ = O.raster_bwd(m2, con, feats, op_eff, W, H, tile_size, offsets,
                                                fids, ra, last, vrc, vra)
    v_col = v_feat[..., :3] * (raw + 0.5 >= 0)
    v_dep = v_feat[..., 3] if depth_channel else np.zeros_like(dep)
    v_coeffs, v_dirs = O.sh_bwd(3, dirs, coeffs, v_col, valid)
    v_opac = (v_op * (comp if calc else 1.0)).sum(0)
    v_comp = v_op * opac[None] if calc else None
    v_means, _, v_quats, v_scales, _ = O.projection_bwd(
        means, None, quats, scales, vm, K, W, H, 0.3, radii, con, comp if calc else None,
        v_m2 * valid[..., None], v_dep * valid, v_con * valid[..., None],
        v_comp * valid if calc else None, camera_model=camera_model)
    v_means = v_means + (v_dirs * valid[..., None]).sum(0)
    return dict(render=rc, alpha=ra, v_means=v_means, v_quats=v_quats, v_scales=v_scales,
                v_opacities=v_opac, v_sh=(v_coeffs * valid[..., None, None]).sum(0))
