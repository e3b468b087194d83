"""The reference's COO gradient path of the packed projection (``sparse_grad``,
gsplat/cuda/_wrapper.py:2258-2310) and its segmented sort (``segmented``,
IntersectTile.cu:525-576), on the GPU.

sparse_grad=True returns the gradients of means / quats / scales as sparse COO
tensors with one row per (camera, Gaussian) pair; summed per Gaussian
(``to_dense``) they must equal the dense gradients bit for bit up to the order of
the per-pair additions. segmented=True must give the same tile ids, splat ids and
offsets as the global sort."""

import math

import numpy as np
import pytest
import torch

from tests import _data
from tests._compare import assert_close, assert_equal

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


@pytest.mark.parametrize("C", [1, 3])
@pytest.mark.parametrize("calc", [False, True])
def test_sparse_grad_matches_dense(C, calc):
    import gsplat_b200

    d = _data.to(_data.scene(5000, seed=21, C=C, width=200, height=160, fx=180.0), DEV)
    out = {}
    for sparse in (False, True):
        leaves = [d[k].clone().requires_grad_(True) for k in ("means", "quats", "scales")]
        (bids, cids, gids, indptr, radii, means2d, depths, conics, comps) = gsplat_b200.fully_fused_projection(
            leaves[0], None, leaves[1], leaves[2], d["viewmats"], d["Ks"], d["width"], d["height"],
            packed=True, sparse_grad=sparse, calc_compensations=calc)
        gen = torch.Generator(device=DEV).manual_seed(5)
        loss = ((means2d * torch.randn(means2d.shape, device=DEV, generator=gen)).sum()
                + (depths * torch.randn(depths.shape, device=DEV, generator=gen)).sum()
                + (conics * torch.randn(conics.shape, device=DEV, generator=gen)).sum())
        if calc:
            loss = loss + (comps * torch.randn(comps.shape, device=DEV, generator=gen)).sum()
        loss.backward()
        out[sparse] = (gids.clone(), [t.grad for t in leaves])
    gids = out[True][0]
    assert_equal(gids, out[False][0], "gaussian_ids")
    assert gids.numel() > 1000
    for name, dense, sp in zip(("means", "quats", "scales"), out[False][1], out[True][1]):
        assert sp.is_sparse, name
        assert sp.shape == dense.shape, name
        assert sp._values().shape == (gids.numel(), dense.shape[-1]), name
        assert_equal(sp._indices()[0], gids, f"{name} indices")
        # one row per pair: the per-Gaussian sum is the dense gradient, up to the
        # order of the float32 additions over cameras (rounding of the terms)
        if C == 1:
            assert_equal(sp.to_dense(), dense, name)
        else:
            scale = float(dense.abs().max())
            assert_close(sp.to_dense(), dense, 1e-5, 1e-6 * scale, name=name)


@pytest.mark.parametrize("packed", [False, True])
def test_segmented_equals_sorted(packed):
    import gsplat_b200

    d = _data.to(_data.scene(8000, seed=23, C=3, width=240, height=180, fx=200.0), DEV)
    res = {}
    for segmented in (False, True):
        out = gsplat_b200.fully_fused_projection(d["means"], None, d["quats"], d["scales"], d["viewmats"],
                                                 d["Ks"], d["width"], d["height"], packed=packed,
                                                 opacities=d["opacities"])
        ts = 16
        tw, th = math.ceil(d["width"] / ts), math.ceil(d["height"] / ts)
        if packed:
            bids, cids, gids, indptr, radii, means2d, depths, conics, _ = out
            res[segmented] = gsplat_b200.isect_tiles(means2d, radii, depths, ts, tw, th, segmented=segmented,
                                                     packed=True, n_images=3, image_ids=cids,
                                                     gaussian_ids=gids)
        else:
            radii, means2d, depths, conics, _ = out
            res[segmented] = gsplat_b200.isect_tiles(means2d, radii, depths, ts, tw, th, segmented=segmented)
    for a, b, name in zip(res[False], res[True], ("tiles_per_gauss", "isect_ids", "flatten_ids")):
        assert_equal(b, a, name)
    # and through rasterization(): same images either way
    imgs = []
    for segmented in (False, True):
        rc, ra, _ = gsplat_b200.rasterization(d["means"], d["quats"], d["scales"], d["opacities"], d["sh"],
                                              d["viewmats"], d["Ks"], d["width"], d["height"], sh_degree=3,
                                              packed=packed, segmented=segmented)
        imgs.append(rc)
    assert_equal(imgs[1], imgs[0], "render")
