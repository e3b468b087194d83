"""rasterize_to_indices_in_range against the CPU oracle, and the fused
rasterizer against the PyTorch compositing path built on it (the reference's
tests/test_basic.py test_rasterize_to_pixels, 1954-2064, which compares
rasterize_to_pixels with _rasterize_to_pixels over the same index triples)."""

import math

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests import _data
from tests._compare import as_np, assert_close
from gsplat_b200.cuda._torch_impl import _rasterize_to_pixels as rasterize_to_pixels_torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def splats(C=2, N=3000, W=160, H=120, seed=41, tile_size=16):
    import gsplat_b200
    from gsplat_b200.cuda._wrapper import isect_offset_encode, isect_tiles

    d = _data.to(_data.scene(N, seed=seed, C=C, width=W, height=H, fx=150.0), DEV)
    d["scales"] = d["scales"] * 1.5
    radii, means2d, depths, conics, _ = gsplat_b200.fully_fused_projection(
        d["means"], None, d["quats"], d["scales"], d["viewmats"], d["Ks"], W, H, opacities=d["opacities"])
    opac = d["opacities"].expand(C, N).contiguous()
    tw, th = math.ceil(W / tile_size), math.ceil(H / tile_size)
    _, isect_ids, flatten_ids = isect_tiles(means2d, radii, depths, tile_size, tw, th, conics=conics,
                                            opacities=opac)
    offsets = isect_offset_encode(isect_ids, C, tw, th)
    return means2d, conics, opac, offsets, flatten_ids, W, H, tile_size


@pytest.mark.parametrize("rng_range", [(0, 10**10), (1, 3), (0, 1)])
def test_rasterize_to_indices_vs_oracle(rng_range):
    from gsplat_b200.cuda._wrapper import rasterize_to_indices_in_range

    means2d, conics, opac, offsets, fids, W, H, ts = splats()
    C = means2d.shape[0]
    g = torch.Generator(device=DEV).manual_seed(3)
    trans = 0.3 + 0.7 * torch.rand((C, H, W), device=DEV, generator=g)
    gids, pids, iids = rasterize_to_indices_in_range(rng_range[0], rng_range[1], trans, means2d, conics, opac,
                                                     W, H, ts, offsets, fids)
    eg, ep, ei, ecnt = O.raster_indices(min(rng_range[0], 2**31 - 1), min(rng_range[1], 2**31 - 1), as_np(trans),
                                        as_np(means2d), as_np(conics), as_np(opac), W, H, ts, as_np(offsets),
                                        as_np(fids))
    assert gids.dtype == torch.int64 and pids.dtype == torch.int64 and iids.dtype == torch.int64
    assert ecnt.sum() > 1000
    # per-pixel pair counts; __expf on the GPU against libm expf here can move a
    # splat across the 1/255 alpha or the transmittance threshold in rare pixels
    flat = (iids * H * W + pids).cpu().numpy()
    cnt = np.bincount(flat, minlength=C * H * W)
    same = cnt == ecnt
    assert same.mean() > 0.999, same.mean()
    # on pixels with equal counts the pairs are identical, in the same order
    sel = same[flat]
    esel = same[ei * H * W + ep]
    np.testing.assert_array_equal(as_np(gids)[sel], eg[esel])
    np.testing.assert_array_equal(flat[sel], (ei * H * W + ep)[esel])
    # grouped by pixel in (image, row, column) order
    assert (np.diff(flat) >= 0).all()


def test_rasterize_to_indices_empty():
    from gsplat_b200.cuda._wrapper import rasterize_to_indices_in_range

    means2d, conics, opac, offsets, fids, W, H, ts = splats(N=200)
    trans = torch.ones((2, H, W), device=DEV)
    out = rasterize_to_indices_in_range(5, 5, trans, means2d, conics, opac, W, H, ts, offsets, fids)
    assert all(t.numel() == 0 for t in out)
    out = rasterize_to_indices_in_range(0, 10, trans, means2d, conics, opac, W, H, ts, offsets, fids[:0])
    assert all(t.numel() == 0 for t in out)
    # fully opaque pixels (transmittance 0) contribute nothing
    out = rasterize_to_indices_in_range(0, 10, torch.zeros_like(trans), means2d, conics, opac, W, H, ts, offsets,
                                        fids)
    assert out[0].numel() == 0


@pytest.mark.parametrize("channels", [3, 32])
def test_rasterize_to_pixels_vs_torch_composition(channels):
    from gsplat_b200.cuda._wrapper import rasterize_to_pixels

    means2d, conics, opac, offsets, fids, W, H, ts = splats(seed=43)
    C, N = means2d.shape[:2]
    g = torch.Generator(device=DEV).manual_seed(11)
    means2d = means2d.detach().clone().requires_grad_(True)
    conics = conics.detach().clone().requires_grad_(True)
    colors = torch.rand((C, N, channels), device=DEV, generator=g).requires_grad_(True)
    opac = opac.detach().clone().requires_grad_(True)
    bg = torch.rand((C, channels), device=DEV, generator=g).requires_grad_(True)
    rc, ra = rasterize_to_pixels(means2d, conics, colors, opac, W, H, ts, offsets, fids, backgrounds=bg)
    trc, tra = rasterize_to_pixels_torch(means2d, conics, colors, opac, W, H, ts, offsets, fids, backgrounds=bg)
    # __expf in the kernel against torch.exp: default float32 tolerances of
    # torch.testing.assert_close (the reference test's), up to threshold flips
    assert_close(rc, trc, 1.3e-6, 1e-5, max_bad_frac=1e-3, name="render")
    assert_close(ra, tra, 1.3e-6, 1e-5, max_bad_frac=1e-3, name="alpha")
    v_rc = torch.randn(rc.shape, device=DEV, generator=g)
    v_ra = torch.randn(ra.shape, device=DEV, generator=g)
    leaves = (means2d, conics, colors, opac, bg)
    grads = torch.autograd.grad((rc * v_rc).sum() + (ra * v_ra).sum(), leaves)
    tgrads = torch.autograd.grad((trc * v_rc).sum() + (tra * v_ra).sum(), leaves)
    # the reference test's tolerances
    tol = {"v_means2d": (5e-3, 5e-3), "v_conics": (1e-3, 1e-3), "v_colors": (1e-3, 1e-3),
           "v_opacities": (8e-3, 6e-3), "v_backgrounds": (1e-3, 1e-3)}
    for (name, (rt, at)), a, b in zip(tol.items(), grads, tgrads):
        assert_close(a, as_np(b), rt, at, max_bad_frac=1e-3, name=name)
