"""accumulate() (the PyTorch compositing utility of gsplat_b200.cuda._torch_impl)
over the oracle's rasterize_to_indices pairs reproduces the oracle rasterizer:
a CPU check of the nerfacc-free transmittance scan (reference
gsplat/cuda/_torch_impl.py:472-570); and _rasterize_to_pixels matches the
reference's own PyTorch rasterizer on its golden vectors."""

import math

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests import _data


def test_accumulate_matches_oracle_rasterizer():
    from gsplat_b200.cuda._torch_impl import accumulate

    d = _data.scene(3000, seed=43, C=2, width=160, height=120, fx=150.0)
    d["scales"] = d["scales"] * 1.5
    W, H, ts, C, N = 160, 120, 16, 2, 3000
    n = lambda t: t.numpy()
    radii, m2, dep, con, _ = O.projection_fwd(n(d["means"]), None, n(d["quats"]), n(d["scales"]),
                                              n(d["opacities"]), n(d["viewmats"]), n(d["Ks"]), W, H)
    op = np.ascontiguousarray(np.broadcast_to(n(d["opacities"])[None], (C, N)))
    tw, th = math.ceil(W / ts), math.ceil(H / ts)
    _, keys, fids = O.isect_tiles(m2, radii, dep, ts, tw, th, conics=con, opacities=op)
    offsets = O.isect_offset_encode(keys, C, tw, th)
    colors = np.random.default_rng(1).random((C, N, 3)).astype(np.float32)
    rc, ra, _ = O.raster_fwd(m2, con, colors, op, W, H, ts, offsets, fids)
    gids, pids, iids, cnt = O.raster_indices(0, 10**6, np.ones((C, H, W), np.float32), m2, con, op, W, H, ts,
                                             offsets, fids)
    assert cnt.sum() == gids.size > 10000
    t = torch.from_numpy
    r, a = accumulate(t(m2), t(con), t(op), t(colors), t(gids), t(pids), t(iids), W, H)
    np.testing.assert_allclose(r.numpy(), rc, rtol=1e-5, atol=2e-6)
    np.testing.assert_allclose(a.numpy(), ra, rtol=1e-5, atol=2e-6)


@pytest.mark.parametrize("case,per_iter", [("one", 100), ("iter", 1), ("soft", 100)])
def test_torch_rasterizer_matches_reference_torch_golden(monkeypatch, case, per_iter):
    """This library's PyTorch _rasterize_to_pixels (the reference's slow path,
    nerfacc-free) against the reference's own, with autograd
    (tests/golden/raster_garden.npz): both composite the same index pairs, so
    images and all gradients agree to float32 rounding (1e-5 of each gradient's
    largest magnitude), saturated pixels included. The index pass comes from
    the oracle on both sides (on the CPU, in place of the CUDA op)."""
    import os

    import gsplat_b200.cuda._wrapper as wrapper
    from gsplat_b200.cuda._torch_impl import _rasterize_to_pixels

    def indices(rs, re, trans, m2, con, op, W, H, ts, offsets, fids):
        n = lambda t: t.detach().numpy()
        g_, p_, i_, _ = O.raster_indices(rs, re, n(trans), n(m2), n(con), n(op), W, H, ts, n(offsets), n(fids))
        return torch.from_numpy(g_), torch.from_numpy(p_), torch.from_numpy(i_)

    monkeypatch.setattr(wrapper, "rasterize_to_indices_in_range", indices)
    g = dict(np.load(os.path.join(os.path.dirname(__file__), "golden", "raster_garden.npz")))
    W, H, ts = int(g["width"]), int(g["height"]), int(g["tile_size"])
    ops = g["soft_opacities"] if case == "soft" else g["opacities"]
    leaves = [torch.from_numpy(x).clone().requires_grad_(True)
              for x in (g["means2d"], g["conics"], g["colors"], ops, g["backgrounds"])]
    rc, ra = _rasterize_to_pixels(*leaves[:4], W, H, ts, torch.from_numpy(g["isect_offsets"]),
                                  torch.from_numpy(g["flatten_ids"]), backgrounds=leaves[4],
                                  batch_per_iter=per_iter)
    np.testing.assert_allclose(rc.detach().numpy(), g[f"{case}_render_colors"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(ra.detach().numpy(), g[f"{case}_render_alphas"], rtol=1e-5, atol=1e-6)
    loss = (rc * torch.from_numpy(g["v_render_colors"])).sum() + (ra * torch.from_numpy(g["v_render_alphas"])).sum()
    grads = torch.autograd.grad(loss, leaves)
    for name, got in zip(("means2d", "conics", "colors", "opacities", "backgrounds"), grads):
        ref = g[f"{case}_v_{name}"]
        assert np.abs(got.numpy().astype(np.float64) - ref).max() <= 1e-5 * np.abs(ref).max(), name
