"""accumulate() (the PyTorch compositing utility of gsplat_b200.cuda._torch_impl)
over the oracle's rasterize_to_indices pairs reproduces the oracle rasterizer:
a CPU check of the nerfacc-free transmittance scan (reference
gsplat/cuda/_torch_impl.py:472-570)."""

import math

import numpy as np
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
