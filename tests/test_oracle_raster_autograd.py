"""Cross-check of the CPU oracle's rasterizer in float64 (the reference's own
PyTorch rasterizer pins it in float32, tests/test_oracle_raster_golden.py): an
independent float64 PyTorch restatement of the
compositing rules of RasterizeToPixels3DGSFwd.cu (front to back per tile, alpha
= min(0.99, o exp(-sigma)), skip sigma < 0 or alpha < 1/255, stop before the
splat that takes the transmittance to 1e-4, background by the final
transmittance) must give the oracle's images, and autograd through it must give
the oracle's hand-derived backward (RasterizeToPixels3DGSBwd.cu) for means2d,
conics, colors and opacities. CPU only; small images."""

import math

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests import _data


def torch_raster(m2, con, col, op, bg, W, H, ts, offsets, fids):
    """[I, N, *] float64 tensors -> (render [I, H, W, C], alpha [I, H, W, 1])."""
    I, _, ch = col.shape
    th, tw = offsets.shape[-2:]
    n = len(fids)
    flat = offsets.reshape(-1).tolist() + [n]
    renders, alphas = [], []
    for i in range(I):
        img = torch.zeros((H, W, ch), dtype=torch.float64)
        alp = torch.zeros((H, W, 1), dtype=torch.float64)
        rows_r, rows_a = [], []
        for ty in range(th):
            cols_r, cols_a = [], []
            for tx in range(tw):
                ys = torch.arange(ty * ts, min(H, ty * ts + ts), dtype=torch.float64) + 0.5
                xs = torch.arange(tx * ts, min(W, tx * ts + ts), dtype=torch.float64) + 0.5
                py, px = torch.meshgrid(ys, xs, indexing="ij")
                T = torch.ones_like(px)
                C = torch.zeros(px.shape + (ch,), dtype=torch.float64)
                done = torch.zeros_like(px, dtype=torch.bool)
                t = (i * th + ty) * tw + tx
                for k in range(flat[t], flat[t + 1]):
                    g = int(fids[k]) % m2.shape[1]
                    dx = m2[i, g, 0] - px
                    dy = m2[i, g, 1] - py
                    sigma = 0.5 * (con[i, g, 0] * dx * dx + con[i, g, 2] * dy * dy) + con[i, g, 1] * dx * dy
                    a = torch.clamp(op[i, g] * torch.exp(-sigma), max=0.99)
                    valid = (sigma >= 0) & (a >= 1.0 / 255.0) & ~done
                    nxt = T * (1 - a)
                    stop = valid & (nxt <= 1e-4)
                    done = done | stop
                    use = valid & ~stop
                    C = C + torch.where(use, a * T, torch.zeros_like(a))[..., None] * col[i, g]
                    T = torch.where(use, nxt, T)
                cols_r.append(C + T[..., None] * bg[i])
                cols_a.append((1 - T)[..., None])
            rows_r.append(torch.cat(cols_r, dim=1))
            rows_a.append(torch.cat(cols_a, dim=1))
        renders.append(torch.cat(rows_r, dim=0))
        alphas.append(torch.cat(rows_a, dim=0))
    return torch.stack(renders), torch.stack(alphas)


@pytest.mark.parametrize("case", ["sparse", "saturated"])
def test_oracle_rasterizer_matches_autograd_restatement(case):
    """sparse: few overlaps; saturated: large, nearly opaque splats, so alphas
    hit the 0.99 clamp and pixels reach the transmittance threshold."""
    W, H, ts, C, N = 48, 40, 16, 2, 120
    d = _data.scene(N, seed=23, C=C, width=W, height=H, fx=45.0)
    d["scales"] = d["scales"] * (3.0 if case == "sparse" else 8.0)
    if case == "saturated":
        d["opacities"][::3] = 0.998
        d["opacities"][1::3] = 0.9
    n = lambda t: t.numpy()
    radii, m2, dep, con, _ = O.projection_fwd(n(d["means"]), None, n(d["quats"]), n(d["scales"]),
                                              n(d["opacities"]), n(d["viewmats"]), n(d["Ks"]), W, H)
    op = np.ascontiguousarray(np.broadcast_to(n(d["opacities"])[None], (C, N))).astype(np.float32)
    rng = np.random.default_rng(5)
    col = rng.random((C, N, 3)).astype(np.float32)
    bg = rng.random((C, 3)).astype(np.float32)
    tw, th = math.ceil(W / ts), math.ceil(H / ts)
    _, keys, fids = O.isect_tiles(m2, radii, dep, ts, tw, th, conics=con, opacities=op)
    offsets = O.isect_offset_encode(keys, C, tw, th)
    assert len(fids) > 300
    rc, ra, last = O.raster_fwd(m2, con, col, op, W, H, ts, offsets, fids, backgrounds=bg)
    G = rng.standard_normal(rc.shape).astype(np.float32)
    Ga = rng.standard_normal(ra.shape).astype(np.float32)
    v_m2, v_con, v_col, v_op, _ = O.raster_bwd(m2, con, col, op, W, H, ts, offsets, fids, ra, last, G, Ga,
                                               backgrounds=bg)

    t = lambda a: torch.from_numpy(a.astype(np.float64)).requires_grad_(True)
    tm2, tcon, tcol, top = t(m2), t(con), t(col), t(op)
    trc, tra = torch_raster(tm2, tcon, tcol, top, torch.from_numpy(bg.astype(np.float64)), W, H, ts, offsets,
                            fids)
    if case == "saturated":  # the rules under test are exercised
        assert (ra > 1 - 1.5e-4).mean() > 0.01
    np.testing.assert_allclose(trc.detach().numpy(), rc, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(tra.detach().numpy(), ra, rtol=1e-5, atol=1e-5)
    loss = (trc * torch.from_numpy(G.astype(np.float64))).sum() + (tra * torch.from_numpy(Ga.astype(np.float64))).sum()
    gm2, gcon, gcol, gop = torch.autograd.grad(loss, (tm2, tcon, tcol, top))
    for name, a, e in (("v_means2d", v_m2, gm2), ("v_conics", v_con, gcon), ("v_colors", v_col, gcol),
                       ("v_opacities", v_op, gop)):
        e = e.numpy()
        scale = np.abs(e).max() + 1e-12
        np.testing.assert_allclose(a, e, rtol=1e-3, atol=1e-4 * scale, err_msg=name)
