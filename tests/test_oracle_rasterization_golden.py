"""Pins the CPU oracle's whole training-step pipeline (projection -> SH ->
AccuTile -> sort -> offsets -> rasterize, and the backward chain to means,
quats, scales, opacities and SH coefficients; tests/_pipeline.py) to the
reference's own pure-PyTorch ``gsplat.rendering._rasterization`` with autograd
(tests/golden/make_golden.py ``make_rasterization``: its CUDA calls replaced by
the reference's PyTorch counterparts, the index pass by the oracle's, nerfacc
restated). Mirrors the reference's tests/test_rasterization.py. CPU only.

The reference path intersects tiles by 3-sigma boxes, the oracle by the
opacity-aware ellipse (AccuTile); both leave the same contributing pixel /
splat pairs, so images and gradients agree.

Tolerances: images, alphas and expected depth within 1e-4 relative / 1e-5
absolute. Gradients: every element within 2e-3 relative plus 1e-4 of the
gradient's largest magnitude, and the largest error within 2e-4 of it. That is
the float32 backward's T_final = 1 - alpha start (RasterizeToPixels3DGSBwd.cu:130)
in pixels near the 1e-4 stop threshold, as tests/test_oracle_raster_golden.py
measures.
"""

import os

import numpy as np
import pytest
import torch

from tests._compare import assert_close
from tests._pipeline import oracle_pipeline

GOLD = os.path.join(os.path.dirname(__file__), "golden", "rasterization_garden.npz")


@pytest.mark.parametrize("tag,calc,depth", [("classic", False, False), ("aa", True, True)])
def test_oracle_pipeline_matches_reference_rasterization(tag, calc, depth):
    g = dict(np.load(GOLD))
    W, H = int(g["width"]), int(g["height"])
    d = {k: torch.from_numpy(g[k]) for k in ("means", "quats", "scales", "opacities", "sh", "viewmats", "Ks")}
    G = g["G"][..., :4 if depth else 3]
    Ga = g["Ga"]

    def v_fn(raw_rc, raw_ra):
        # upstream gradients with respect to the rasterizer's raw outputs; the
        # "ED" channel is accumulated depth / max(alpha, 1e-10)
        if not depth:
            return G, Ga
        a = np.maximum(raw_ra, 1e-10)
        vrc = G.copy()
        vrc[..., 3:4] = G[..., 3:4] / a
        vra = Ga + np.where(raw_ra > 1e-10, -G[..., 3:4] * raw_rc[..., 3:4] / a ** 2, 0.0)
        return vrc, vra.astype(np.float32)

    e = oracle_pipeline(d, W, H, 16, calc, depth, v_fn, 0)
    render = e["render"].copy()
    if depth:
        render[..., 3:4] = render[..., 3:4] / np.maximum(e["alpha"], 1e-10)
    assert g[f"{tag}_alpha"].max() > 0.9998  # pixels reach the transmittance stop
    assert_close(e["alpha"], g[f"{tag}_alpha"], 1e-4, 1e-5, name="alphas")
    assert_close(render[..., :3], g[f"{tag}_render"][..., :3], 1e-4, 1e-5, name="colors")
    if depth:
        covered = e["alpha"][..., 0] > 0.05
        assert_close(render[..., 3][covered], g[f"{tag}_render"][..., 3][covered], 1e-4, 1e-5,
                     name="expected depth")
    for k in ("means", "quats", "scales", "opacities", "sh"):
        ref = g[f"{tag}_v_{k}"]
        scale = float(np.abs(ref).max())
        assert_close(e[f"v_{k}"], ref, 2e-3, 1e-4 * scale, name=k)
        assert np.abs(e[f"v_{k}"].astype(np.float64) - ref).max() <= 2e-4 * scale, k
