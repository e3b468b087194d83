"""The CUDA path against golden vectors of the reference's own pure-PyTorch
implementation (tests/golden/make_golden.py), on the same inputs:

- rasterize_to_pixels forward + backward against the reference's
  _rasterize_to_pixels with autograd (raster_garden.npz; the case of the
  reference's test_rasterize_to_pixels);
- rasterization() forward + backward to the Gaussian parameters against the
  reference's _rasterization (rasterization_garden.npz; the case of the
  reference's test_rasterization.py).

The CPU oracle is pinned to the same fixtures (tests/test_oracle_raster_golden.py,
tests/test_oracle_rasterization_golden.py) and the kernels to the oracle
(test_gpu_ops.py, test_gpu_rasterization.py); this checks the two ends directly.
Tolerances: images within 1e-4 relative / 1e-5 absolute outside 1e-3 of the
elements (a pair whose alpha lands within an ulp of 1/255 may be kept by one
side only); gradients within 2e-3 relative plus 3e-4 of each gradient's largest
magnitude outside 2e-3 of the elements (float32 atomics in any order; the
backward's T_final = 1 - alpha start near the transmittance stop, which the
autograd path does not have).
"""

import os

import numpy as np
import pytest
import torch

from tests._compare import assert_close

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
GOLD = os.path.join(os.path.dirname(__file__), "golden")


def load(name):
    return dict(np.load(os.path.join(GOLD, name)))


def to_dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def grads_close(got, ref, name):
    scale = float(np.abs(ref).max())
    assert_close(got, ref, 2e-3, 3e-4 * scale, max_bad_frac=2e-3, name=name)


@pytest.mark.parametrize("case", ["one", "soft"])
def test_rasterize_to_pixels_vs_reference_torch_golden(case):
    import gsplat_b200

    g = load("raster_garden.npz")
    W, H, ts = int(g["width"]), int(g["height"]), int(g["tile_size"])
    ops = g["soft_opacities"] if case == "soft" else g["opacities"]
    leaves = [to_dev(g["means2d"]), to_dev(g["conics"]), to_dev(g["colors"]), to_dev(ops),
              to_dev(g["backgrounds"])]
    leaves = [x.clone().requires_grad_(True) for x in leaves]
    rc, ra = gsplat_b200.rasterize_to_pixels(leaves[0], leaves[1], leaves[2], leaves[3], W, H, ts,
                                             to_dev(g["isect_offsets"]), to_dev(g["flatten_ids"]),
                                             backgrounds=leaves[4])
    assert_close(rc, g[f"{case}_render_colors"], 1e-4, 1e-5, max_bad_frac=1e-3, name="render_colors")
    assert_close(ra, g[f"{case}_render_alphas"], 1e-4, 1e-5, max_bad_frac=1e-3, name="render_alphas")
    loss = (rc * to_dev(g["v_render_colors"])).sum() + (ra * to_dev(g["v_render_alphas"])).sum()
    grads = torch.autograd.grad(loss, leaves)
    for name, got in zip(("means2d", "conics", "colors", "opacities", "backgrounds"), grads):
        grads_close(got, g[f"{case}_v_{name}"], name)


@pytest.mark.parametrize("tag,mode,rmode", [("classic", "RGB", "classic"), ("aa", "RGB+ED", "antialiased")])
def test_rasterization_vs_reference_torch_golden(tag, mode, rmode):
    import gsplat_b200

    g = load("rasterization_garden.npz")
    W, H = int(g["width"]), int(g["height"])
    names = ("means", "quats", "scales", "opacities", "sh")
    leaves = [to_dev(g[k]).clone().requires_grad_(True) for k in names]
    rc, ra, _ = gsplat_b200.rasterization(*leaves, to_dev(g["viewmats"]), to_dev(g["Ks"]), W, H, sh_degree=3,
                                          render_mode=mode, rasterize_mode=rmode)
    ref_rc, ref_ra = g[f"{tag}_render"], g[f"{tag}_alpha"]
    assert_close(ra, ref_ra, 1e-4, 1e-5, max_bad_frac=1e-3, name="alphas")
    assert_close(rc[..., :3], ref_rc[..., :3], 1e-4, 1e-5, max_bad_frac=1e-3, name="colors")
    if mode == "RGB+ED":
        covered = ref_ra[..., 0] > 0.05
        assert_close(rc[..., 3][torch.from_numpy(covered).to(DEV)], ref_rc[..., 3][covered], 1e-3, 1e-4,
                     max_bad_frac=1e-3, name="expected depth")
    loss = (rc * to_dev(g["G"][..., :rc.shape[-1]])).sum() + (ra * to_dev(g["Ga"])).sum()
    grads = torch.autograd.grad(loss, leaves)
    for name, got in zip(names, grads):
        grads_close(got, g[f"{tag}_v_{name}"], name)
