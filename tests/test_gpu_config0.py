"""BASELINE config 0 end to end on the GPU: ``gsplat_b200.rasterization()``
forward + backward to means, quats, scales, opacities and SH, against the
reference's own pure-PyTorch ``_rasterization`` run in float64
(tests/golden/config0.npz, made by tests/golden/make_golden.py ``make_config0``).

Bar: images and alphas within 1e-4 relative / 1e-5 absolute (all but 1e-4 of
the pixels: a pair whose alpha lands within rounding of 1/255, or a pixel whose
transmittance lands within rounding of the 1e-4 stop, may be decided the other
way by float32 arithmetic). Gradients: within 1e-4 relative / 1e-5 absolute on
at least as large a fraction of elements as the reference's own float32 run of
the same function achieves against its float64 run, and a largest error (over
the gradient's largest magnitude) no larger than that run's -- i.e. the kernels
are at least as close to the float64 truth as the reference's float32 path.
"""

import os

import numpy as np
import pytest
import torch

from tests import _data
from tests._compare import assert_parity, observed_error

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
GOLD = os.path.join(os.path.dirname(__file__), "golden", "config0.npz")
NAMES = ("means", "quats", "scales", "opacities", "sh")


@pytest.mark.parametrize("packed", [True, False])
def test_config0_rasterization_vs_reference_float64(packed):
    import gsplat_b200

    g = dict(np.load(GOLD))
    d = _data.to(_data.config0(), DEV)
    W, H = int(g["width"]), int(g["height"])
    leaves = [d[k].clone().requires_grad_(True) for k in NAMES]
    rc, ra, _ = gsplat_b200.rasterization(*leaves, d["viewmats"], d["Ks"], W, H, sh_degree=3,
                                          packed=packed)
    loss = (rc * torch.from_numpy(g["G"]).to(DEV)).sum() + (ra * torch.from_numpy(g["Ga"]).to(DEV)).sum()
    grads = torch.autograd.grad(loss, leaves)
    assert_parity(rc, g["render"], "render", max_bad_frac=1e-4)
    assert_parity(ra, g["alpha"], "alpha", max_bad_frac=1e-4)
    for k, gr in zip(NAMES, grads):
        _, ref_scaled, ref_frac = g[f"ref32_v_{k}"]
        obs = observed_error(gr, g[f"v_{k}"])
        assert obs["max_scaled"] <= ref_scaled, (k, obs, g[f"ref32_v_{k}"])
        assert_parity(gr, g[f"v_{k}"], f"v_{k}", max_bad_frac=ref_frac, max_scaled=ref_scaled)
