"""gsplat_b200.strategy.update_state against the reference's
DefaultStrategy._update_state (gsplat/strategy/default.py:218-276), restated
below with the same tensor ops, on the meta of a real rasterization() step."""

from types import SimpleNamespace

import pytest
import torch

from tests import _data
from tests._compare import assert_close

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def reference_update_state(strategy, params, state, info, packed):
    grads = (info["means2d"].absgrad if strategy.absgrad else info["means2d"].grad).clone()
    grads[..., 0] *= info["width"] / 2.0 * info["n_cameras"]
    grads[..., 1] *= info["height"] / 2.0 * info["n_cameras"]
    n = len(list(params.values())[0])
    if state["grad2d"] is None:
        state["grad2d"] = torch.zeros(n, device=grads.device)
    if state["count"] is None:
        state["count"] = torch.zeros(n, device=grads.device)
    if strategy.refine_scale2d_stop_iter > 0 and state["radii"] is None:
        state["radii"] = torch.zeros(n, device=grads.device)
    if packed:
        gs_ids = info["gaussian_ids"]
        radii = info["radii"].max(dim=-1).values
    else:
        sel = (info["radii"] > 0.0).all(dim=-1)
        gs_ids = torch.where(sel)[1]
        grads = grads[sel]
        radii = info["radii"][sel].max(dim=-1).values
    state["grad2d"].index_add_(0, gs_ids, grads.norm(dim=-1))
    state["count"].index_add_(0, gs_ids, torch.ones_like(gs_ids, dtype=torch.float32))
    if strategy.refine_scale2d_stop_iter > 0:
        # the intended scatter maximum (the reference's indexed assignment keeps
        # one value when a Gaussian is visible in several cameras)
        r = radii / float(max(info["width"], info["height"]))
        state["radii"].scatter_reduce_(0, gs_ids, r, reduce="amax")


@pytest.mark.parametrize("packed", [True, False])
@pytest.mark.parametrize("absgrad", [False, True])
@pytest.mark.parametrize("C", [1, 3])
def test_update_state_matches_reference(packed, absgrad, C):
    import gsplat_b200
    from gsplat_b200.strategy import update_state

    d = _data.scene(20000, seed=7, C=C, width=200, height=160, fx=180.0)
    p = {k: d[k].clone().to(DEV).requires_grad_(True) for k in ("means", "quats", "scales", "opacities", "sh")}
    rc, ra, meta = gsplat_b200.rasterization(p["means"], p["quats"], p["scales"], p["opacities"], p["sh"],
                                             d["viewmats"].to(DEV), d["Ks"].to(DEV), 200, 160, sh_degree=3,
                                             packed=packed, absgrad=absgrad)
    meta["means2d"].retain_grad()
    g = torch.Generator(device=DEV).manual_seed(1)
    (rc * torch.randn(rc.shape, device=DEV, generator=g)).sum().backward()
    strat = SimpleNamespace(absgrad=absgrad, key_for_gradient="means2d", refine_scale2d_stop_iter=100)
    mine = {"grad2d": None, "count": None, "radii": None}
    ref = {"grad2d": None, "count": None, "radii": None}
    for _ in range(2):  # the state accumulates over steps
        update_state(strat, p, mine, meta, packed=packed)
        reference_update_state(strat, p, ref, meta, packed)
    assert float(ref["count"].sum()) > 1000
    assert torch.equal(mine["count"], ref["count"])
    assert_close(mine["grad2d"], ref["grad2d"].cpu().numpy(), 1e-5, 1e-7, name="grad2d")
    assert torch.equal(mine["radii"], ref["radii"])
