"""Parity of the stand-alone covariance and projection ops (quat_scale_to_covar_preci,
proj for the pinhole / ortho / fisheye models) and of the fisheye branch of the
fused projection, with the CPU oracle and the reference golden vectors. Mirrors the
reference tests tests/test_basic.py test_quat_scale_to_covar_preci (117-152),
test_proj (155-211) and test_projection (214-324, camera_model="fisheye")."""

import os

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests import _data
from tests._compare import as_np, assert_close

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
GOLD = os.path.join(os.path.dirname(__file__), "golden")
MODELS = {"pinhole": 0, "ortho": 1, "fisheye": 2}


def gsb():
    import gsplat_b200

    return gsplat_b200


def golden(name):
    return dict(np.load(os.path.join(GOLD, name)))


@pytest.mark.parametrize("triu", [False, True])
@pytest.mark.parametrize("batch", [(), (2,)])
def test_covar_preci_vs_oracle(triu, batch):
    rng = np.random.default_rng(5)
    quats = rng.standard_normal(batch + (3000, 4)).astype(np.float32)
    scales = (rng.random(batch + (3000, 3)) * 0.1 + 2e-2).astype(np.float32)
    q = torch.from_numpy(quats).to(DEV).requires_grad_(True)
    s = torch.from_numpy(scales).to(DEV).requires_grad_(True)
    covars, precis = gsb().quat_scale_to_covar_preci(q, s, triu=triu)
    ec, ep = O.covar_preci_fwd(quats, scales, triu=triu)
    assert_close(covars, ec, 1e-5, 1e-7, name="covars")
    assert_close(precis, ep, 1e-4, 1e-3, name="precis")
    vc = rng.standard_normal(ec.shape).astype(np.float32)
    vp = (rng.standard_normal(ep.shape) * 0.01).astype(np.float32)
    loss = (covars * torch.from_numpy(vc).to(DEV)).sum() + (precis * torch.from_numpy(vp).to(DEV)).sum()
    gq, gs = torch.autograd.grad(loss, (q, s))
    eq, es = O.covar_preci_bwd(quats, scales, triu, vc, vp)
    # fp32 kernel vs float64 oracle
    assert_close(gq, eq, 1e-3, 1e-3, name="v_quats")
    assert_close(gs, es, 1e-3, 1e-2, name="v_scales")


def test_covar_preci_only_one_and_golden():
    g = golden("covar_grad.npz")
    q = torch.from_numpy(g["quats"]).to(DEV)
    s = torch.from_numpy(g["scales"]).to(DEV)
    c, p = gsb().quat_scale_to_covar_preci(q, s, compute_preci=False)
    assert p is None
    assert_close(c, g["full_covars"], 1e-5, 1e-7, name="covars")
    c, p = gsb().quat_scale_to_covar_preci(q, s, compute_covar=False, triu=True)
    assert c is None
    assert_close(p, g["triu_precis"], 2e-3, 1e-2, name="precis")
    for tag, triu in (("full", False), ("triu", True)):
        qq = q.clone().requires_grad_(True)
        ss = s.clone().requires_grad_(True)
        c, p = gsb().quat_scale_to_covar_preci(qq, ss, triu=triu)
        loss = (c * torch.from_numpy(g[f"{tag}_v_covars"]).to(DEV)).sum() + \
            (p * torch.from_numpy(g[f"{tag}_v_precis"]).to(DEV)).sum()
        gq, gs = torch.autograd.grad(loss, (qq, ss))
        # against the fp32 torch graph of the reference (its own test: rtol 1, atol 1e-1)
        assert_close(gq, g[f"{tag}_v_quats"], 1e-2, 1e-2, name="v_quats")
        assert_close(gs, g[f"{tag}_v_scales"], 1e-2, 1e-1, name="v_scales")


@pytest.mark.parametrize("model", ["pinhole", "ortho", "fisheye"])
@pytest.mark.parametrize("batch", [(), (2,)])
def test_proj_vs_oracle(model, batch):
    d = _data.scene(3000, seed=8, C=3, width=320, height=240, fx=200.0)
    import gsplat_b200

    covars, _ = O.covar_preci_fwd(d["quats"].numpy(), d["scales"].numpy(), compute_preci=False)
    with pytest.warns(DeprecationWarning):
        mc, cc = gsplat_b200.world_to_cam(d["means"], torch.from_numpy(covars), d["viewmats"])
    mc = mc.expand(batch + mc.shape).contiguous().numpy()
    cc = cc.expand(batch + cc.shape).contiguous().numpy()
    Ks = d["Ks"].expand(batch + d["Ks"].shape).contiguous().numpy()
    W, H, mid = d["width"], d["height"], MODELS[model]
    m = torch.from_numpy(mc).to(DEV).requires_grad_(True)
    c = torch.from_numpy(cc).to(DEV).requires_grad_(True)
    m2, c2 = gsb().proj(m, c, torch.from_numpy(Ks).to(DEV), W, H, camera_model=model)
    em2, ec2 = O.proj_fwd(mc, cc, Ks, W, H, mid)
    assert_close(m2, em2, 1e-5, 1e-3, name="means2d")
    assert_close(c2, ec2, 1e-4, 1e-3, name="covars2d")
    rng = np.random.default_rng(9)
    vm = rng.standard_normal(em2.shape).astype(np.float32)
    vc = rng.standard_normal(ec2.shape).astype(np.float32)
    loss = (m2 * torch.from_numpy(vm).to(DEV)).sum() + (c2 * torch.from_numpy(vc).to(DEV)).sum()
    gm, gc = torch.autograd.grad(loss, (m, c))
    evm, evc = O.proj_bwd(mc, cc, Ks, W, H, mid, vm, vc)
    scale_m = np.abs(evm).max()
    assert_close(gc, evc, 1e-3, 1e-3, name="v_covars")
    assert_close(gm, evm, 1e-3, 1e-5 * scale_m, name="v_means")


@pytest.mark.parametrize("model", ["pinhole", "ortho", "fisheye"])
def test_proj_golden(model):
    g = golden("proj_garden.npz")
    W, H = int(g["width"]), int(g["height"])
    m = torch.from_numpy(g["means_c"]).to(DEV).requires_grad_(True)
    c = torch.from_numpy(g["covars_c"]).to(DEV).requires_grad_(True)
    m2, c2 = gsb().proj(m, c, torch.from_numpy(g["Ks"]).to(DEV), W, H, camera_model=model)
    assert_close(m2, g[f"{model}_means2d"], 1e-5, 1e-3, name="means2d")
    assert_close(c2, g[f"{model}_covars2d"], 1e-4, 1e-3, name="covars2d")
    loss = (m2 * torch.from_numpy(g[f"{model}_v_means2d"]).to(DEV)).sum() + \
        (c2 * torch.from_numpy(g[f"{model}_v_covars2d"]).to(DEV)).sum()
    gm, gc = torch.autograd.grad(loss, (m, c))
    # the reference test: rtol 6e-1 / atol 1e-2 (means), 1e-1 / 1e-1 (covars)
    assert_close(gc, g[f"{model}_v_covars"], 1e-2, 1e-3, name="v_covars")
    assert_close(gm, g[f"{model}_v_means"], 1e-2, 1e-2, name="v_means")


def test_persp_proj_is_pinhole():
    d = _data.scene(500, seed=2, C=1)
    mc = torch.randn(1, 500, 3, device=DEV) + torch.tensor([0.0, 0.0, 5.0], device=DEV)
    cc = torch.eye(3, device=DEV).expand(1, 500, 3, 3).contiguous() * 0.01
    K = d["Ks"].to(DEV)
    with pytest.warns(DeprecationWarning):
        a = gsb().persp_proj(mc, cc, K, 256, 256)
    b = gsb().proj(mc, cc, K, 256, 256)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


@pytest.mark.parametrize("calc", [False, True])
def test_fisheye_projection_vs_oracle(calc):
    d = _data.to(_data.scene(4000, seed=14, C=2, width=320, height=240, fx=150.0), DEV)
    means = d["means"].clone().requires_grad_(True)
    quats = d["quats"].clone().requires_grad_(True)
    scales = d["scales"].clone().requires_grad_(True)
    viewmats = d["viewmats"].clone().requires_grad_(True)
    radii, means2d, depths, conics, comps = gsb().fully_fused_projection(
        means, None, quats, scales, viewmats, d["Ks"], d["width"], d["height"], calc_compensations=calc,
        opacities=d["opacities"], camera_model="fisheye")
    er, em, ed, ec, ecomp = O.projection_fwd(as_np(d["means"]), None, as_np(d["quats"]), as_np(d["scales"]),
                                             as_np(d["opacities"]), as_np(d["viewmats"]), as_np(d["Ks"]),
                                             d["width"], d["height"], calc_compensations=calc, camera_model=2)
    r = as_np(radii)
    assert np.abs(r.astype(np.int64) - er).max() <= 1
    both = (r > 0).all(-1) & (er > 0).all(-1)
    assert ((r > 0).all(-1) != (er > 0).all(-1)).mean() < 1e-3
    bt = torch.from_numpy(both).to(DEV)
    assert_close(means2d[bt], em[both], 1e-5, 1e-4, name="means2d")
    assert_close(conics[bt], ec[both], 1e-4, 1e-5, name="conics")
    valid = (radii > 0).all(-1)
    gen = torch.Generator(device=DEV).manual_seed(5)
    vm2 = torch.randn(means2d.shape, device=DEV, generator=gen) * valid[..., None]
    vd = torch.randn(depths.shape, device=DEV, generator=gen) * valid
    vc = torch.randn(conics.shape, device=DEV, generator=gen) * valid[..., None]
    loss = (means2d * vm2).sum() + (depths * vd).sum() + (conics * vc).sum()
    vcomp = None
    if calc:
        vcomp = torch.randn(comps.shape, device=DEV, generator=gen) * valid
        loss = loss + (comps * vcomp).sum()
    gm, gq, gs, gv = torch.autograd.grad(loss, (means, quats, scales, viewmats))
    em_, _, eq, es, ev = O.projection_bwd(
        as_np(d["means"]), None, as_np(d["quats"]), as_np(d["scales"]), as_np(d["viewmats"]), as_np(d["Ks"]),
        d["width"], d["height"], 0.3, as_np(radii), as_np(conics), as_np(comps) if calc else None, as_np(vm2),
        as_np(vd), as_np(vc), as_np(vcomp) if calc else None, camera_model=2)
    assert_close(gm, em_, 1e-3, 1e-4, name="v_means")
    assert_close(gq, eq, 1e-3, 1e-4, name="v_quats")
    assert_close(gs, es, 1e-3, 1e-3, name="v_scales")
    assert_close(gv, ev, 1e-3, 1e-2, name="v_viewmats")


def test_fisheye_projection_golden_and_packed():
    g = golden("proj_garden.npz")
    t = lambda k: torch.from_numpy(g[k]).to(DEV)
    W, H = int(g["width"]), int(g["height"])
    means = t("means").requires_grad_(True)
    quats = t("quats").requires_grad_(True)
    scales = t("scales").requires_grad_(True)
    viewmats = t("viewmats").requires_grad_(True)
    radii, means2d, depths, conics, _ = gsb().fully_fused_projection(
        means, None, quats, scales, viewmats, t("Ks"), W, H, camera_model="fisheye")
    er = g["fused_radii"]
    assert np.abs(as_np(radii).astype(np.int64) - er).max() <= 1
    both = torch.from_numpy((as_np(radii) > 0).all(-1) & (er > 0).all(-1)).to(DEV)
    bn = as_np(both)
    assert_close(means2d[both], g["fused_means2d"][bn], 1e-5, 1e-3, name="means2d")
    assert_close(conics[both], g["fused_conics"][bn], 1e-3, 1e-4, name="conics")
    loss = (means2d * t("fused_v_means2d")).sum() + (depths * t("fused_v_depths")).sum() + \
        (conics * t("fused_v_conics")).sum()
    gm, gq, gs, gv = torch.autograd.grad(loss, (means, quats, scales, viewmats))
    assert_close(gm, g["fused_v_means"], 1e-2, 1e-2, name="v_means")
    assert_close(gs, g["fused_v_scales"], 1e-2, 5e-2, name="v_scales")
    assert_close(gq, g["fused_v_quats"], 1e-2, 1e-2, name="v_quats")
    assert_close(gv, g["fused_v_viewmats"], 1e-2, 5e-2, name="v_viewmats")
    # packed layout: the same splats in COO order
    out = gsb().fully_fused_projection(t("means"), None, t("quats"), t("scales"), t("viewmats"), t("Ks"), W, H,
                                       camera_model="fisheye", packed=True)
    bids, cids, gids = out[0], out[1], out[2]
    dense = (radii > 0).all(-1)
    assert int(dense.sum()) == gids.numel()
    assert torch.equal(out[5], means2d[cids, gids]) and torch.equal(out[7], conics[cids, gids])
