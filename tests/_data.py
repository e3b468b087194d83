"""Seeded synthetic scenes shared by the tests, the smoke check and the bench.

Distributions follow the benchmark configurations of the reference task:
means N(0,1) in x, y and U[2,8] in z (config 0), scales exp(N(-3.5, 0.5)),
quats N(0,1)^4 normalised, opacities sigmoid(N(0,1)), SH degree 3 with DC
N(0.5, 0.2) and higher bands N(0, 0.05); pinhole cameras. The golden fixtures in
tests/golden/ come from the reference's own test data instead.
"""

import torch


def scene(N, seed=0, width=256, height=256, fx=300.0, cx=None, cy=None, z_range=(2.0, 8.0),
          xy_scale=1.0, C=1, sh_degree=3, viewmats=None, xy_uniform=None):
    g = torch.Generator().manual_seed(seed)
    means = torch.randn((N, 3), generator=g)
    means[:, :2] *= xy_scale
    if xy_uniform is not None:  # x, y ~ U(-xy_uniform, xy_uniform)
        means[:, :2] = (torch.rand((N, 2), generator=g) * 2.0 - 1.0) * xy_uniform
    means[:, 2] = torch.rand((N,), generator=g) * (z_range[1] - z_range[0]) + z_range[0]
    scales = torch.exp(torch.randn((N, 3), generator=g) * 0.5 - 3.5)
    quats = torch.nn.functional.normalize(torch.randn((N, 4), generator=g), dim=-1)
    opacities = torch.sigmoid(torch.randn((N,), generator=g))
    K = (sh_degree + 1) ** 2
    sh = torch.randn((N, K, 3), generator=g) * 0.05
    sh[:, 0, :] = torch.randn((N, 3), generator=g) * 0.2 + 0.5
    cx = width / 2 if cx is None else cx
    cy = height / 2 if cy is None else cy
    Ks = torch.tensor([[fx, 0.0, cx], [0.0, fx, cy], [0.0, 0.0, 1.0]]).expand(C, 3, 3).contiguous()
    if viewmats is None:
        viewmats = torch.eye(4).expand(C, 4, 4).contiguous().clone()
        for c in range(1, C):  # small camera offsets for multi-view cases
            viewmats[c, 0, 3] = 0.3 * c
            viewmats[c, 1, 3] = -0.2 * c
    return dict(means=means, quats=quats, scales=scales, opacities=opacities, sh=sh,
                viewmats=viewmats, Ks=Ks, width=width, height=height)


def config0():
    """10k Gaussians, one 256x256 camera, fx=fy=300."""
    return scene(10_000, seed=0, width=256, height=256, fx=300.0)


def config1(N=1_000_000, seed=1):
    """1M Gaussians in a 10-unit cube in front of one
    1297x840 camera (fx=fy=1150, cx=648.5, cy=420): x, y ~ U(-5, 5), z ~ U(2, 12)."""
    return scene(N, seed=seed, width=1297, height=840, fx=1150.0, cx=648.5, cy=420.0,
                 z_range=(2.0, 12.0), xy_uniform=5.0)


def config2(N=500_000, seed=2, C=4):
    """BASELINE config 2 (the feature variant): N Gaussians with means ~ N(0,1)^3,
    the other distributions as config 0, and C cameras at 1024x1024 (fx=fy=1024,
    cx=cy=512) at angles 2 pi k / C on a radius-6 ring in the x-z plane, looking at
    the origin."""
    import math

    viewmats = torch.stack([look_at((6.0 * math.cos(2 * math.pi * k / C), 0.0, 6.0 * math.sin(2 * math.pi * k / C)),
                                    up=(0.0, 1.0, 0.0)) for k in range(C)])
    d = scene(N, seed=seed, width=1024, height=1024, fx=1024.0, cx=512.0, cy=512.0, C=C, viewmats=viewmats)
    d["means"] = torch.randn((N, 3), generator=torch.Generator().manual_seed(seed))
    return d


def look_at(eye, target=(0.0, 0.0, 0.0), up=(0.0, 0.0, 1.0)):
    """World-to-camera 4x4 (OpenCV axes: z toward the target) for a camera at eye."""
    eye = torch.as_tensor(eye, dtype=torch.float32)
    z = torch.nn.functional.normalize(torch.as_tensor(target, dtype=torch.float32) - eye, dim=0)
    u = torch.as_tensor(up, dtype=torch.float32)
    if torch.cross(z, u, dim=0).norm() < 1e-4:
        u = torch.tensor([0.0, 1.0, 0.0])
    x = torch.nn.functional.normalize(torch.cross(z, u, dim=0), dim=0)
    y = torch.cross(z, x, dim=0)
    R = torch.stack([x, y, z])
    vm = torch.eye(4)
    vm[:3, :3] = R
    vm[:3, 3] = -R @ eye
    return vm


def config3(N=3_000_000, seed=3, C=8):
    """3M Gaussians with means ~ N(0, 2^2)^3, C cameras at
    1920x1080 (fx=fy=1500) at uniformly random directions on a radius-8 sphere,
    looking at the origin."""
    g = torch.Generator().manual_seed(1000 + seed)
    dirs = torch.nn.functional.normalize(torch.randn((C, 3), generator=g), dim=-1)
    viewmats = torch.stack([look_at(8.0 * d) for d in dirs])
    d = scene(N, seed=seed, width=1920, height=1080, fx=1500.0, cx=960.0, cy=540.0, C=C,
              viewmats=viewmats)
    d["means"] = torch.randn((N, 3), generator=torch.Generator().manual_seed(seed)) * 2.0
    return d


def config4(N=750_000, seed=4, rank=0, world=1, C=32):
    """BASELINE config 4, one rank's part: its shard of a 6M-Gaussian scene
    (means ~ N(0, 2^2)^3, the other distributions as config 0; N Gaussians drawn
    with the rank's own seed, i.i.d. like a strided slice [rank::world] of the
    whole scene) and its C / world of the C cameras at 1600x1200 (fx=fy=1200):
    uniformly random directions on a radius-8 sphere looking at the origin, the
    same C poses on every rank."""
    assert C % world == 0, "the cameras split evenly over the ranks"
    g = torch.Generator().manual_seed(2000 + seed)
    dirs = torch.nn.functional.normalize(torch.randn((C, 3), generator=g), dim=-1)
    per = C // world
    viewmats = torch.stack([look_at(8.0 * d) for d in dirs[rank * per:(rank + 1) * per]])
    shard_seed = 1000 * seed + rank
    d = scene(N, seed=shard_seed, width=1600, height=1200, fx=1200.0, cx=800.0, cy=600.0, C=per,
              viewmats=viewmats)
    d["means"] = torch.randn((N, 3), generator=torch.Generator().manual_seed(shard_seed)) * 2.0
    return d


def to(d, device):
    return {k: (v.to(device) if isinstance(v, torch.Tensor) else v) for k, v in d.items()}


def np_(t):
    return t.detach().cpu().numpy() if isinstance(t, torch.Tensor) else t
