"""Argument handling of the drop-in ``rasterization()`` on CPU, before any kernel
runs: options outside the training hot path raise NotImplementedError naming
them, and the reference's own argument errors (rendering.py:538-546 messages,
shape assertions, distributed restrictions) are raised the same way."""

import pytest
import torch

import gsplat_b200


def scene(N=8, C=1, sh=True):
    g = torch.Generator().manual_seed(0)
    means = torch.randn(N, 3, generator=g)
    quats = torch.nn.functional.normalize(torch.randn(N, 4, generator=g), dim=-1)
    scales = torch.rand(N, 3, generator=g) * 0.1
    opacities = torch.rand(N, generator=g)
    colors = torch.rand(N, 16, 3, generator=g) if sh else torch.rand(N, 3, generator=g)
    viewmats = torch.eye(4).expand(C, 4, 4).contiguous()
    Ks = torch.tensor([[100.0, 0, 32], [0, 100.0, 32], [0, 0, 1]]).expand(C, 3, 3).contiguous()
    return means, quats, scales, opacities, colors, viewmats, Ks, 64, 64


@pytest.mark.parametrize("kwargs, name", [
    ({"with_ut": True}, "with_ut"),
    ({"with_eval3d": True}, "with_eval3d"),
    ({"radial_coeffs": torch.zeros(1, 6)}, "radial_coeffs"),
    ({"lidar_coeffs": object()}, "lidar_coeffs"),
    ({"rolling_shutter": 1}, "rolling_shutter"),
    ({"global_z_order": False}, "global_z_order=False"),
    ({"render_mode": "RGB-Ed"}, "hit-distance render modes"),
    ({"return_normals": True}, "return_normals"),
])
def test_out_of_scope_options_raise(kwargs, name):
    with pytest.raises(NotImplementedError, match=name):
        gsplat_b200.rasterization(*scene(), sh_degree=3, **kwargs)


def test_global_rolling_shutter_is_accepted_up_to_the_device_check():
    # 4 = GLOBAL: no rolling shutter, so the call proceeds until the CPU tensors are refused
    with pytest.raises(RuntimeError, match="CUDA"):
        gsplat_b200.rasterization(*scene(), sh_degree=3, rolling_shutter=4)


def test_reference_argument_errors():
    means, quats, scales, opacities, colors, viewmats, Ks, W, H = scene()
    with pytest.raises(ValueError, match="colors must be provided"):
        gsplat_b200.rasterization(means, quats, scales, opacities, None, viewmats, Ks, W, H)
    with pytest.raises(ValueError, match="sh_degree must be None"):
        gsplat_b200.rasterization(means, quats, scales, opacities, None, viewmats, Ks, W, H, sh_degree=3,
                                  render_mode="D")
    with pytest.raises(AssertionError):
        gsplat_b200.rasterization(means[:, :2], quats, scales, opacities, colors, viewmats, Ks, W, H, sh_degree=3)
    with pytest.raises(AssertionError):
        gsplat_b200.rasterization(means, quats, scales, opacities[:-1], colors, viewmats, Ks, W, H, sh_degree=3)
    with pytest.raises(AssertionError, match="AbsGrad"):
        gsplat_b200.rasterization(means, quats, scales, opacities, colors, viewmats, Ks, W, H, sh_degree=3,
                                  absgrad=True, distributed=True)


def test_cpu_tensors_are_refused_not_rendered():
    """No CPU path: the library refuses host tensors instead of falling back."""
    with pytest.raises(RuntimeError, match="CUDA"):
        gsplat_b200.rasterization(*scene(), sh_degree=3)
