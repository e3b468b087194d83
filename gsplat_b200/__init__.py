"""gsplat_b200: B200-native (sm_100a) Gaussian-splatting training hot path.

Drop-in for the reference gsplat Python API of that path: ``rasterization``,
the ``gsplat.cuda._wrapper`` operators and ``gsplat.optimizers.SelectiveAdam``.
All compute runs in the hand-written kernels of ``libgsplat_b200.so`` (C ABI in
``include/gsplat_b200.h``); there is no CPU fallback.
"""

from .cuda._torch_impl import accumulate
from .cuda._wrapper import (
    CameraModel,
    adam,
    fully_fused_projection,
    has_2dgs,
    has_3dgs,
    has_3dgut,
    has_adam,
    has_camera_wrappers,
    has_reloc,
    isect_offset_encode,
    isect_tiles,
    persp_proj,
    proj,
    quat_scale_to_covar_preci,
    rasterize_to_indices_in_range,
    rasterize_to_pixels,
    spherical_harmonics,
    world_to_cam,
)
from .optimizers import SelectiveAdam
from .rendering import RasterizeMode, RenderMode, rasterization

__version__ = "0.1.0"

__all__ = [
    "CameraModel",
    "RasterizeMode",
    "RenderMode",
    "SelectiveAdam",
    "accumulate",
    "adam",
    "fully_fused_projection",
    "has_2dgs",
    "has_3dgs",
    "has_3dgut",
    "has_adam",
    "has_camera_wrappers",
    "has_reloc",
    "isect_offset_encode",
    "isect_tiles",
    "persp_proj",
    "proj",
    "quat_scale_to_covar_preci",
    "rasterization",
    "rasterize_to_indices_in_range",
    "rasterize_to_pixels",
    "spherical_harmonics",
    "world_to_cam",
]
