"""Rasterization constants of the reference fork (gsplat/cuda/_constants.py:16-29,
gsplat/cuda/include/Common.h:73-93); the kernels use the same values."""

ALPHA_THRESHOLD = 1.0 / 255.0
MAX_ALPHA = 0.99
TRANSMITTANCE_THRESHOLD = 1e-4
MAX_KERNEL_DENSITY_CUTOFF = 0.0113
MIN_COMPENSATION = 0.005
MIN_ONE_MINUS_ALPHA = 1e-6
GAUSSIAN_EXTEND = 3.33
