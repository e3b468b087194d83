"""Alpha compositing in plain PyTorch over the index triples of
rasterize_to_indices_in_range: the reference's accumulate() and
_rasterize_to_pixels() (gsplat/cuda/_torch_impl.py:472-683), a slow path for
experiments and debugging whose backward is PyTorch autograd. The reference
needs nerfacc for the per-pixel transmittance; here nerfacc's
render_weight_from_alpha / accumulate_along_rays are segment ops over the
pairs, which rasterize_to_indices_in_range returns grouped by pixel and front
to back. The training path (rasterization()) never uses this module."""

import math

import torch

MAX_ALPHA = 0.99


def accumulate(means2d, conics, opacities, colors, gaussian_ids, pixel_ids, image_ids, width, height):
    """Reference _torch_impl.py:472-570: composites the listed (Gaussian, pixel,
    image) pairs front to back; returns renders [..., H, W, channels] and alphas
    [..., H, W, 1] as if every pixel started at transmittance 1."""
    image_dims = means2d.shape[:-2]
    I = math.prod(image_dims)
    N = means2d.shape[-2]
    ch = colors.shape[-1]
    means2d = means2d.reshape(I, N, 2)
    conics = conics.reshape(I, N, 3)
    opacities = opacities.reshape(I, N)
    colors = colors.reshape(I, N, ch)
    px = (pixel_ids % width).to(means2d.dtype) + 0.5
    py = torch.div(pixel_ids, width, rounding_mode="floor").to(means2d.dtype) + 0.5
    d = torch.stack([px, py], -1) - means2d[image_ids, gaussian_ids]
    c = conics[image_ids, gaussian_ids]
    sigma = 0.5 * (c[:, 0] * d[:, 0] ** 2 + c[:, 2] * d[:, 1] ** 2) + c[:, 1] * d[:, 0] * d[:, 1]
    alpha = torch.clamp_max(opacities[image_ids, gaussian_ids] * torch.exp(-sigma), MAX_ALPHA)
    ray = image_ids * height * width + pixel_ids
    n_rays = I * height * width
    # exclusive transmittance inside each ray: exp of the exclusive cumulative sum
    # of log(1 - alpha), restarted at each ray's first entry (in float64: the sum
    # runs over all rays, and its differences must keep float32 precision)
    log1m = torch.log1p(-alpha.double())
    excl = torch.cumsum(log1m, 0) - log1m
    first = torch.ones_like(ray, dtype=torch.bool)
    first[1:] = ray[1:] != ray[:-1]
    seg = torch.cumsum(first.to(torch.int64), 0) - 1
    start_val = excl[first][seg]
    weights = torch.exp(excl - start_val).to(alpha.dtype) * alpha
    renders = torch.zeros((n_rays, ch), dtype=colors.dtype, device=colors.device)
    renders = renders.index_add(0, ray, weights[:, None] * colors[image_ids, gaussian_ids])
    alphas = torch.zeros((n_rays, 1), dtype=colors.dtype, device=colors.device).index_add(0, ray, weights[:, None])
    return (renders.reshape(image_dims + (height, width, ch)), alphas.reshape(image_dims + (height, width, 1)))


def _rasterize_to_pixels(means2d, conics, colors, opacities, width, height, tile_size, isect_offsets,
                         flatten_ids, backgrounds=None, batch_per_iter=100):
    """Reference _torch_impl.py:573-683: rasterize_to_pixels as alternating
    rasterize_to_indices_in_range and accumulate() over batch_per_iter splat
    batches at a time."""
    from ._wrapper import rasterize_to_indices_in_range

    image_dims = means2d.shape[:-2]
    ch = colors.shape[-1]
    dev = means2d.device
    n_isects = len(flatten_ids)
    render_colors = torch.zeros(image_dims + (height, width, ch), device=dev)
    render_alphas = torch.zeros(image_dims + (height, width, 1), device=dev)
    block = tile_size * tile_size
    offs = torch.cat([isect_offsets.flatten(), torch.tensor([n_isects], device=dev)])
    max_range = int((offs[1:] - offs[:-1]).max().item())
    n_batches = (max_range + block - 1) // block
    for step in range(0, n_batches, batch_per_iter):
        trans = 1.0 - render_alphas[..., 0]
        gids, pids, iids = rasterize_to_indices_in_range(step, step + batch_per_iter, trans.detach(), means2d,
                                                         conics, opacities, width, height, tile_size,
                                                         isect_offsets, flatten_ids)
        if len(gids) == 0:
            break
        r, a = accumulate(means2d, conics, opacities, colors, gids, pids, iids, width, height)
        render_colors = render_colors + r * trans[..., None]
        render_alphas = render_alphas + a * trans[..., None]
    if backgrounds is not None:
        render_colors = render_colors + backgrounds[..., None, None, :] * (1.0 - render_alphas)
    return render_colors, render_alphas
