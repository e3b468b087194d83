"""Densification-strategy support for the training hot path.

``update_state`` is a drop-in for the reference's
``DefaultStrategy._update_state`` (gsplat/strategy/default.py:218-276): same
arguments, same state tensors ("grad2d", "count", "radii"), computed by one
kernel (``gsb_densify_accumulate``) instead of a chain of tensor ops. A trainer
that uses the reference's strategy classes binds it with

    DefaultStrategy._update_state = gsplat_b200.strategy.update_state
"""

from typing import Any, Dict

import torch

from ..cuda import _backend as _B
from ..cuda._backend import call, check_cuda, device_guard, ptr, stream_of

__all__ = ["update_state", "accumulate_screen_stats"]


def accumulate_screen_stats(grads: torch.Tensor, radii: torch.Tensor, width: int, height: int, n_cameras: int,
                            grad2d: torch.Tensor, count: torch.Tensor, max_radii=None, gaussian_ids=None) -> None:
    """Adds the normalised 2D gradient norms and view counts of one step to
    ``grad2d`` / ``count`` (and the largest normalised radius to ``max_radii``).
    ``grads``/``radii``: [nnz, 2] with ``gaussian_ids`` [nnz] (packed), or
    [C, N, 2] (dense; a pair counts when both radii are positive)."""
    N = grad2d.numel()
    grads = grads.contiguous()
    radii = radii.to(torch.int32).contiguous()
    if gaussian_ids is not None:
        gaussian_ids = gaussian_ids.to(torch.int64).contiguous()
    n = grads.numel() // 2
    for name, t in (("grads", grads), ("radii", radii), ("grad2d", grad2d), ("count", count),
                    ("max_radii", max_radii), ("gaussian_ids", gaussian_ids)):
        check_cuda(name, t)
    with device_guard(grads.device):
        call("gsb_densify_accumulate", n, N, ptr(gaussian_ids), ptr(grads), ptr(radii), int(width), int(height),
             int(n_cameras), ptr(grad2d), ptr(count), ptr(max_radii), stream_of(grads))


def update_state(strategy: Any, params, state: Dict[str, Any], info: Dict[str, Any], packed: bool = False) -> None:
    """DefaultStrategy._update_state: reads ``strategy.absgrad``,
    ``strategy.key_for_gradient`` and ``strategy.refine_scale2d_stop_iter`` like
    the reference method, creates the state tensors on first use and adds this
    step's statistics."""
    key = getattr(strategy, "key_for_gradient", "means2d")
    for k in ["width", "height", "n_cameras", "radii", "gaussian_ids", key]:
        assert k in info, f"{k} is required but missing."
    src = info[key]
    grads = src.absgrad if getattr(strategy, "absgrad", False) else src.grad
    n_gaussian = len(list(params.values())[0])
    dev = grads.device
    if state["grad2d"] is None:
        state["grad2d"] = torch.zeros(n_gaussian, device=dev)
    if state["count"] is None:
        state["count"] = torch.zeros(n_gaussian, device=dev)
    use_radii = getattr(strategy, "refine_scale2d_stop_iter", 0) > 0
    if use_radii and state["radii"] is None:
        state["radii"] = torch.zeros(n_gaussian, device=dev)
    accumulate_screen_stats(grads, info["radii"], info["width"], info["height"], info["n_cameras"],
                            state["grad2d"], state["count"], state["radii"] if use_radii else None,
                            info["gaussian_ids"] if packed else None)
