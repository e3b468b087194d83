"""SelectiveAdam: masked Adam whose whole step is one fused kernel launch.

Same class, constructor and ``step(visibility)`` contract as the reference's
``gsplat/optimizers/selective_adam.py:21-101``: a ``torch.optim.Adam`` subclass,
one tensor per parameter group, lazily created ``exp_avg`` / ``exp_avg_sq`` /
``step`` state (so ``state_dict()`` checkpoints are interchangeable), no bias
correction, rows whose visibility is False left untouched. Where the reference
launches one kernel per group, all groups go through ``gsb_adam_multi`` in one
launch.
"""

import torch

from ..cuda._wrapper import adam_multi


class SelectiveAdam(torch.optim.Adam):
    def __init__(self, params, eps, betas):
        super().__init__(params=params, eps=eps, betas=betas)

    @torch.no_grad()
    def step(self, visibility):
        visibility = visibility.contiguous()
        groups = {}
        for group in self.param_groups:
            lr = group["lr"]
            eps = group["eps"]
            beta1, beta2 = group["betas"]
            assert len(group["params"]) == 1, "more than one tensor in group"
            param = group["params"][0]
            if param.grad is None:
                continue
            state = self.state[param]
            if len(state) == 0:
                state["step"] = torch.tensor(0.0, dtype=torch.float32)
                state["exp_avg"] = torch.zeros_like(param, memory_format=torch.preserve_format)
                state["exp_avg_sq"] = torch.zeros_like(param, memory_format=torch.preserve_format)
            grad = param.grad
            if grad.is_sparse:
                grad = grad.to_dense()
            grad = grad.contiguous()
            groups.setdefault((beta1, beta2), []).append(
                (param, grad, state["exp_avg"], state["exp_avg_sq"], lr, eps))
        for (b1, b2), entries in groups.items():
            adam_multi(entries, visibility, b1, b2)
