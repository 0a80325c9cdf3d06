"""GramReaperSparse (engram/GramReaperSparse.py:7-66): per-row RMSProp on a
sparse (COO) embedding gradient, optionally re-projecting each touched row
onto the unit L2 sphere."""
from __future__ import annotations

import torch
from torch.optim import Optimizer


class GramReaperSparse(Optimizer):
    def __init__(self, params, lr: float = 1e-2, beta: float = 0.9, eps: float = 1e-10, unit_norm: bool = False):
        if lr <= 0:
            raise ValueError(f"lr must be > 0, got {lr}")
        if not (0.0 < beta < 1.0):
            raise ValueError(f"beta must be in (0, 1), got {beta}")
        super().__init__(params, dict(lr=lr, beta=beta, eps=eps, unit_norm=unit_norm))

    @torch.no_grad()
    def step(self, closure=None):
        loss = closure() if closure is not None else None
        for group in self.param_groups:
            lr, beta, eps, unit = group["lr"], group["beta"], group["eps"], group["unit_norm"]
            for p in group["params"]:
                if p.grad is None:
                    continue
                if p.dim() != 2:
                    raise ValueError("GramReaperSparse supports 2-D params [n_rows, dim] only")
                if not p.grad.is_sparse:
                    raise ValueError("GramReaperSparse expects a sparse gradient (nn.Embedding(..., sparse=True))")
                grad = p.grad.coalesce()
                idx = grad.indices()[0]
                g = grad.values()
                if idx.numel() == 0:
                    continue
                state = self.state[p]
                if "v" not in state:
                    state["v"] = torch.zeros(p.shape[0], dtype=p.dtype, device=p.device)
                    state["t"] = 0
                state["t"] += 1
                v = state["v"]
                v[idx] = beta * v[idx] + (1 - beta) * (g * g).sum(dim=1)
                step = lr / ((v[idx] / (1 - beta ** state["t"])).sqrt() + eps)
                row = p.data[idx] - step.unsqueeze(1) * g
                if unit:
                    row = row / row.norm(dim=1, keepdim=True).clamp_min(eps)
                p.data[idx] = row
        return loss
