"""`linear_cross_entropy` on the B200 kernels, importable as the third-party
`cut_cross_entropy` package the reference trainer uses (main.py:24, called at
main.py:761 as linear_cross_entropy(e, c, targets, ignore_index=-100)).

Mean next-token cross entropy of e @ c^T over the targets that are not
ignore_index, computed by libzs.so's fused classifier GEMM without storing
logits.  Only the arguments the reference passes are supported; other
options of the upstream package raise NotImplementedError.
"""
from __future__ import annotations

import torch

from zs_b200.xent import DEFAULT_V_CHUNK, fused_linear_cross_entropy

__all__ = ["linear_cross_entropy"]


def linear_cross_entropy(e: torch.Tensor, c: torch.Tensor, targets: torch.Tensor, bias=None,
                         ignore_index: int = -100, softcap=None, reduction: str = "mean", shift: bool = False,
                         **unsupported) -> torch.Tensor:
    if bias is not None or softcap is not None or shift or unsupported:
        raise NotImplementedError("only linear_cross_entropy(e, c, targets, ignore_index=..., reduction=...) "
                                  "is provided")
    if reduction not in ("mean", "sum"):
        raise NotImplementedError(f"reduction={reduction!r}")
    D = e.size(-1)
    h = e.reshape(-1, D)
    t = targets.reshape(-1)
    active = t != ignore_index
    labels = torch.where(active, t, torch.zeros_like(t)).to(torch.int64).unsqueeze(1)
    s = active.to(torch.int32)
    loss = fused_linear_cross_entropy(h, c, labels, s, DEFAULT_V_CHUNK)
    if reduction == "sum":
        loss = loss * s.sum().to(loss.dtype)
    return loss
