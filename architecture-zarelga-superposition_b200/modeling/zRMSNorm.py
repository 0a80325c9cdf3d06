"""ZeroCenteredRMSNorm on the B200 kernels.

Same constructor, parameter (`weight`, zeros, the gain is 1 + weight) and
forward contract as the reference (modeling/zRMSNorm.py:4-20): computed in
f32, returned in the input dtype.  Forward and backward are single
warp-per-row kernels of libzs.so (zs_zrmsnorm_forward / _backward).
"""
from __future__ import annotations

import torch
import torch.nn as nn

from zs_b200 import _lib as Z


class ZRMSNormFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, eps):
        Z.require_cuda(x, weight)
        shape = x.shape
        d = shape[-1]
        xc = x.contiguous().view(-1, d)
        w = weight.contiguous() if weight.dtype == torch.float32 else weight.float().contiguous()
        y = torch.empty_like(xc)
        rstd = torch.empty(xc.size(0), dtype=torch.float32, device=x.device)
        Z.count(1)
        Z.check(Z.lib().zs_zrmsnorm_forward(xc.data_ptr(), w.data_ptr(), y.data_ptr(), rstd.data_ptr(), xc.size(0),
                                            d, float(eps), Z.dtype_code(xc.dtype), Z.dtype_code(w.dtype),
                                            Z.stream_of(xc)), "zs_zrmsnorm_forward")
        ctx.save_for_backward(xc, w, rstd)
        ctx.meta = (shape, weight.dtype)
        return y.view(shape)

    @staticmethod
    def backward(ctx, dy):
        xc, w, rstd = ctx.saved_tensors
        shape, w_dt = ctx.meta
        d = xc.size(1)
        dyc = dy.to(xc.dtype).contiguous().view(-1, d)
        dx = torch.empty_like(xc)
        dw = torch.empty(d, dtype=torch.float32, device=xc.device)
        ws = torch.empty(int(Z.lib().zs_zrmsnorm_backward_workspace(xc.size(0), d)), dtype=torch.uint8,
                         device=xc.device)
        Z.count(2)
        Z.check(Z.lib().zs_zrmsnorm_backward(dyc.data_ptr(), xc.data_ptr(), w.data_ptr(), rstd.data_ptr(),
                                             dx.data_ptr(), dw.data_ptr(), xc.size(0), d, Z.dtype_code(xc.dtype),
                                             Z.dtype_code(w.dtype), ws.data_ptr(), ws.numel(), Z.stream_of(xc)),
                "zs_zrmsnorm_backward")
        return dx.view(shape), dw.to(w_dt), None


class ZeroCenteredRMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float = 1e-6):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.zeros(dim))

    def forward(self, x):
        return ZRMSNormFunction.apply(x, self.weight, self.eps)

    def extra_repr(self):
        return f"{tuple(self.weight.shape)}, eps={self.eps}"
