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


class AddZRMSNormFunction(torch.autograd.Function):
    """(h, y) = (x + r, bf16 zRMSNorm(x + r)) for an f32 residual stream x and a bf16
    branch r in one pass (r None: y = bf16 zRMSNorm(x), h is x).  The values equal
    the reference block's `h = x + branch` (f32) followed by the norm (f32) and the
    bf16 cast its next autocast GEMM applies; the backward adds the residual-path
    gradient of h and writes the bf16 gradient of r in the same pass."""

    @staticmethod
    def forward(ctx, x, r, weight, eps):
        Z.require_cuda(x, weight)
        shape = x.shape
        d = shape[-1]
        xc = x.contiguous().view(-1, d)
        w = weight.contiguous() if weight.dtype == torch.float32 else weight.float().contiguous()
        rows = xc.size(0)
        rc = r.contiguous().view(-1, d) if r is not None else None
        h = torch.empty_like(xc) if rc is not None else xc
        y = torch.empty(xc.shape, dtype=torch.bfloat16, device=x.device)
        rstd = torch.empty(rows, dtype=torch.float32, device=x.device)
        Z.count(1)
        Z.check(Z.lib().zs_add_zrmsnorm_forward(xc.data_ptr(), Z.ptr(rc), w.data_ptr(),
                                                h.data_ptr() if rc is not None else None, y.data_ptr(),
                                                rstd.data_ptr(), rows, d, float(eps), Z.stream_of(xc)),
                "zs_add_zrmsnorm_forward")
        ctx.save_for_backward(h, w, rstd)
        ctx.meta = (shape, weight.dtype, r is not None, r.dtype if r is not None else None)
        if rc is not None:
            return h.view(shape), y.view(shape)
        return y.view(shape)

    @staticmethod
    def backward(ctx, *grads):
        h, w, rstd = ctx.saved_tensors
        shape, w_dt, has_r, r_dt = ctx.meta
        d = h.size(1)
        rows = h.size(0)
        if has_r:
            dh, dy = grads
        else:
            (dy,) = grads
            dh = None
        dyc = (dy if dy is not None else torch.zeros(shape, dtype=torch.bfloat16, device=h.device))
        dyc = dyc.to(torch.bfloat16).contiguous().view(-1, d)
        dhc = dh.float().contiguous().view(-1, d) if dh is not None else None
        dx = torch.empty_like(h)
        dr = torch.empty(h.shape, dtype=torch.bfloat16, device=h.device) if has_r else None
        dw = torch.empty(d, dtype=torch.float32, device=h.device)
        ws = torch.empty(int(Z.lib().zs_zrmsnorm_backward_workspace(rows, d)), dtype=torch.uint8, device=h.device)
        Z.count(2)
        Z.check(Z.lib().zs_add_zrmsnorm_backward(dyc.data_ptr(), h.data_ptr(), w.data_ptr(), rstd.data_ptr(),
                                                 Z.ptr(dhc), dx.data_ptr(), Z.ptr(dr), dw.data_ptr(), rows, d,
                                                 ws.data_ptr(), ws.numel(), Z.stream_of(h)),
                "zs_add_zrmsnorm_backward")
        gr = dr.view(shape).to(r_dt) if has_r else None
        return dx.view(shape), gr, dw.to(w_dt), None


def fused_add_norm_ok(x, r=None) -> bool:
    """The fused residual-add + norm path applies: f32 CUDA residual stream, bf16 branch,
    row width a multiple of 128 the kernel is built for."""
    d = x.size(-1)
    return (x.is_cuda and x.dtype == torch.float32 and (r is None or r.dtype == torch.bfloat16)
            and d % 128 == 0 and d // 128 in (1, 2, 4, 8, 12, 16))


class ZeroCenteredRMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float = 1e-6):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.zeros(dim))

    def forward(self, x):
        return ZRMSNormFunction.apply(x, self.weight, self.eps)

    def extra_repr(self):
        return f"{tuple(self.weight.shape)}, eps={self.eps}"
