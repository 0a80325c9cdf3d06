"""Autograd wrapper of the fused cross-entropy kernels (zs_xent_forward /
zs_xent_backward in libzs.so), shared by the MCCE and CCE drop-in modules."""
from __future__ import annotations

import torch

from . import _lib as Z
from .shadow import bf16_shadow

DEFAULT_V_CHUNK = 16384


class FusedLinearCrossEntropy(torch.autograd.Function):
    """loss = (sum_t s_t lse_t - sum_t sum_{j<s_t} z[t, labels[t, j]]) / sum_t s_t,
    z = hidden @ classifier^T, never materialised."""

    @staticmethod
    def forward(ctx, hidden, classifier, labels, s_count, v_chunk):
        Z.require_cuda(hidden, classifier, labels, s_count)
        cdt = hidden.dtype if hidden.dtype in (torch.bfloat16, torch.float16) else torch.bfloat16
        h = hidden.to(cdt).contiguous()
        c = bf16_shadow(classifier) if cdt == torch.bfloat16 else classifier.to(cdt).contiguous()
        lab = labels.to(torch.int64).contiguous()
        sc = s_count.to(torch.int32).contiguous()
        T, D = h.shape
        V = c.size(0)
        dev = h.device
        lse = torch.empty(T, dtype=torch.float32, device=dev)
        row_loss = torch.empty(T, dtype=torch.float32, device=dev)
        loss = torch.empty((), dtype=torch.float32, device=dev)
        denom = torch.empty((), dtype=torch.float32, device=dev)
        ws = torch.empty(int(Z.lib().zs_xent_forward_workspace(T, V)), dtype=torch.uint8, device=dev)
        Z.count(4)
        with Z.timed("xent_fwd", 2.0 * T * V * D):
            Z.check(Z.lib().zs_xent_forward(h.data_ptr(), T, D, h.stride(0), c.data_ptr(), V, c.stride(0),
                                            lab.data_ptr(), lab.size(1), sc.data_ptr(), lse.data_ptr(),
                                            row_loss.data_ptr(), loss.data_ptr(), denom.data_ptr(), ws.data_ptr(),
                                            ws.numel(), Z.dtype_code(cdt), Z.stream_of(h)), "zs_xent_forward")
        ctx.save_for_backward(h, c, lab, sc, lse, denom)
        ctx.meta = (hidden.dtype, classifier.dtype, int(v_chunk))
        return loss

    @staticmethod
    def backward(ctx, grad_loss):
        h, c, lab, sc, lse, denom = ctx.saved_tensors
        h_dt, c_dt, v_chunk = ctx.meta
        need_h, need_c = ctx.needs_input_grad[:2]
        T, D = h.shape
        V = c.size(0)
        dev = h.device
        g = grad_loss.detach().to(torch.float32).reshape(()).contiguous()
        dh = torch.empty((T, D), dtype=torch.float32, device=dev) if need_h else None
        dc = torch.empty((V, D), dtype=torch.float32, device=dev) if need_c else None
        if not (need_h or need_c):
            return None, None, None, None, None
        vch = min(v_chunk, ((V + 255) // 256) * 256)
        ws = torch.empty(int(Z.lib().zs_xent_backward_workspace(T, vch, Z.dtype_code(h.dtype))), dtype=torch.uint8,
                         device=dev)
        nchunks = (V + vch - 1) // vch
        Z.count(nchunks * (1 + int(need_h) + int(need_c)))
        with Z.timed("xent_bwd", 2.0 * T * V * D * (1 + int(need_h) + int(need_c))):
            Z.check(Z.lib().zs_xent_backward(h.data_ptr(), T, D, h.stride(0), c.data_ptr(), V, c.stride(0),
                                             lab.data_ptr(), lab.size(1), sc.data_ptr(), lse.data_ptr(), g.data_ptr(),
                                             denom.data_ptr(), Z.ptr(dh), Z.ptr(dc), vch, ws.data_ptr(), ws.numel(),
                                             Z.dtype_code(h.dtype), Z.stream_of(h)), "zs_xent_backward")
        return (dh.to(h_dt) if need_h else None, dc.to(c_dt) if need_c else None, None, None, None)


def fused_linear_cross_entropy(hidden, classifier, labels, s_count, v_chunk=DEFAULT_V_CHUNK):
    return FusedLinearCrossEntropy.apply(hidden, classifier, labels, s_count, v_chunk)
