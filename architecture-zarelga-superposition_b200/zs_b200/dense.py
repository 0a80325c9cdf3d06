"""Dense projections of the training step on the grouped tcgen05 GEMM of libzs.so.

The attention input projections (q, k, v and the head gate read the same
input: one product over their concatenated weights), the attention output
projection and the shared expert's SwiGLU MLP (modeling/attention.py:187-189,226
and modeling/expert_layer.py:23-24 of the reference, nn.Linear there) run as
one-group grouped GEMMs: every row belongs to group 0, rows stay in order
(x_grouped = y_grouped), so the routed experts' kernels serve them unchanged:

  forward   Y = X W^T                       zs_scatter2scatter
            act = silu(X Wg^T) * (X Wu^T)   zs_expert_up_swiglu (SwiGLU in the epilogue)
  backward  dX = dY W                       zs_scatter2scatter on W's other major order
            dW = dY^T X (f32)               zs_group_xty_f32, straight into one f32 buffer
            d[up | gate] = SwiGLU'(dY Wd)   zs_expert_down_dswiglu (SwiGLU backward in the epilogue)

Operands are bf16 (f32 inputs and weights are rounded, as the reference's
autocast linears round them); weight gradients come back in the weights' dtype
through autograd, one slice of the f32 product per weight.
"""
from __future__ import annotations

import torch

from . import _lib as Z
from .shadow import bf16_shadow, concat_shadow

_ROUTES = {}


def one_group_routing(T: int, device) -> tuple:
    """(sorted_expert_idxs zeros [T], sorted_scattered_idxs arange [T], expert_offsets [T]) for
    a one-group GEMM over T rows in order; cached per (T, device)."""
    key = (T, str(device))
    r = _ROUTES.get(key)
    if r is None:
        r = (torch.zeros(T, dtype=torch.int64, device=device), torch.arange(T, dtype=torch.int64, device=device),
             torch.full((1,), T, dtype=torch.int64, device=device))
        if len(_ROUTES) > 16:
            _ROUTES.clear()
        _ROUTES[key] = r
    return r


def _bf16(t):
    return t if t.dtype == torch.bfloat16 else t.to(torch.bfloat16)


def _w16(w):
    """A weight in bf16: its persistent shadow when it is an f32 parameter."""
    return w if w.dtype == torch.bfloat16 else bf16_shadow(w).contiguous()


def _rows(x):
    return _bf16(x).reshape(-1, x.size(-1)).contiguous()


def _weight_cat(weights, pad):
    """bf16 row-concatenation of the weights plus `pad` zero rows: the persistent shadow buffer
    of f32 parameters (zs_b200.shadow, no per-step cast or cat), else a fresh cast/cat."""
    return concat_shadow(weights, pad)


def _product(x2, W3, tag):
    """x2 [T, K] @ W3[0] -> [T, N] (bf16) on the grouped GEMM; W3 is a [1, K, N] view with
    either of its two inner strides 1."""
    from scattermoe.kernels import ops

    T = x2.size(0)
    sei, ssi, offs = one_group_routing(T, x2.device)
    y = torch.empty((T, W3.size(2)), dtype=torch.bfloat16, device=x2.device)
    ops._launch_scatter2scatter(y, W3, x2, 1, sei, ssi, None, True, True, expert_offsets=offs, tag=tag)
    return y


_SPLITS = {}


def _split_offsets(T: int, S: int, device):
    """Inclusive row boundaries of S near-equal chunks of T rows (64-row multiples), cached."""
    key = (T, S, str(device))
    r = _SPLITS.get(key)
    if r is None:
        step = -(-T // S)
        step = -(-step // 64) * 64
        r = torch.tensor([min(T, (i + 1) * step) for i in range(S)], dtype=torch.int64, device=device)
        if len(_SPLITS) > 32:
            _SPLITS.clear()
        _SPLITS[key] = r
    return r


def _weight_grad(dy2, x2, N, K, tag):
    """f32 [N, K] = dy2^T x2.  The product's 128 x 256 output tiles are too few to fill the
    GPU for the small projections (a 1536 x 768 weight is 36 tiles for 148 SMs), so the T
    rows are split into S chunks computed as S groups of one grouped launch into f32
    partials, which are then summed in a fixed order."""
    T = x2.size(0)
    tiles = -(-N // 128) * -(-K // 256)
    S = max(1, min(8, 148 // tiles, T // 1024))
    Z.count(1)
    if S == 1:
        _, _, offs = one_group_routing(T, x2.device)
        g = torch.empty((N, K), dtype=torch.float32, device=x2.device)
    else:
        offs = _split_offsets(T, S, x2.device)
        g = torch.empty((S, N, K), dtype=torch.float32, device=x2.device)
    with Z.timed(tag, 2.0 * T * N * K):
        Z.check(Z.lib().zs_group_xty_f32(S, g.data_ptr(), N * K, 1, K, dy2.data_ptr(), dy2.stride(0), x2.data_ptr(),
                                         x2.stride(0), T, K, N, offs.data_ptr(), Z.dtype_code(x2.dtype), 0,
                                         Z.stream_of(x2)), "zs_group_xty_f32")
    return g if S == 1 else g.sum(0)


class DenseLinearFunction(torch.autograd.Function):
    """y = x @ cat(weights)^T (bf16 out); the concatenation is padded with zero rows to `pad`
    extra columns of y (callers slice them off)."""

    @staticmethod
    def forward(ctx, x, tag, pad, *weights):
        Z.require_cuda(x, *weights)
        x2 = _rows(x)
        W = _weight_cat(weights, pad)
        y = _product(x2, W.unsqueeze(0).permute(0, 2, 1), tag)
        ctx.save_for_backward(x2, W)
        ctx.meta = (tag, x.shape, x.dtype)
        ctx.weights_meta = [(w.size(0), w.dtype) for w in weights]
        return y.view(*x.shape[:-1], W.size(0))

    @staticmethod
    def backward(ctx, dy):
        x2, W = ctx.saved_tensors
        tag, x_shape, x_dt = ctx.meta
        dy2 = _rows(dy)
        grads = [None, None, None]
        if ctx.needs_input_grad[0]:
            dx = _product(dy2, W.unsqueeze(0), tag + "_dx")
            grads[0] = dx.view(x_shape).to(x_dt)
        if any(ctx.needs_input_grad[3:]):
            g = _weight_grad(dy2, x2, W.size(0), W.size(1), tag + "_dw")
            off = 0
            for n, dt in ctx.weights_meta:
                grads.append(g[off:off + n].to(dt))
                off += n
        else:
            grads.extend([None] * len(ctx.weights_meta))
        return tuple(grads)


def _out_dtype(x):
    if x.dtype in (torch.bfloat16, torch.float16) or torch.is_autocast_enabled():
        return torch.bfloat16
    return x.dtype


def dense_linear(x, weights, tag="dense", pad=0):
    """x [..., K] @ cat(weights, 0)^T on libzs, with `pad` zero output columns after the
    weights' rows (a 16-column multiple keeps the output rows 32-byte aligned).  bf16 result
    under autocast or for 16-bit inputs (what an autocast nn.Linear returns), else x's dtype."""
    y = DenseLinearFunction.apply(x, tag, int(pad), *weights)
    dt = _out_dtype(x)
    return y if y.dtype == dt else y.to(dt)


class DenseSwiGLUFunction(torch.autograd.Function):
    """down(silu(x gate^T) * (x up^T)) with the activation fused into the up-projection's
    epilogue and its backward into the down-projection's input-gradient epilogue."""

    @staticmethod
    def forward(ctx, x, w_gate, w_up, w_down, tag):
        from scattermoe.mlp import up_swiglu
        from scattermoe.kernels import ops

        Z.require_cuda(x, w_gate, w_up, w_down)
        x2 = _rows(x)
        T = x2.size(0)
        f = w_up.size(0)
        sei, ssi, offs = one_group_routing(T, x2.device)
        W1 = concat_shadow([w_up, w_gate]).unsqueeze(0)                  # [1, 2f, d]: up rows, then gate rows
        W2 = _w16(w_down).unsqueeze(0)                                    # [1, d, f]
        act, hfull = up_swiglu(x2, W1, sei, offs)
        y = torch.empty((T, W2.size(1)), dtype=torch.bfloat16, device=x2.device)
        ops._launch_scatter2scatter(y, W2.permute(0, 2, 1), act, 1, sei, ssi, None, True, True,
                                    expert_offsets=offs, tag=tag + "_down")
        ctx.save_for_backward(x2, act, hfull, W1, W2)
        ctx.meta = (tag, x.shape, x.dtype, f, w_gate.dtype, w_up.dtype, w_down.dtype)
        return y.view(*x.shape[:-1], W2.size(1))

    @staticmethod
    def backward(ctx, dy):
        from scattermoe.mlp import down_dswiglu
        from scattermoe.kernels import ops

        x2, act, hfull, W1, W2 = ctx.saved_tensors
        tag, x_shape, x_dt, f, g_dt, u_dt, d_dt = ctx.meta
        dy2 = _rows(dy)
        T, d = x2.shape
        sei, ssi, offs = one_group_routing(T, x2.device)
        dh = down_dswiglu(dy2, W2, hfull, sei, offs)                        # [T, 2f]: d(up) | d(gate)
        g_down = _weight_grad(dy2, act, d, f, tag + "_down_dw")
        g_up_gate = _weight_grad(dh, x2, 2 * f, d, tag + "_up_dw")
        dx = torch.empty((T, d), dtype=torch.bfloat16, device=x2.device)
        ops._launch_scatter2scatter(dx, W1, dh, 1, sei, ssi, None, True, True, expert_offsets=offs,
                                    tag=tag + "_up_dx")
        return (dx.view(x_shape).to(x_dt), g_up_gate[f:].to(g_dt), g_up_gate[:f].to(u_dt), g_down.to(d_dt), None)


def dense_swiglu(x, w_gate, w_up, w_down, tag="shared_expert"):
    """down(silu(x @ w_gate^T) * (x @ w_up^T)) on libzs (dtype as dense_linear)."""
    y = DenseSwiGLUFunction.apply(x, w_gate, w_up, w_down, tag)
    dt = _out_dtype(x)
    return y if y.dtype == dt else y.to(dt)
