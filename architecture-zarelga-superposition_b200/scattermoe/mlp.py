"""scattermoe.mlp on the B200 kernels.

MLP and GLUMLP keep the reference's constructor arguments, parameter names
and shapes (scattermoe/mlp.py:6-95): experts.weight [E, 2f, d] for GLUMLP with
the first f rows the "up" half and the last f rows the "gate" half, and
output_experts.weight [E, d, f].

GLUMLP.forward runs one autograd function whose forward is
  sort -> gather -> grouped GEMM with SwiGLU fused in its epilogue ->
  grouped GEMM scattered to (token, slot) rows -> gate-weighted combine
and whose backward is the reference's ParallelLinear backward for both
projections, with the SwiGLU backward fused into the epilogue of the
down-projection's input-gradient GEMM.
"""
from __future__ import annotations

import torch
from torch import nn

from zs_b200 import _lib as Z
from zs_b200.shadow import bf16_shadow
from .kernels import ops
from .parallel_experts import ParallelExperts, flatten_sort_count


def _compute_dtype(x: torch.Tensor) -> torch.dtype:
    return x.dtype if x.dtype in (torch.bfloat16, torch.float16) else torch.bfloat16


def weighted_row_sum(rows: torch.Tensor, weights, T: int, k: int) -> torch.Tensor:
    """out[t] = sum_j w[t, j] * rows[t*k + j] (plain sum when weights is None)."""
    C = rows.size(1)
    out = torch.empty((T, C), dtype=rows.dtype, device=rows.device)
    w = None if weights is None else weights.contiguous()
    Z.count(1)
    Z.check(Z.lib().zs_weighted_row_sum(out.data_ptr(), out.stride(0), rows.data_ptr(), rows.stride(0), Z.ptr(w),
                                        Z.dtype_code(w.dtype) if w is not None else 0, T, k, C,
                                        Z.dtype_code(rows.dtype), Z.stream_of(rows)), "zs_weighted_row_sum")
    return out


def up_swiglu(xg, W1, sorted_expert_idxs, expert_offsets):
    """(act [n, f], hfull [n, 2f]) of the fused up projection."""
    n, d = xg.shape
    E, f2, _ = W1.shape
    f = f2 // 2
    act = torch.empty((n, f), dtype=xg.dtype, device=xg.device)
    hfull = torch.empty((n, f2), dtype=xg.dtype, device=xg.device)
    Z.count(1)
    with Z.timed("up_swiglu", 4.0 * n * d * f):
        Z.check(Z.lib().zs_expert_up_swiglu(act.data_ptr(), hfull.data_ptr(), W1.data_ptr(), E, d, f,
                                            xg.data_ptr(), xg.stride(0), sorted_expert_idxs.data_ptr(),
                                            expert_offsets.data_ptr(), n, Z.dtype_code(xg.dtype), Z.stream_of(xg)),
                "zs_expert_up_swiglu")
    return act, hfull


def down_dswiglu(dyg, W2, hfull, sorted_expert_idxs, expert_offsets):
    """d[h | g] [n, 2f] of the SwiGLU input from the gate-scaled grouped output
    gradient, in one grouped GEMM whose epilogue applies the SwiGLU backward."""
    n, d = dyg.shape
    E, _, f = W2.shape
    dh = torch.empty((n, 2 * f), dtype=dyg.dtype, device=dyg.device)
    Z.count(1)
    with Z.timed("down_dx", 2.0 * n * d * f):
        Z.check(Z.lib().zs_expert_down_dswiglu(dh.data_ptr(), hfull.data_ptr(), W2.data_ptr(), E, d, f,
                                               dyg.data_ptr(), dyg.stride(0), sorted_expert_idxs.data_ptr(),
                                               expert_offsets.data_ptr(), n, Z.dtype_code(dyg.dtype),
                                               Z.stream_of(dyg)), "zs_expert_down_dswiglu")
    return dh


def swiglu_backward(dact, hfull):
    n, f = dact.shape
    dh = torch.empty((n, 2 * f), dtype=dact.dtype, device=dact.device)
    Z.count(1)
    Z.check(Z.lib().zs_swiglu_backward(dh.data_ptr(), dact.data_ptr(), hfull.data_ptr(), n, f,
                                       Z.dtype_code(dact.dtype), Z.stream_of(dact)), "zs_swiglu_backward")
    return dh


def accumulate_weight_grad(W, DY, X, offs, tag):
    """W.grad (W's [E, N, K] layout) += DY_e^T X_e per expert, straight from the GEMM epilogue:
    f32 weights accumulate in f32; 16-bit weights get their gradient written in their dtype
    (added to an existing .grad).  W.grad is created when absent, and overwritten instead of
    accumulated when an optimizer's zero_grad marked it stale (W._zs_grad_stale, see
    optimizer.hybrid.HybridGraphOptimizer.zero_grad).  Data-parallel reducers registered for
    W are told the gradient is complete (zs_b200.dp.notify_grad_ready)."""
    from zs_b200.dp import notify_grad_ready

    E, N, K = W.shape
    g = W.grad
    if g is not None and (g.dtype != W.dtype or not g.is_contiguous() or g.is_sparse):
        raise Z.ZsError("fused weight-gradient accumulation needs a dense contiguous .grad of the weight's dtype")
    Z.count(1)
    if W.dtype == torch.float32:
        acc = 1
        if g is None:
            g = W.grad = torch.empty_like(W, memory_format=torch.contiguous_format)
            acc = 0
        elif getattr(W, "_zs_grad_stale", False):
            acc = 0   # zero_grad left this buffer stale: the GEMM overwrites it
        W._zs_grad_stale = False
        with Z.timed(tag, 2.0 * X.size(0) * K * N):
            Z.check(Z.lib().zs_group_xty_f32(E, g.data_ptr(), N * K, 1, K, DY.data_ptr(), DY.stride(0),
                                             X.data_ptr(), X.stride(0), X.size(0), K, N, offs.data_ptr(),
                                             Z.dtype_code(X.dtype), acc, Z.stream_of(X)), "zs_group_xty_f32")
    else:
        out = torch.empty_like(W, memory_format=torch.contiguous_format) if g is None else torch.empty_like(g)
        with Z.timed(tag, 2.0 * X.size(0) * K * N):
            Z.check(Z.lib().zs_group_xty(E, out.data_ptr(), N * K, 1, K, None, 0, 0, DY.data_ptr(), DY.stride(0),
                                         X.data_ptr(), X.stride(0), X.size(0), K, N, offs.data_ptr(),
                                         Z.dtype_code(X.dtype), Z.stream_of(X)), "zs_group_xty")
        if g is None:
            W.grad = out
        else:
            g.add_(out)
    notify_grad_ready(W)


class GLUExpertsFunction(torch.autograd.Function):
    """Fused GLU experts.  With fuse_wgrad the weights' gradients are accumulated into
    W1.grad / W2.grad by the weight-gradient GEMMs themselves (and None is returned for them),
    which skips the bf16 gradient's permuted copy, its cast and autograd's accumulation pass,
    and lets a data-parallel reducer start on each as soon as it is complete."""

    @staticmethod
    def forward(ctx, x, expert_p, expert_idxs, W1, W2, num_experts, k, fuse_wgrad=False, shared=None, residual=None):
        Z.require_cuda(x, expert_p, expert_idxs, W1, W2, shared, residual)
        cdt = _compute_dtype(x)
        xc = x.to(cdt).contiguous()
        # f32 master weights are read through their bf16 shadows (zs_b200.shadow): cast once,
        # then kept in step by the optimizer instead of re-cast every forward
        W1c = bf16_shadow(W1) if cdt == torch.bfloat16 else W1.to(cdt).contiguous()
        W2c = bf16_shadow(W2) if cdt == torch.bfloat16 else W2.to(cdt).contiguous()
        pc = expert_p.to(cdt).contiguous()
        T = xc.size(0)
        sei, ssi, offs = flatten_sort_count(expert_idxs, num_experts)
        xg = ops.group(xc, ssi, fan_out=k)
        act, hfull = up_swiglu(xg, W1c, sei, offs)
        y_rows = torch.empty((T * k, W2c.size(1)), dtype=cdt, device=x.device)
        ops._launch_scatter2scatter(y_rows, W2c.permute(0, 2, 1), act, 1, sei, ssi, None, True, False,
                                    expert_offsets=offs, tag="down_fwd")
        ctx.save_for_backward(xg, act, hfull, y_rows, sei, ssi, offs, pc, W1c, W2c)
        ctx.meta = (x.dtype, expert_p.dtype, W1.dtype, W2.dtype, num_experts, k, T)
        ctx.fused_params = (W1, W2) if fuse_wgrad and W1.is_leaf and W2.is_leaf else None
        ctx.closed = shared is not None or residual is not None
        if ctx.closed:
            # residual + (shared + routed) in f32, one pass (zs_moe_combine)
            y = torch.empty((T, W2c.size(1)), dtype=torch.float32, device=x.device)
            sh = shared.reshape(T, -1).to(cdt).contiguous() if shared is not None else None
            rs = residual.reshape(T, -1).contiguous() if residual is not None else None
            if rs is not None and rs.dtype != torch.float32:
                raise Z.ZsError("the residual stream of the fused MoE close must be f32")
            Z.count(1)
            Z.check(Z.lib().zs_moe_combine(y.data_ptr(), y.stride(0), y_rows.data_ptr(), y_rows.stride(0),
                                           pc.data_ptr(), Z.dtype_code(pc.dtype), T, k, y.size(1),
                                           Z.dtype_code(cdt), Z.ptr(sh), sh.stride(0) if sh is not None else 0,
                                           Z.ptr(rs), rs.stride(0) if rs is not None else 0, Z.stream_of(y)),
                    "zs_moe_combine")
            ctx.shared_meta = (shared.shape, shared.dtype) if shared is not None else None
            ctx.residual_meta = (residual.shape, residual.dtype) if residual is not None else None
            return y
        y = weighted_row_sum(y_rows, pc, T, k)
        return y.to(x.dtype)

    @staticmethod
    def backward(ctx, dy):
        xg, act, hfull, y_rows, sei, ssi, offs, pc, W1c, W2c = ctx.saved_tensors
        x_dt, p_dt, w1_dt, w2_dt, E, k, T = ctx.meta
        cdt = xg.dtype
        dyc = dy.to(cdt).contiguous()
        d = dyc.size(1)
        d_p = ops.rowwise_sum_product(y_rows.view(T, k, d), dyc, dtype=p_dt)
        dyg = ops.group(dyc, ssi, fan_out=k, coeff=pc.flatten())
        dhfull = down_dswiglu(dyg, W2c, hfull, sei, offs)
        if ctx.fused_params is not None:
            # W1's gradient first: its data-parallel all-reduce (the larger one) then
            # overlaps the two GEMMs that follow
            W1, W2 = ctx.fused_params
            if ctx.needs_input_grad[3]:
                accumulate_weight_grad(W1, dhfull, xg, offs, "up_dw")
            if ctx.needs_input_grad[4]:
                accumulate_weight_grad(W2, dyg, act, offs, "down_dw")
            gW1 = gW2 = None
        else:
            dW2, _ = ops.group_bwd_W(dyg, act, offs, E, tag="down_dw")   # [E, f, d] view of [E, d, f]
            dW1, _ = ops.group_bwd_W(dhfull, xg, offs, E, tag="up_dw")   # [E, d, 2f] view of [E, 2f, d]
            gW1, gW2 = dW1.permute(0, 2, 1).to(w1_dt), dW2.permute(0, 2, 1).to(w2_dt)
        dx_rows = torch.empty((T * k, xg.size(1)), dtype=cdt, device=dy.device)
        ops._launch_scatter2scatter(dx_rows, W1c, dhfull, 1, sei, ssi, None, True, False, expert_offsets=offs,
                                    tag="up_dx")
        dx = weighted_row_sum(dx_rows, None, T, k)
        d_shared = d_res = None
        if ctx.closed:
            # the f32 gradient of the closed sum goes to the residual as is and, in the
            # compute dtype already cast once above, to the shared expert
            if ctx.shared_meta is not None:
                d_shared = dyc.view(ctx.shared_meta[0]).to(ctx.shared_meta[1])
            if ctx.residual_meta is not None:
                d_res = dy.view(ctx.residual_meta[0])
        return dx.to(x_dt), d_p, None, gW1, gW2, None, None, None, d_shared, d_res


class MLP(nn.Module):
    def __init__(self, input_size, hidden_size, num_experts, top_k, bias=False, activation=None):
        super().__init__()
        self.num_experts = num_experts
        self.input_size = input_size
        self.hidden_size = hidden_size
        self.experts = ParallelExperts(num_experts, input_size, hidden_size, bias=bias)
        self.output_experts = ParallelExperts(num_experts, hidden_size, input_size, bias=bias)
        self.top_k = min(top_k, self.num_experts)
        self.activation = activation

    def extra_repr(self):
        return "k={}".format(self.top_k)

    def forward(self, x: torch.Tensor, expert_p: torch.Tensor, expert_idxs: torch.Tensor):
        x_shape = x.size()
        x = x.view(-1, x_shape[-1])
        sei, ssi, offs = flatten_sort_count(expert_idxs, num_experts=self.num_experts)
        h = self.experts(x, self.top_k, sei, ssi, offs, grouped_out=True)
        h = self.activation(h)
        y = self.output_experts(h, 1, sei, ssi, offs, grouped_in=True, gates=expert_p)
        return y.view(*x_shape[:-1], y.size(-1))


class GLUMLP(nn.Module):
    def __init__(self, input_size, hidden_size, num_experts, top_k, bias=False, activation=nn.SiLU()):
        super().__init__()
        self.num_experts = num_experts
        self.input_size = input_size
        self.hidden_size = hidden_size
        self.experts = ParallelExperts(num_experts, input_size, 2 * hidden_size, bias=bias)
        self.output_experts = ParallelExperts(num_experts, hidden_size, input_size, bias=bias)
        self.top_k = min(top_k, self.num_experts)
        self.activation = activation
        # When set, backward adds the f32 expert weight gradients into .grad directly (see
        # GLUExpertsFunction); torch.autograd.grad then sees no gradient for these weights.
        self.fuse_weight_grad = False

    def extra_repr(self):
        return "k={}".format(self.top_k)

    def _fused_ok(self) -> bool:
        return self.experts.bias is None and isinstance(self.activation, nn.SiLU)

    def forward(self, x: torch.Tensor, expert_p: torch.Tensor, expert_idxs: torch.Tensor, shared=None,
                residual=None):
        """y = the routed experts' output; with shared and/or residual (this package's fused
        path only: bias-free SiLU experts, k <= 8, 16-bit compute) y = residual + (shared + routed)
        in f32, the transformer block's MoE close in one pass."""
        x_shape = x.size()
        x = x.view(-1, x_shape[-1])
        if shared is not None or residual is not None:
            if not (self._fused_ok() and self.top_k <= 8):
                raise Z.ZsError("the fused MoE close needs bias-free SiLU experts with top_k <= 8")
            y = GLUExpertsFunction.apply(x, expert_p.reshape(x.size(0), -1), expert_idxs.reshape(x.size(0), -1),
                                         self.experts.weight, self.output_experts.weight, self.num_experts,
                                         self.top_k, self.fuse_weight_grad, shared, residual)
        elif self._fused_ok():
            y = GLUExpertsFunction.apply(x, expert_p.reshape(x.size(0), -1), expert_idxs.reshape(x.size(0), -1),
                                         self.experts.weight, self.output_experts.weight, self.num_experts,
                                         self.top_k, self.fuse_weight_grad)
        else:
            sei, ssi, offs = flatten_sort_count(expert_idxs, num_experts=self.num_experts)
            h, gates = self.experts(x, self.top_k, sei, ssi, offs, grouped_out=True).chunk(2, dim=-1)
            h = self.activation(gates) * h
            y = self.output_experts(h, 1, sei, ssi, offs, grouped_in=True, gates=expert_p)
        return y.view(*x_shape[:-1], y.size(-1))
