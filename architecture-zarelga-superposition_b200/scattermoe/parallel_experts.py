"""scattermoe.parallel_experts on the B200 kernels.

Mirrors the reference module (scattermoe/parallel_experts.py): the
scattermoe::bincount op (:6-19), flatten_sort_count (:21-28), the
ParallelLinear autograd function (:32-135), parallel_linear (:137-147) and the
ParallelExperts module (:149-183, weight [E, out, in], N(0, 0.02) init).
The sort and the counts run in the routing kernels of libzs.so; the linear
layers run in its tcgen05 grouped GEMM.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from zs_b200 import _lib as Z
from . import kernels


@torch.library.custom_op("scattermoe::bincount", mutates_args={})
def compileable_bincount(x: torch.Tensor, minlength: int) -> torch.Tensor:
    Z.require_cuda(x)
    xl = x if (x.dtype == torch.int64 and x.is_contiguous()) else x.long().contiguous()
    out = torch.empty(minlength, dtype=torch.long, device=x.device)
    Z.count(1)
    Z.check(Z.lib().zs_bincount(xl.data_ptr(), xl.numel(), int(minlength), out.data_ptr(), Z.stream_of(x)),
            "zs_bincount")
    return out


@compileable_bincount.register_fake
def _(x: torch.Tensor, minlength: int) -> torch.Tensor:
    return torch.empty(minlength, dtype=torch.long, device=x.device)


@torch.library.custom_op("zs::flatten_sort_count", mutates_args={})
def _flatten_sort_count_op(expert_idxs: torch.Tensor, num_experts: int) -> tuple[torch.Tensor, torch.Tensor,
                                                                                  torch.Tensor]:
    Z.require_cuda(expert_idxs)
    flat = expert_idxs.reshape(-1)
    flat = flat if (flat.dtype == torch.int64 and flat.is_contiguous()) else flat.long().contiguous()
    n = flat.numel()
    sei = torch.empty(n, dtype=torch.long, device=flat.device)
    ssi = torch.empty(n, dtype=torch.long, device=flat.device)
    offs = torch.empty(num_experts, dtype=torch.long, device=flat.device)
    ws = torch.empty(max(int(Z.lib().zs_flatten_sort_count_workspace(n, int(num_experts))), 1), dtype=torch.uint8,
                     device=flat.device)
    Z.count(3)
    Z.check(Z.lib().zs_flatten_sort_count(flat.data_ptr(), n, int(num_experts), sei.data_ptr(), ssi.data_ptr(),
                                          offs.data_ptr(), ws.data_ptr(), ws.numel(), Z.stream_of(flat)),
            "zs_flatten_sort_count")
    return sei, ssi, offs


@_flatten_sort_count_op.register_fake
def _(expert_idxs, num_experts):
    n = expert_idxs.numel()
    dev = expert_idxs.device
    return (torch.empty(n, dtype=torch.long, device=dev), torch.empty(n, dtype=torch.long, device=dev),
            torch.empty(num_experts, dtype=torch.long, device=dev))


def flatten_sort_count(expert_idxs: torch.Tensor, num_experts: int):
    """(sorted_expert_idxs, sorted_scattered_idxs, expert_offsets) of the flat
    expert ids: stable order, inclusive int64 offsets."""
    with torch.no_grad():
        return _flatten_sort_count_op(expert_idxs, int(num_experts))


class ParallelLinear(torch.autograd.Function):
    """Grouped expert linear layer; same arguments and gradients as the reference."""

    @staticmethod
    def forward(ctx, x: torch.Tensor, expert_weights: torch.Tensor, k: int,
                sorted_expert_idxs: torch.Tensor, sorted_scattered_idxs: torch.Tensor,
                expert_offsets: torch.Tensor, expert_biases: Optional[torch.Tensor] = None,
                gates: Optional[torch.Tensor] = None, grouped_in: bool = False, grouped_out: bool = False):
        out = kernels.ops.scatter2scatter(X=x, W=expert_weights, b=expert_biases, k=k,
                                          sorted_expert_idxs=sorted_expert_idxs,
                                          sorted_scattered_idxs=sorted_scattered_idxs,
                                          x_grouped=grouped_in, y_grouped=grouped_out)
        per_slot = None
        if gates is not None:
            # out holds one row per (token, slot); combine the k slots of each
            # token with its gate weights.
            per_slot = out.view(gates.size(0), gates.size(1), out.size(-1))
            out = torch.bmm(gates.unsqueeze(1), per_slot).squeeze(1)
        ctx.save_for_backward(x, expert_weights, expert_biases, sorted_expert_idxs, sorted_scattered_idxs,
                              expert_offsets, gates, per_slot)
        ctx.k, ctx.grouped_in, ctx.grouped_out = k, grouped_in, grouped_out
        return out

    @staticmethod
    def backward(ctx, grad_out: torch.Tensor):
        (x, W, b, sei, ssi, offs, gates, per_slot) = ctx.saved_tensors
        k, grouped_in, grouped_out = ctx.k, ctx.grouped_in, ctx.grouped_out
        if gates is not None:
            d_gates = kernels.ops.rowwise_sum_product(per_slot, grad_out, dtype=gates.dtype)
            # gradient per (token, slot) row, scaled by that slot's gate, in expert order
            dy_rows = kernels.ops.group(grad_out, ssi, fan_out=gates.size(1), coeff=gates.flatten(),
                                        out=per_slot.flatten(0, 1))
        else:
            d_gates = None
            dy_rows = grad_out if grouped_out else kernels.ops.group(grad_out, ssi, fan_out=1)
        x_rows = x if grouped_in else kernels.ops.group(x, ssi, fan_out=k)
        d_w, d_b = kernels.ops.group_bwd_W(DY=dy_rows, X=x_rows, expert_offsets=offs, E=W.size(0),
                                           has_bias=b is not None)
        d_rows = kernels.ops.scatter2scatter(X=dy_rows, x_grouped=True, W=W.permute(0, 2, 1),
                                             sorted_expert_idxs=sei, sorted_scattered_idxs=ssi, k=1,
                                             y_grouped=grouped_in, out=None if grouped_in else x_rows)
        d_x = d_rows if k == 1 else d_rows.view(x.size(0), k, d_rows.size(-1)).sum(-2)
        return d_x, d_w, None, None, None, None, d_b, d_gates, None, None


def parallel_linear(inputs, expert_weights, k, sorted_expert_idxs, sorted_scattered_idxs, expert_offsets,
                    expert_biases=None, gates=None, grouped_in=False, grouped_out=False):
    return ParallelLinear.apply(inputs, expert_weights, k, sorted_expert_idxs, sorted_scattered_idxs,
                                expert_offsets, expert_biases, gates, grouped_in, grouped_out)


class ParallelExperts(nn.Module):
    def __init__(self, num_experts, input_size, output_size, bias=False) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.empty(num_experts, output_size, input_size))
        self.bias = nn.Parameter(torch.empty(num_experts, output_size)) if bias else None
        self.num_experts = num_experts
        self.input_size = input_size
        self.output_size = output_size
        self.reset_parameters()

    def extra_repr(self):
        return "num_experts={}, input_size={}, output_size={}".format(self.num_experts, self.input_size,
                                                                     self.output_size)

    def reset_parameters(self) -> None:
        nn.init.normal_(self.weight, std=0.02)
        if self.bias is not None:
            nn.init.zeros_(self.bias)

    def forward(self, inputs, k, sorted_expert_idxs, sorted_scattered_idxs, expert_offsets, gates=None,
                grouped_in=False, grouped_out=False):
        return parallel_linear(inputs, self.weight.permute(0, 2, 1), k, sorted_expert_idxs, sorted_scattered_idxs,
                               expert_offsets, expert_biases=self.bias, gates=gates, grouped_in=grouped_in,
                               grouped_out=grouped_out)
