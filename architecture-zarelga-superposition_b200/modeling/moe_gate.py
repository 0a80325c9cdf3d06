"""MoEGate on the B200 routing kernel.

Same constructor, parameter (`weight` [E, d]), buffer (`expert_biases` [E])
and forward contract as the reference (modeling/moe_gate.py:5-35): sigmoid
router scores, top-k of score + bias, weights = L1-normalised unbiased scores.
The router GEMM and sigmoid stay torch ops (cuBLAS; 2*T*d*E flops); the biased
top-k, the gather and the normalisation run in one warp-per-token kernel whose
indices match CUDA torch.topk(sorted=False) exactly.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from zs_b200 import _lib as Z


def gate_topk(gate_probs: torch.Tensor, expert_biases: torch.Tensor, top_k: int):
    """(topk_idx int64 [T, k], topk_weight [T, k] in gate_probs' dtype)."""
    Z.require_cuda(gate_probs, expert_biases)
    probs = gate_probs.contiguous()
    T, E = probs.shape
    bias = expert_biases.float().contiguous()
    idx = torch.empty((T, top_k), dtype=torch.long, device=probs.device)
    w = torch.empty((T, top_k), dtype=probs.dtype, device=probs.device)
    Z.count(1)
    Z.check(Z.lib().zs_moe_gate_topk(probs.data_ptr(), Z.dtype_code(probs.dtype), bias.data_ptr(), T, E, int(top_k),
                                     idx.data_ptr(), w.data_ptr(), Z.stream_of(probs)), "zs_moe_gate_topk")
    return idx, w


class GateTopK(torch.autograd.Function):
    """Biased top-k + normalised weights with the gradient of the weights
    flowing back to the unbiased scores (the reference's gather + F.normalize
    are differentiable; the indices are not)."""

    @staticmethod
    def forward(ctx, gate_probs, expert_biases, top_k):
        idx, w = gate_topk(gate_probs, expert_biases, top_k)
        ctx.save_for_backward(gate_probs.contiguous(), idx)
        ctx.mark_non_differentiable(idx)
        return idx, w

    @staticmethod
    def backward(ctx, _grad_idx, grad_w):
        probs, idx = ctx.saved_tensors
        if grad_w is None:
            return None, None, None
        T, E = probs.shape
        k = idx.size(1)
        g = grad_w.to(probs.dtype).contiguous()
        grad = torch.empty_like(probs)
        Z.count(1)
        Z.check(Z.lib().zs_moe_gate_topk_backward(probs.data_ptr(), Z.dtype_code(probs.dtype), idx.data_ptr(),
                                                  g.data_ptr(), Z.dtype_code(g.dtype), T, E, k, grad.data_ptr(),
                                                  Z.stream_of(probs)), "zs_moe_gate_topk_backward")
        return grad, None, None


class MoEGate(nn.Module):
    def __init__(self, config):
        super().__init__()
        self.config = config
        self.top_k = config.n_experts_per_token
        self.n_routed_experts = config.n_routed_experts
        self.gating_dim = config.hidden_size
        self.weight = nn.Parameter(torch.empty((self.n_routed_experts, self.gating_dim)))
        self.register_buffer("expert_biases", torch.zeros(self.n_routed_experts))
        self.reset_parameters()

    def reset_parameters(self):
        nn.init.normal_(self.weight, mean=0.0, std=self.config.initializer_range)

    def forward(self, hidden_states):
        bsz, seq_len, h = hidden_states.shape
        idx, w = self.route(F.linear(hidden_states.view(-1, h), self.weight, None))
        return idx.view(bsz, seq_len, -1), w.view(bsz, seq_len, -1)

    def route(self, logits):
        """(topk_idx [T, k], topk_weight [T, k]) from router logits [T, E] = x W^T."""
        return GateTopK.apply(torch.sigmoid(logits), self.expert_biases, self.top_k)
