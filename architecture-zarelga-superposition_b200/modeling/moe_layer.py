"""MoELayer: router + shared expert + routed GLU experts (modeling/moe_layer.py:11-58).
Parameter names match the reference (gate, shared_experts, routed_experts).

The router and the shared expert's gate/up projections read the same input, so
they run as one GEMM over their concatenated weights; the input is cast to the
autocast dtype once and shared with the routed experts.  Same products as the
reference's separate autocast linears (the input gradient is accumulated in f32
inside one GEMM instead of summing bf16 gradients)."""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from scattermoe.mlp import GLUMLP

from .expert_layer import ExpertMLP
from .moe_gate import MoEGate


class MoELayer(nn.Module):
    def __init__(self, config):
        super().__init__()
        self.config = config
        self.n_experts_per_token = config.n_experts_per_token
        self.gate = MoEGate(config)
        self.shared_experts = ExpertMLP(config, intermediate_size=config.intermediate_size * config.n_shared_experts)
        self.routed_experts = GLUMLP(input_size=config.hidden_size, hidden_size=config.intermediate_size,
                                     num_experts=config.n_routed_experts, top_k=config.n_experts_per_token,
                                     activation=nn.SiLU())
        self.reset_routed_expert_parameters()

    def reset_routed_expert_parameters(self):
        std = self.config.initializer_range
        nn.init.normal_(self.routed_experts.experts.weight, mean=0.0, std=std)
        nn.init.normal_(self.routed_experts.output_experts.weight, mean=0.0, std=std)

    def forward(self, hidden_states, unpad_indices=None, out_dtype=None):
        """(out, topk_idx); out in the input's dtype, or out_dtype when given (a block whose
        norm already produced the bf16 input passes its f32 residual dtype)."""
        if unpad_indices is not None:
            bsz, seq_len, d = hidden_states.shape
            x = hidden_states.reshape(bsz * seq_len, d).index_select(0, unpad_indices).unsqueeze(0)
        else:
            x = hidden_states
        k = self.n_experts_per_token
        se = self.shared_experts
        E, f = self.gate.weight.size(0), se.gate_proj.weight.size(0)
        in_dtype = x.dtype if out_dtype is None else out_dtype
        if torch.is_autocast_enabled() and x.dtype == torch.float32:
            x = x.to(torch.get_autocast_dtype("cuda"))
        d = x.size(-1)
        w_cat = torch.cat([self.gate.weight, se.gate_proj.weight, se.up_proj.weight], 0)
        logits, g, u = torch.split(F.linear(x.reshape(-1, d), w_cat), [E, f, f], dim=-1)
        topk_idx, topk_weight = self.gate.route(logits)
        shared = se.down_proj(se.act_fn(g) * u).view(x.shape)
        routed = self.routed_experts(x, topk_weight, topk_idx)
        # the reference adds a bf16 shared output to f32 routed rows: the sum in f32
        out = shared.to(in_dtype) + routed
        topk_idx = topk_idx.view(*x.shape[:-1], k)
        if unpad_indices is not None:
            full = out.new_zeros(bsz * seq_len, out.size(-1))
            full.index_copy_(0, unpad_indices, out.squeeze(0))
            out = full.view(bsz, seq_len, -1)
            idx_full = topk_idx.new_zeros(bsz * seq_len, k)
            idx_full.index_copy_(0, unpad_indices, topk_idx.reshape(-1, k))
            topk_idx = idx_full.view(bsz, seq_len, k)
        return out, topk_idx
