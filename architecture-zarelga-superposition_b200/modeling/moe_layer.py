"""MoELayer: router + shared expert + routed GLU experts (modeling/moe_layer.py:11-58).
Parameter names match the reference (gate, shared_experts, routed_experts).

The input is cast to the autocast dtype once and shared by the router (a
T x E cuBLAS product, 2*T*d*E flops), the shared expert (one-group grouped
GEMMs with the SwiGLU fused, modeling/expert_layer.py) and the routed experts."""
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

    # the block's residual add, the shared expert's output and the routed combine as one
    # kernel (scattermoe.mlp.GLUExpertsFunction with shared / residual); off: torch adds
    fused_close = True

    def forward(self, hidden_states, unpad_indices=None, out_dtype=None, residual=None):
        """(out, topk_idx); out in the input's dtype, or out_dtype when given (a block whose
        norm already produced the bf16 input passes its f32 residual dtype).  With residual
        (f32, the stream the block adds the layer's output to) out = residual + layer output."""
        if unpad_indices is not None:
            bsz, seq_len, d = hidden_states.shape
            x = hidden_states.reshape(bsz * seq_len, d).index_select(0, unpad_indices).unsqueeze(0)
        else:
            x = hidden_states
        k = self.n_experts_per_token
        se = self.shared_experts
        in_dtype = x.dtype if out_dtype is None else out_dtype
        if torch.is_autocast_enabled() and x.dtype == torch.float32:
            x = x.to(torch.get_autocast_dtype("cuda"))
        d = x.size(-1)
        logits = F.linear(x.reshape(-1, d), self.gate.weight)   # the router: T x E, tiny
        topk_idx, topk_weight = self.gate.route(logits)
        shared = se(x)
        if (residual is not None and unpad_indices is None and self.fused_close and residual.dtype == torch.float32
                and x.dtype in (torch.bfloat16, torch.float16) and type(self.routed_experts) is GLUMLP
                and self.routed_experts._fused_ok()
                and self.routed_experts.top_k <= 8 and x.size(-1) % 8 == 0):
            out = self.routed_experts(x, topk_weight, topk_idx, shared=shared, residual=residual)
            return out.view(residual.shape), topk_idx.view(*x.shape[:-1], k)
        routed = self.routed_experts(x, topk_weight, topk_idx)
        # the reference adds a bf16 shared output to f32 routed rows: the sum in f32
        out = shared.to(in_dtype) + routed
        topk_idx = topk_idx.view(*x.shape[:-1], k)
        if residual is not None and unpad_indices is None:
            out = residual + out
        if unpad_indices is not None:
            full = out.new_zeros(bsz * seq_len, out.size(-1))
            full.index_copy_(0, unpad_indices, out.squeeze(0))
            out = full.view(bsz, seq_len, -1)
            idx_full = topk_idx.new_zeros(bsz * seq_len, k)
            idx_full.index_copy_(0, unpad_indices, topk_idx.reshape(-1, k))
            topk_idx = idx_full.view(bsz, seq_len, k)
            if residual is not None:
                out = residual + out
        return out, topk_idx
