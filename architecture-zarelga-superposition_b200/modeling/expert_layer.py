"""ExpertMLP (the shared expert): down(silu(gate(x)) * up(x)) with bias-free
linears named gate_proj / up_proj / down_proj (modeling/expert_layer.py:6-24).
The forward runs on the grouped tcgen05 GEMM as a one-group expert: the up and
gate products in one launch with the SwiGLU in its epilogue, the down product in
a second; the backward fuses the SwiGLU derivative into the down product's
input-gradient epilogue (zs_b200.dense.dense_swiglu)."""
from __future__ import annotations

import torch.nn as nn

from zs_b200.dense import dense_swiglu


class ExpertMLP(nn.Module):
    def __init__(self, config, intermediate_size=None):
        super().__init__()
        self.config = config
        self.hidden_size = config.hidden_size
        self.intermediate_size = intermediate_size or config.intermediate_size
        self.initializer_range = config.initializer_range
        self.gate_proj = nn.Linear(self.hidden_size, self.intermediate_size, bias=False)
        self.up_proj = nn.Linear(self.hidden_size, self.intermediate_size, bias=False)
        self.down_proj = nn.Linear(self.intermediate_size, self.hidden_size, bias=False)
        self.act_fn = nn.SiLU()
        self.reset_parameters()

    def reset_parameters(self):
        for lin in (self.gate_proj, self.up_proj, self.down_proj):
            nn.init.normal_(lin.weight, mean=0.0, std=self.initializer_range)

    def forward(self, x):
        # one-group grouped GEMMs with the SwiGLU fused into their epilogues (zs_b200.dense)
        return dense_swiglu(x, self.gate_proj.weight, self.up_proj.weight, self.down_proj.weight)
