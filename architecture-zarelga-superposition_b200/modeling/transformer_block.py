"""Pre-norm residual block: norm -> attention -> add -> norm -> MoE -> add
(modeling/transformer_block.py:6-46)."""
from __future__ import annotations

import torch.nn as nn

from .moe_layer import MoELayer
from .zRMSNorm import ZeroCenteredRMSNorm


class TransformerBlock(nn.Module):
    def __init__(self, config, layer_type, input_layernorm=True):
        super().__init__()
        self.input_layernorm = (ZeroCenteredRMSNorm(config.hidden_size, eps=config.rms_norm_eps)
                                if input_layernorm else nn.Identity())
        self.self_attn = layer_type(config)
        self.post_attention_layernorm = ZeroCenteredRMSNorm(config.hidden_size, eps=config.rms_norm_eps)
        self.mlp = MoELayer(config)

    def forward(self, hidden_states, position_ids=None, cu_seqlens=None, max_seqlen=None, unpad_indices=None):
        h = hidden_states + self.self_attn(self.input_layernorm(hidden_states), position_ids=position_ids,
                                           cu_seqlens=cu_seqlens, max_seqlen=max_seqlen, unpad_indices=unpad_indices)
        moe_out, topk_idx = self.mlp(self.post_attention_layernorm(h), unpad_indices=unpad_indices)
        return h + moe_out, topk_idx
