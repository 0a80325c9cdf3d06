"""Pre-norm residual block: norm -> attention -> add -> norm -> MoE -> add
(modeling/transformer_block.py:6-46).  Under bf16 autocast with an f32 residual
stream, the residual add and the following norm run as one kernel that also
emits the bf16 input of the next GEMM (AddZRMSNormFunction): same values as the
reference's add, f32 norm and autocast cast, fewer passes over the stream."""
from __future__ import annotations

import torch
import torch.nn as nn

from .moe_layer import MoELayer
from .zRMSNorm import AddZRMSNormFunction, ZeroCenteredRMSNorm, fused_add_norm_ok


class TransformerBlock(nn.Module):
    # the fused residual-add + norm path under autocast (off: the reference's op sequence)
    fused_add_norm = True

    def __init__(self, config, layer_type, input_layernorm=True):
        super().__init__()
        self.input_layernorm = (ZeroCenteredRMSNorm(config.hidden_size, eps=config.rms_norm_eps)
                                if input_layernorm else nn.Identity())
        self.self_attn = layer_type(config)
        self.post_attention_layernorm = ZeroCenteredRMSNorm(config.hidden_size, eps=config.rms_norm_eps)
        self.mlp = MoELayer(config)

    def forward(self, hidden_states, position_ids=None, cu_seqlens=None, max_seqlen=None, unpad_indices=None):
        if self._fused_path(hidden_states):
            return self._forward_fused(hidden_states, position_ids, cu_seqlens, max_seqlen, unpad_indices)
        h = hidden_states + self.self_attn(self.input_layernorm(hidden_states), position_ids=position_ids,
                                           cu_seqlens=cu_seqlens, max_seqlen=max_seqlen, unpad_indices=unpad_indices)
        moe_out, topk_idx = self.mlp(self.post_attention_layernorm(h), unpad_indices=unpad_indices)
        return h + moe_out, topk_idx

    def _fused_path(self, x):
        """Under bf16 autocast with an f32 residual stream the norms feed bf16 GEMMs only:
        the residual add and the norm run as one kernel with a bf16 output."""
        return (self.fused_add_norm and torch.is_autocast_enabled()
                and torch.get_autocast_dtype("cuda") == torch.bfloat16
                and isinstance(self.input_layernorm, ZeroCenteredRMSNorm) and fused_add_norm_ok(x))

    def _forward_fused(self, x, position_ids, cu_seqlens, max_seqlen, unpad_indices):
        n1, n2 = self.input_layernorm, self.post_attention_layernorm
        y1 = AddZRMSNormFunction.apply(x, None, n1.weight, n1.eps)
        attn = self.self_attn(y1, position_ids=position_ids, cu_seqlens=cu_seqlens, max_seqlen=max_seqlen,
                              unpad_indices=unpad_indices)
        if attn.dtype != torch.bfloat16:
            attn = attn.to(torch.bfloat16)
        h, y2 = AddZRMSNormFunction.apply(x, attn, n2.weight, n2.eps)
        return self.mlp(y2, unpad_indices=unpad_indices, out_dtype=torch.float32, residual=h)
