"""GatedAttention (https://arxiv.org/abs/2505.06708) with the reference's
interface (modeling/attention.py:14-226): q/k/v/o and head-gate projections,
per-head QK zero-centred RMSNorm, partial position-RoPE on the first
pos_rope_dims of each head, causal GQA attention with an optional sliding
window, and a per-head sigmoid output gate.  An optional learned sink logit
per head (the key-sink of modeling/hca.py:138-144, value 0) is off by default
so the state dict matches the reference's.

Everything runs in libzs.so: the q/k/v/head-gate projections as one grouped-GEMM
product over the concatenated weights; then, on the fused path, one kernel for the
QK-norm + RoPE of q and k and the tcgen05 flash attention reading v and the gate
logits in place from the projection output, with the sigmoid gate applied in its
epilogue (backward: the attention kernels and the norm/RoPE transpose write the
projection output's gradient directly); and the output projection.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from zs_b200.attn import attention as attention_core
from zs_b200.attn import gated_attention_core
from zs_b200.dense import dense_linear

from .liger_rope import LigerRopeFunction, PartialRopeFunction  # noqa: F401
from .zRMSNorm import ZeroCenteredRMSNorm


def _seq_ids_from_cu_seqlens(cu_seqlens, unpad_indices, bsz, seq_len):
    """Sequence id per (batch, position) for a packed batch; -1 on padding."""
    total = int(cu_seqlens[-1])
    ids = torch.repeat_interleave(torch.arange(cu_seqlens.numel() - 1, device=cu_seqlens.device),
                                  cu_seqlens[1:] - cu_seqlens[:-1], output_size=total)
    full = torch.full((bsz * seq_len,), -1, dtype=torch.long, device=cu_seqlens.device)
    full[unpad_indices] = ids
    return full.view(bsz, seq_len)


class GatedAttention(nn.Module):
    def __init__(self, config, window_size: Optional[int] = None, use_sink: Optional[bool] = None):
        super().__init__()
        self.hidden_size = config.hidden_size
        self.num_heads = config.n_attention_heads
        self.num_key_value_heads = config.n_key_value_heads
        self.num_key_value_groups = self.num_heads // self.num_key_value_heads
        self.head_dim = config.hidden_size // config.n_attention_heads
        self.max_position_embeddings = config.max_position_embeddings
        self.rope_theta = config.rope_theta
        self.do_rope = config.do_rope
        self.initializer_range = config.initializer_range
        self.window_size = window_size
        self.window = (window_size - 1, 0) if window_size is not None else (-1, -1)
        if self.head_dim * self.num_heads != self.hidden_size:
            raise ValueError("hidden_size must be divisible by num_attention_heads")
        self.q_proj = nn.Linear(self.hidden_size, self.num_heads * self.head_dim, bias=False)
        self.k_proj = nn.Linear(self.hidden_size, self.num_key_value_heads * self.head_dim, bias=False)
        self.v_proj = nn.Linear(self.hidden_size, self.num_key_value_heads * self.head_dim, bias=False)
        self.o_proj = nn.Linear(self.num_heads * self.head_dim, self.hidden_size, bias=False)
        self.head_gate_proj = nn.Linear(self.hidden_size, self.num_heads, bias=False)
        self.use_qk_norm = config.use_qk_norm
        if self.use_qk_norm:
            self.q_norm = ZeroCenteredRMSNorm(self.head_dim, eps=config.rms_norm_eps)
            self.k_norm = ZeroCenteredRMSNorm(self.head_dim, eps=config.rms_norm_eps)
        else:
            self.q_norm = nn.Identity()
            self.k_norm = nn.Identity()
        if use_sink is None:
            use_sink = getattr(config, "attention_sink", False)
        self.k_sink = nn.Parameter(torch.empty(self.num_heads, self.head_dim)) if use_sink else None
        self.reset_parameters()
        self.pos_rope_dims = config.pos_rope_dims
        self.pos_rope_pairs = config.pos_rope_dims // 2
        if self.do_rope:
            pos_cos, pos_sin = self._build_pos_rope_tables(self.max_position_embeddings, self.head_dim,
                                                           self.rope_theta, dtype=torch.float32,
                                                           device=self.q_proj.weight.device)
        else:
            pos_cos = pos_sin = None
        self.register_buffer("pos_cos_cache", pos_cos, persistent=False)
        self.register_buffer("pos_sin_cache", pos_sin, persistent=False)

    def reset_parameters(self):
        for lin in (self.q_proj, self.k_proj, self.v_proj, self.o_proj, self.head_gate_proj):
            nn.init.normal_(lin.weight, mean=0.0, std=self.initializer_range)
        if self.k_sink is not None:
            nn.init.normal_(self.k_sink, mean=0.0, std=self.initializer_range)

    def _build_pos_rope_tables(self, max_position_embeddings, head_dim, base, dtype, device):
        """cos/sin [max_pos, head_dim/2]: rotation on the first pos_rope_dims/2 pairs, identity after."""
        half = head_dim // 2
        cos_table = torch.ones(max_position_embeddings, half, dtype=dtype, device=device)
        sin_table = torch.zeros(max_position_embeddings, half, dtype=dtype, device=device)
        if self.pos_rope_pairs == 0:
            return cos_table, sin_table
        inv_freq = 1.0 / (base ** (torch.arange(0, self.pos_rope_dims, 2, device=device, dtype=torch.float32)
                                   / self.pos_rope_dims))
        freqs = torch.outer(torch.arange(max_position_embeddings, device=device, dtype=torch.float32), inv_freq)
        cos_table[:, : self.pos_rope_pairs] = freqs.cos().to(dtype)
        sin_table[:, : self.pos_rope_pairs] = freqs.sin().to(dtype)
        return cos_table, sin_table

    # q/k norm + RoPE + attention + output gate as one autograd function over the fused
    # projection output (zs_b200.attn.gated_attention_core); off: the step-by-step path
    fused_core = True

    def _fused_core_ok(self, qkvg):
        return (self.fused_core and qkvg.dtype == torch.bfloat16 and qkvg.is_contiguous() and self.use_qk_norm
                and isinstance(self.q_norm, ZeroCenteredRMSNorm) and isinstance(self.k_norm, ZeroCenteredRMSNorm)
                and self.q_norm.weight.dtype == torch.float32 and self.k_norm.weight.dtype == torch.float32
                and self.q_norm.eps == self.k_norm.eps and self.head_dim in (64, 128)
                and qkvg.shape[-1] % 8 == 0)

    def forward(self, hidden_states, position_ids=None, cu_seqlens=None, max_seqlen=None, unpad_indices=None):
        bsz, seq_len, _ = hidden_states.shape
        # q, k, v and the head gate read the same input: one GEMM over the
        # concatenated weights (the input is cast once, and its gradient is one
        # f32-accumulated product instead of a sum of four).  Zero rows pad the
        # output width to a multiple of 16 so every output row starts on a
        # 32-byte boundary (an odd width sends cuBLAS to unaligned kernels).
        qd, kd = self.num_heads * self.head_dim, self.num_key_value_heads * self.head_dim
        n_out = qd + 2 * kd + self.num_heads
        pad = -n_out % 16
        ws = [self.q_proj.weight, self.k_proj.weight, self.v_proj.weight, self.head_gate_proj.weight]
        qkvg = dense_linear(hidden_states, ws, tag="proj_qkvg", pad=pad)
        seq_ids = None
        if cu_seqlens is not None:
            seq_ids = _seq_ids_from_cu_seqlens(cu_seqlens, unpad_indices, bsz, seq_len)
        if self._fused_core_ok(qkvg):
            # q/k norm + RoPE, attention and the output gate straight from the projection output
            rp = self.pos_rope_pairs if self.do_rope else 0
            cos = sin = None
            if rp:
                if position_ids is None:
                    cos = self.pos_cos_cache[:seq_len, :rp].unsqueeze(0)
                    sin = self.pos_sin_cache[:seq_len, :rp].unsqueeze(0)
                else:
                    cos = self.pos_cos_cache[:, :rp][position_ids]
                    sin = self.pos_sin_cache[:, :rp][position_ids]
            attn = gated_attention_core(qkvg, self.q_norm.weight, self.k_norm.weight, n_heads=self.num_heads,
                                        n_kv_heads=self.num_key_value_heads, head_dim=self.head_dim, cos=cos, sin=sin,
                                        rot_pairs=rp, eps=self.q_norm.eps, window=self.window_size, seq_ids=seq_ids,
                                        k_sink=self.k_sink, pad=pad)
            return dense_linear(attn, [self.o_proj.weight], tag="proj_o")
        if self.do_rope and position_ids is None:
            position_ids = torch.arange(seq_len, device=hidden_states.device).expand(bsz, seq_len)
        q, k, v, gate_logits = torch.split(qkvg, [qd, kd, kd, self.num_heads + pad], dim=-1)
        gate_logits = gate_logits[..., : self.num_heads]
        q = q.reshape(bsz, seq_len, self.num_heads, self.head_dim)
        k = k.reshape(bsz, seq_len, self.num_key_value_heads, self.head_dim)
        v = v.reshape(bsz, seq_len, self.num_key_value_heads, self.head_dim)
        q = self.q_norm(q)
        k = self.k_norm(k)
        if self.do_rope and self.pos_rope_pairs > 0:
            # only the first pos_rope_pairs pairs rotate (the tables are the identity
            # beyond them), so only those columns of the tables are gathered and touched
            rp = self.pos_rope_pairs
            cos = self.pos_cos_cache[:, :rp][position_ids]
            sin = self.pos_sin_cache[:, :rp][position_ids]
            q, k = PartialRopeFunction.apply(q, k, cos, sin, rp)
        attn = attention_core(q, k, v, window=self.window_size, seq_ids=seq_ids, k_sink=self.k_sink)
        gate = torch.sigmoid(gate_logits)
        attn = attn * gate.unsqueeze(-1)
        return dense_linear(attn.reshape(bsz, seq_len, self.num_heads * self.head_dim), [self.o_proj.weight],
                            tag="proj_o")
