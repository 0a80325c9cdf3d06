"""Attention core used by GatedAttention: causal GQA softmax attention over
packed or batched sequences with an optional causal sliding window and an
optional learned per-head sink logit (a key with zero value that every query
sees).

q [B, S, H, hd], k/v [B, S, Hkv, hd]; returns [B, S, H, hd] in q's dtype.
Sequences: either each batch row is one sequence (cu_seqlens is None) or the
rows are packed and seq_ids [B, S] (-1 for padding) tells which sequence a
token belongs to.

The computation runs in PyTorch's fused scaled-dot-product attention; the
sink is folded in as one extra key/value column.  This module is the single
place the model reaches attention through.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def _mask(S, device, window, seq_ids=None, sink=False):
    i = torch.arange(S, device=device)
    allowed = i[None, :] <= i[:, None]
    if window is not None:
        allowed &= i[:, None] - i[None, :] < window
    allowed = allowed[None]
    if seq_ids is not None:
        allowed = allowed & (seq_ids[:, :, None] == seq_ids[:, None, :]) & (seq_ids[:, :, None] >= 0)
    if sink:
        allowed = torch.cat([allowed, torch.ones_like(allowed[..., :1])], dim=-1)
    return allowed[:, None]  # [B or 1, 1, S, S(+1)]


def attention(q, k, v, *, window=None, seq_ids=None, k_sink=None, scale=None):
    from . import _lib as Z

    with Z.timed("attention_fwd"):
        return _attention(q, k, v, window=window, seq_ids=seq_ids, k_sink=k_sink, scale=scale)


def _attention(q, k, v, *, window=None, seq_ids=None, k_sink=None, scale=None):
    B, S, H, hd = q.shape
    Hkv = k.shape[2]
    scale = 1.0 / math.sqrt(hd) if scale is None else scale
    qt, kt, vt = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    if k_sink is not None:
        # one always-visible key per head with a zero value row
        ks = k_sink.to(q.dtype).view(1, H, 1, hd).expand(B, H, 1, hd)
        if Hkv != H:
            kt = kt.repeat_interleave(H // Hkv, dim=1)
            vt = vt.repeat_interleave(H // Hkv, dim=1)
        kt = torch.cat([kt, ks], dim=2)
        vt = torch.cat([vt, torch.zeros_like(ks)], dim=2)
        out = F.scaled_dot_product_attention(qt, kt, vt, attn_mask=_mask(S, q.device, window, seq_ids, sink=True),
                                             scale=scale)
    elif window is None and seq_ids is None:
        out = F.scaled_dot_product_attention(qt, kt, vt, is_causal=True, scale=scale, enable_gqa=Hkv != H)
    else:
        out = F.scaled_dot_product_attention(qt, kt, vt, attn_mask=_mask(S, q.device, window, seq_ids), scale=scale,
                                             enable_gqa=Hkv != H)
    return out.transpose(1, 2)
