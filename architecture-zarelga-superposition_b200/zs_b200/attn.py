"""Attention core used by GatedAttention: causal GQA softmax attention over
packed or batched sequences with an optional causal sliding window and an
optional learned per-head sink key (a key with zero value that every query
sees), on the tcgen05 flash-attention kernels of libzs.so.

Replaces the reference's flash_attn_varlen_func call
(modeling/attention.py:117-169; window (W-1, 0) at :31) and the sink of
modeling/hca.py:138-144,264-298.

q [B, S, H, hd], k/v [B, S, Hkv, hd] bf16, hd 64 or 128; returns [B, S, H, hd].
Sequences: either each batch row is one sequence (seq_ids is None) or the rows
hold packed sequences and seq_ids [B, S] (-1 for padding) names each token's
sequence.  A sequence's tokens are contiguous and in order inside one batch
row, which is how unpad/cu_seqlens batches are laid out (right- or
left-padded rows, documents packed back to back); causal order and the window
then follow row positions exactly as flash_attn's varlen positions.
"""
from __future__ import annotations

import math

import torch

from . import _lib as Z


def attention_flops(B, S, H, hd, window=0):
    """Algorithmic tensor FLOPs of the causal forward (S = QK^T and O = PV over the
    visible key positions of every query: i+1, or min(i+1, window))."""
    if window and window < S:
        visible = window * (window + 1) // 2 + (S - window) * window
    else:
        visible = S * (S + 1) // 2
    return 4.0 * B * H * hd * visible


def seg_start_from_seq_ids(seq_ids: torch.Tensor) -> torch.Tensor:
    """int32 [B, S]: first row position of each token's sequence, -1 on padding (no host sync)."""
    B, S = seq_ids.shape
    pos = torch.arange(S, device=seq_ids.device).expand(B, S)
    prev = torch.cat([torch.full_like(seq_ids[:, :1], -2), seq_ids[:, :-1]], dim=1)
    starts = torch.where(seq_ids != prev, pos, torch.zeros_like(pos))
    seg = torch.cummax(starts, dim=1).values
    return torch.where(seq_ids >= 0, seg, torch.full_like(seg, -1)).to(torch.int32).contiguous()


class _Attention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, k_sink, window, seg_start, scale):
        B, S, H, hd = q.shape
        Hkv = k.shape[2]
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
        o = torch.empty_like(q)
        lse = torch.empty(B, H, S, dtype=torch.float32, device=q.device)
        L = Z.lib()
        with Z.timed("attention_fwd", attention_flops(B, S, H, hd, window)):
            Z.check(L.zs_attention_forward(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(),
                                           B, S, H, Hkv, hd, window, Z.ptr(seg_start), Z.ptr(k_sink),
                                           Z.dtype_code(k_sink.dtype) if k_sink is not None else 0, scale,
                                           Z.stream_of(q)), "zs_attention_forward")
        Z.count(1)
        ctx.save_for_backward(q, k, v, o, lse, seg_start, k_sink)
        ctx.window, ctx.scale = window, scale
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse, seg_start, k_sink = ctx.saved_tensors
        B, S, H, hd = q.shape
        Hkv = k.shape[2]
        do = do.contiguous()
        if do.dtype != q.dtype:
            do = do.to(q.dtype)
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        D = torch.empty(B, H, S, dtype=torch.float32, device=q.device)
        ds_sink = torch.empty(B, H, S, dtype=torch.float32, device=q.device) if k_sink is not None else None
        L = Z.lib()
        with Z.timed("attention_bwd", 2.5 * attention_flops(B, S, H, hd, ctx.window)):
            Z.check(L.zs_attention_backward(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), do.data_ptr(),
                                            lse.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(),
                                            D.data_ptr(), B, S, H, Hkv, hd, ctx.window, Z.ptr(seg_start),
                                            Z.ptr(k_sink), Z.dtype_code(k_sink.dtype) if k_sink is not None else 0,
                                            Z.ptr(ds_sink), ctx.scale, Z.stream_of(q)), "zs_attention_backward")
        Z.count(3)
        dk_sink = None
        if k_sink is not None and ctx.needs_input_grad[3]:
            dk_sink = (torch.einsum("bhs,bshd->hd", ds_sink, q.float()) * ctx.scale).to(k_sink.dtype)
        return dq, dk, dv, dk_sink, None, None, None


def attention(q, k, v, *, window=None, seq_ids=None, k_sink=None, scale=None):
    Z.require_cuda(q, k, v, k_sink, seq_ids)
    B, S, H, hd = q.shape
    Hkv = k.shape[2]
    if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16 or v.dtype != torch.bfloat16:
        raise Z.ZsError(f"attention runs in bf16 (got {q.dtype}, {k.dtype}, {v.dtype})")
    if hd not in (64, 128) or H % Hkv:
        raise Z.ZsError(f"attention supports head_dim 64/128 and H % Hkv == 0 (got hd={hd}, H={H}, Hkv={Hkv})")
    scale = 1.0 / math.sqrt(hd) if scale is None else float(scale)
    seg_start = seg_start_from_seq_ids(seq_ids) if seq_ids is not None else None
    return _Attention.apply(q, k, v, k_sink, int(window) if window else 0, seg_start, scale)
