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


def sink_grad(ds_sink, q, ldq, B, S, H, hd, scale):
    """dk_sink [H, hd] f32 = scale * sum_{b,s} ds_sink[b, h, s] * q[b, s, h, :], q bf16 rows of ldq
    elements from q's first element (zs_attention_sink_grad: q read once, fixed-order sums)."""
    dk = torch.empty(H, hd, dtype=torch.float32, device=q.device)
    L = Z.lib()
    ws = torch.empty(int(L.zs_attention_sink_grad_workspace(B, S, H, hd)), dtype=torch.uint8, device=q.device)
    Z.count(2)
    Z.check(L.zs_attention_sink_grad(ds_sink.data_ptr(), q.data_ptr(), ldq, B, S, H, hd, float(scale), dk.data_ptr(),
                                     ws.data_ptr(), ws.numel(), Z.stream_of(q)), "zs_attention_sink_grad")
    return dk


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
            dk_sink = sink_grad(ds_sink, q, H * hd, B, S, H, hd, ctx.scale).to(k_sink.dtype)
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


class _GatedAttentionCore(torch.autograd.Function):
    """GatedAttention between its two projections, on the fused q/k/v/gate projection
    output qkvg [B, S, W] (bf16; columns: H query heads, Hkv key heads, Hkv value heads,
    H gate logits, zero padding): the per-head q/k zero-centred RMSNorm + partial RoPE
    (zs_qk_norm_rope_forward, one kernel writing the normalised q and k), attention with
    the sigmoid output gate applied in its epilogue, reading v and the gate logits in
    place (zs_gated_attention_forward).  The backward writes the whole gradient of qkvg
    -- dq/dk through the norm/RoPE transpose, dv and the gate logits' gradient from the
    attention kernels, zeros in the padding -- with no split, cat or copy."""

    @staticmethod
    def forward(ctx, qkvg, wq, wk, k_sink, cos, sin, H, Hkv, hd, rot, eps, window, seg_start, scale, pad):
        B, S, W = qkvg.shape
        dev = qkvg.device
        qk = torch.empty(B, S, (H + Hkv) * hd, dtype=torch.bfloat16, device=dev)
        rstd = torch.empty(B * S * (H + Hkv), dtype=torch.float32, device=dev)
        L = Z.lib()
        tab_dt = Z.dtype_code(cos.dtype) if cos is not None else Z.ZS_F32
        cos_bs = cos.shape[0] if cos is not None else 1
        cos_ld = cos.stride(-2) if cos is not None else 0
        Z.count(1)
        Z.check(L.zs_qk_norm_rope_forward(qkvg.data_ptr(), W, wq.data_ptr(), wk.data_ptr(), Z.ptr(cos), Z.ptr(sin),
                                          tab_dt, cos_ld, cos_bs, rot, qk.data_ptr(), (H + Hkv) * hd,
                                          rstd.data_ptr(), B * S, S, H, Hkv, hd, float(eps), Z.stream_of(qkvg)),
                "zs_qk_norm_rope_forward")
        o = torch.empty(B, S, H * hd, dtype=torch.bfloat16, device=dev)
        lse = torch.empty(B, H, S, dtype=torch.float32, device=dev)
        ld_qk = (H + Hkv) * hd
        v_ptr = qkvg.data_ptr() + 2 * (H + Hkv) * hd
        g_ptr = qkvg.data_ptr() + 2 * (H + 2 * Hkv) * hd
        with Z.timed("attention_fwd", attention_flops(B, S, H, hd, window)):
            Z.check(L.zs_gated_attention_forward(qk.data_ptr(), ld_qk, qk.data_ptr() + 2 * H * hd, ld_qk, v_ptr, W,
                                                 o.data_ptr(), H * hd, lse.data_ptr(), g_ptr, W, B, S, H, Hkv, hd,
                                                 window, Z.ptr(seg_start), Z.ptr(k_sink),
                                                 Z.dtype_code(k_sink.dtype) if k_sink is not None else 0, scale,
                                                 Z.stream_of(qkvg)), "zs_gated_attention_forward")
        Z.count(1)
        ctx.save_for_backward(qkvg, qk, o, lse, rstd, wq, wk, k_sink, cos, sin, seg_start)
        ctx.meta = (H, Hkv, hd, rot, window, scale, pad)
        return o

    @staticmethod
    def backward(ctx, do):
        qkvg, qk, o, lse, rstd, wq, wk, k_sink, cos, sin, seg_start = ctx.saved_tensors
        H, Hkv, hd, rot, window, scale, pad = ctx.meta
        B, S, W = qkvg.shape
        dev = qkvg.device
        do = do.contiguous()
        if do.dtype != torch.bfloat16:
            do = do.to(torch.bfloat16)
        L = Z.lib()
        dqkvg = torch.empty_like(qkvg)
        dqk = torch.empty_like(qk)
        D = torch.empty(B, H, S, dtype=torch.float32, device=dev)
        ds_sink = torch.empty(B, H, S, dtype=torch.float32, device=dev) if k_sink is not None else None
        ws = torch.empty(int(L.zs_gated_attention_backward_workspace(B, S, H, hd, 1)), dtype=torch.uint8, device=dev)
        ld_qk = (H + Hkv) * hd
        base = qkvg.data_ptr()
        dbase = dqkvg.data_ptr()
        with Z.timed("attention_bwd", 2.5 * attention_flops(B, S, H, hd, window)):
            Z.check(L.zs_gated_attention_backward(
                qk.data_ptr(), ld_qk, qk.data_ptr() + 2 * H * hd, ld_qk, base + 2 * (H + Hkv) * hd, W,
                o.data_ptr(), H * hd, do.data_ptr(), H * hd, lse.data_ptr(), base + 2 * (H + 2 * Hkv) * hd, W,
                dqk.data_ptr(), ld_qk, dqk.data_ptr() + 2 * H * hd, ld_qk, dbase + 2 * (H + Hkv) * hd, W,
                dbase + 2 * (H + 2 * Hkv) * hd, W, pad, D.data_ptr(), B, S, H, Hkv, hd, window, Z.ptr(seg_start),
                Z.ptr(k_sink), Z.dtype_code(k_sink.dtype) if k_sink is not None else 0, Z.ptr(ds_sink), scale,
                ws.data_ptr(), ws.numel(), Z.stream_of(qkvg)), "zs_gated_attention_backward")
        Z.count(3)
        dwq = torch.empty(hd, dtype=torch.float32, device=dev)
        dwk = torch.empty(hd, dtype=torch.float32, device=dev)
        ws2 = torch.empty(int(L.zs_qk_norm_rope_backward_workspace(hd)), dtype=torch.uint8, device=dev)
        tab_dt = Z.dtype_code(cos.dtype) if cos is not None else Z.ZS_F32
        cos_bs = cos.shape[0] if cos is not None else 1
        cos_ld = cos.stride(-2) if cos is not None else 0
        Z.count(2)
        Z.check(L.zs_qk_norm_rope_backward(dqk.data_ptr(), ld_qk, base, W, wq.data_ptr(), wk.data_ptr(), Z.ptr(cos),
                                           Z.ptr(sin), tab_dt, cos_ld, cos_bs, rot, rstd.data_ptr(), dbase, W,
                                           dwq.data_ptr(), dwk.data_ptr(), B * S, S, H, Hkv, hd, ws2.data_ptr(),
                                           ws2.numel(), Z.stream_of(qkvg)),
                "zs_qk_norm_rope_backward")
        dk_sink = None
        if k_sink is not None and ctx.needs_input_grad[3]:
            dk_sink = sink_grad(ds_sink, qk, ld_qk, B, S, H, hd, scale).to(k_sink.dtype)
        return (dqkvg, dwq.to(wq.dtype), dwk.to(wk.dtype), dk_sink) + (None,) * 11


def gated_attention_core(qkvg, wq, wk, *, n_heads, n_kv_heads, head_dim, cos=None, sin=None, rot_pairs=0,
                         eps=1e-6, window=None, seq_ids=None, k_sink=None, scale=None, pad=0):
    """o [B, S, H * hd] (bf16) = sigmoid(gate) * attention(rope(norm(q)), rope(norm(k)), v) from the
    fused projection output qkvg [B, S, (H + 2 Hkv) * hd + H + pad] (bf16, contiguous); cos/sin
    [1 or B, S, rot_pairs] RoPE tables (None when rot_pairs is 0)."""
    Z.require_cuda(qkvg, wq, wk, k_sink, seq_ids, cos, sin)
    H, Hkv, hd = int(n_heads), int(n_kv_heads), int(head_dim)
    if qkvg.dtype != torch.bfloat16 or not qkvg.is_contiguous():
        raise Z.ZsError("the fused projection output must be a contiguous bf16 tensor")
    if hd not in (64, 128) or H % Hkv:
        raise Z.ZsError(f"attention supports head_dim 64/128 and H % Hkv == 0 (got hd={hd}, H={H}, Hkv={Hkv})")
    W = qkvg.shape[-1]
    if W != (H + 2 * Hkv) * hd + H + pad or W % 8 or not 0 <= pad < 32:
        raise Z.ZsError(f"qkvg width {W} does not match H={H}, Hkv={Hkv}, hd={hd}, pad={pad} (rows must be "
                        "multiples of 8 elements)")
    if wq.dtype != torch.float32 or wk.dtype != torch.float32:
        raise Z.ZsError("the q/k norm weights must be f32")
    scale = 1.0 / math.sqrt(hd) if scale is None else float(scale)
    seg_start = seg_start_from_seq_ids(seq_ids) if seq_ids is not None else None
    if rot_pairs:
        cos, sin = cos.contiguous(), sin.contiguous()
    else:
        cos = sin = None
    return _GatedAttentionCore.apply(qkvg, wq.contiguous(), wk.contiguous(), k_sink, cos, sin, H, Hkv, hd,
                                     int(rot_pairs), float(eps), int(window) if window else 0, seg_start, scale,
                                     int(pad))

