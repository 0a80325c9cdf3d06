"""LigerRopeFunction on the B200 kernel.

Same autograd function and argument order as the reference
(modeling/liger_rope.py:183-206): apply(q, k, q_cos, q_sin, k_cos, k_sin)
rotates q [bsz, seq, n_q_head, head_dim] and k [bsz, seq, n_kv_head,
head_dim] in place (rotate-half pairs (i, i + head_dim/2)) with cos/sin tables
[1 or bsz, seq, head_dim/2]; the backward rotates the gradients back in place.
"""
from __future__ import annotations

import torch

from zs_b200 import _lib as Z


def _launch(q, k, q_cos, q_sin, k_cos, k_sin, backward, rot_pairs=None):
    Z.require_cuda(q, k, q_cos, q_sin, k_cos, k_sin)
    bsz, seq_len, n_qh, hd = q.shape
    n_kh = k.shape[2]
    q = q.contiguous()
    k = k.contiguous()
    tables = [t.contiguous() for t in (q_cos, q_sin, k_cos, k_sin)]
    if len({t.dtype for t in tables}) != 1:
        tables = [t.float() for t in tables]
    qc, qs, kc, ks = tables
    if qc.shape != kc.shape:
        raise ValueError(f"q_cos and k_cos must share a shape, got {tuple(qc.shape)} vs {tuple(kc.shape)}")
    rot = hd // 2 if rot_pairs is None else int(rot_pairs)
    if rot_pairs is not None and qc.shape[-1] != rot:
        raise ValueError(f"partial RoPE tables must hold {rot} pairs per row, got {qc.shape[-1]}")
    Z.count(1)
    Z.check(Z.lib().zs_rope_partial(q.data_ptr(), q.stride(1), k.data_ptr(), k.stride(1), qc.data_ptr(),
                                    qs.data_ptr(), kc.data_ptr(), ks.data_ptr(), qc.stride(-2), bsz, seq_len,
                                    qc.shape[0], n_qh, n_kh, hd, rot, Z.dtype_code(q.dtype), Z.dtype_code(qc.dtype),
                                    int(backward), Z.stream_of(q)), "zs_rope_partial")
    return q, k


def rope_forward(q, k, q_cos, q_sin, k_cos, k_sin):
    q, k = _launch(q, k, q_cos, q_sin, k_cos, k_sin, backward=False)
    return q, k, q_cos, q_sin, k_cos, k_sin


def rope_backward(dq, dk, q_cos, q_sin, k_cos, k_sin):
    return _launch(dq, dk, q_cos, q_sin, k_cos, k_sin, backward=True)


class LigerRopeFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, q_cos, q_sin, k_cos, k_sin):
        q, k, q_cos, q_sin, k_cos, k_sin = rope_forward(q, k, q_cos, q_sin, k_cos, k_sin)
        ctx.save_for_backward(q_cos, q_sin, k_cos, k_sin)
        return q, k

    @staticmethod
    def backward(ctx, dq, dk):
        q_cos, q_sin, k_cos, k_sin = ctx.saved_tensors
        dq, dk = rope_backward(dq, dk, q_cos, q_sin, k_cos, k_sin)
        return dq, dk, None, None, None, None


class PartialRopeFunction(torch.autograd.Function):
    """RoPE on the first `rot_pairs` pairs (i, i + head_dim/2) of every head only, in
    place: what LigerRopeFunction computes when the tables' remaining pairs are the
    identity (cos 1, sin 0), as GatedAttention's partial position RoPE builds them
    (modeling/attention.py:85-104), without touching the identity pairs.  Tables
    [1 or bsz, seq, rot_pairs]."""

    @staticmethod
    def forward(ctx, q, k, cos, sin, rot_pairs):
        q, k = _launch(q, k, cos, sin, cos, sin, backward=False, rot_pairs=rot_pairs)
        ctx.save_for_backward(cos, sin)
        ctx.rot = rot_pairs
        return q, k

    @staticmethod
    def backward(ctx, dq, dk):
        cos, sin = ctx.saved_tensors
        dq, dk = _launch(dq, dk, cos, sin, cos, sin, backward=True, rot_pairs=ctx.rot)
        return dq, dk, None, None, None
