"""CPU restatement of the reference's attention-side ops — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
arm may import this module, as the checker or the timed CPU baseline.

Restates (CoffeeVampir3/Architecture-Zarelga-Superposition):
  * ZeroCenteredRMSNorm            modeling/zRMSNorm.py:10-17
  * position-RoPE tables           modeling/attention.py:85-104
  * rotate-half RoPE fwd / bwd     modeling/liger_rope.py:98-119
  * attention core                 modeling/attention.py:117-169 (flash_attn_varlen_func,
                                   causal, window (W-1, 0) from :31) restated as exact
                                   per-sequence causal softmax attention; the sink key
                                   of modeling/hca.py:138-144,264-298 (k_sink[h], value 0,
                                   always visible).  flash-attn itself (pyproject.toml:16)
                                   ships no test for this, so this restatement is pinned
                                   to PyTorch's scaled_dot_product_attention on the CPU
                                   with hca.py's sink concatenation (tests/test_attn_oracle.py).
"""
from __future__ import annotations

import numpy as np


def zrmsnorm(x, w, eps):
    """(y, rstd) in float64 from float32-valued inputs."""
    x = np.asarray(x, dtype=np.float64)
    r = 1.0 / np.sqrt((x * x).mean(axis=-1, keepdims=True) + eps)
    return x * r * (1.0 + np.asarray(w, dtype=np.float64)), r[..., 0]


def zrmsnorm_backward(dy, x, w, eps):
    x = np.asarray(x, dtype=np.float64)
    dy = np.asarray(dy, dtype=np.float64)
    d = x.shape[-1]
    r = 1.0 / np.sqrt((x * x).mean(axis=-1, keepdims=True) + eps)
    n = x * r
    dn = dy * (1.0 + np.asarray(w, dtype=np.float64))
    dx = r * (dn - n * (dn * n).mean(axis=-1, keepdims=True))
    dw = (dy * n).reshape(-1, d).sum(axis=0)
    return dx, dw


def rope_tables(max_pos, head_dim, base, pos_rope_dims):
    """cos/sin tables [max_pos, head_dim/2]: rotation on the first pos_rope_dims/2 pairs, identity after."""
    half = head_dim // 2
    cos = np.ones((max_pos, half), dtype=np.float32)
    sin = np.zeros((max_pos, half), dtype=np.float32)
    pairs = pos_rope_dims // 2
    if pairs == 0:
        return cos, sin
    inv_freq = (1.0 / (np.float32(base) ** (np.arange(0, pos_rope_dims, 2, dtype=np.float32) / np.float32(pos_rope_dims)))).astype(np.float32)
    t = np.arange(max_pos, dtype=np.float32)
    freqs = np.outer(t, inv_freq).astype(np.float32)
    cos[:, :pairs] = np.cos(freqs)
    sin[:, :pairs] = np.sin(freqs)
    return cos, sin


def rope(x, cos, sin, backward=False):
    """x [b, s, h, hd]; cos/sin [b or 1, s, hd/2]."""
    x = np.asarray(x, dtype=np.float64)
    hd = x.shape[-1]
    c = np.asarray(cos, dtype=np.float64)[:, :, None, :]
    s = np.asarray(sin, dtype=np.float64)[:, :, None, :]
    if backward:
        s = -s
    x1, x2 = x[..., : hd // 2], x[..., hd // 2:]
    return np.concatenate([x1 * c - x2 * s, x2 * c + x1 * s], axis=-1)


def attention_visibility(S, window=0, seg_start=None):
    """bool [B or 1, S(q), S(k)]: k <= q, q - k < window (window > 0), same packed sequence.

    seg_start [B, S] int: first row position of each token's sequence, -1 on padding.
    """
    i = np.arange(S)
    vis = i[None, :] <= i[:, None]
    if window and window > 0:
        vis &= (i[:, None] - i[None, :]) < window
    vis = vis[None]
    if seg_start is not None:
        seg = np.asarray(seg_start)
        vis = vis & (seg[:, :, None] >= 0) & (i[None, None, :] >= seg[:, :, None])
    return vis


def attention_forward(q, k, v, *, window=0, seg_start=None, k_sink=None, scale=None):
    """(o [B,S,H,hd], lse [B,H,S]) in float64.  q [B,S,H,hd], k/v [B,S,Hkv,hd], k_sink [H,hd] or None.

    softmax over the visible keys (plus the sink logit scale*q.k_sink with a zero value row);
    lse is the natural log of the denominator; a row that sees nothing gives o = 0, lse = -inf.
    """
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    B, S, H, hd = q.shape
    G = H // k.shape[2]
    scale = 1.0 / np.sqrt(hd) if scale is None else scale
    vis = attention_visibility(S, window, seg_start)
    vis = np.broadcast_to(vis, (B, S, S))
    o = np.zeros_like(q)
    lse = np.full((B, H, S), -np.inf)
    for b in range(B):
        for h in range(H):
            s = scale * q[b, :, h] @ k[b, :, h // G].T
            s = np.where(vis[b], s, -np.inf)
            vv = v[b, :, h // G]
            if k_sink is not None:
                ks = np.asarray(k_sink, dtype=np.float64)[h]
                s = np.concatenate([s, scale * (q[b, :, h] @ ks)[:, None]], axis=1)
                vv = np.concatenate([vv, np.zeros((1, hd))], axis=0)
            m = s.max(axis=1, keepdims=True)
            live = np.isfinite(m[:, 0])
            msafe = np.where(np.isfinite(m), m, 0.0)
            p = np.exp(s - msafe)
            l = p.sum(axis=1, keepdims=True)
            o[b, :, h] = np.where(live[:, None], (p @ vv) / np.where(l > 0, l, 1.0), 0.0)
            lse[b, h] = np.where(live, msafe[:, 0] + np.log(np.where(l[:, 0] > 0, l[:, 0], 1.0)), -np.inf)
    return o, lse


def attention_backward(do, q, k, v, *, window=0, seg_start=None, k_sink=None, scale=None):
    """(dq, dk, dv, dk_sink or None) in float64 for the loss sum(do * o) of attention_forward."""
    do = np.asarray(do, dtype=np.float64)
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    B, S, H, hd = q.shape
    G = H // k.shape[2]
    scale = 1.0 / np.sqrt(hd) if scale is None else scale
    o, lse = attention_forward(q, k, v, window=window, seg_start=seg_start, k_sink=k_sink, scale=scale)
    vis = np.broadcast_to(attention_visibility(S, window, seg_start), (B, S, S))
    dq, dk, dv = np.zeros_like(q), np.zeros_like(k), np.zeros_like(v)
    dks = np.zeros((H, hd)) if k_sink is not None else None
    for b in range(B):
        for h in range(H):
            kk, vv = k[b, :, h // G], v[b, :, h // G]
            L = lse[b, h][:, None]
            Lsafe = np.where(np.isfinite(L), L, 0.0)
            s = scale * q[b, :, h] @ kk.T
            p = np.where(vis[b], np.exp(s - Lsafe), 0.0)
            dP = do[b, :, h] @ vv.T
            D = (do[b, :, h] * o[b, :, h]).sum(axis=1, keepdims=True)
            dS = p * (dP - D)
            dq[b, :, h] = scale * dS @ kk
            dk[b, :, h // G] += scale * dS.T @ q[b, :, h]
            dv[b, :, h // G] += p.T @ do[b, :, h]
            if k_sink is not None:
                ks = np.asarray(k_sink, dtype=np.float64)[h]
                ps = np.where(np.isfinite(L[:, 0]), np.exp(scale * (q[b, :, h] @ ks) - Lsafe[:, 0]), 0.0)
                dss = -ps * D[:, 0]
                dq[b, :, h] += scale * dss[:, None] * ks[None, :]
                dks[h] += scale * dss @ q[b, :, h]
    return dq, dk, dv, dks
