"""CPU restatement of the reference's attention-side ops — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
arm may import this module, as the checker or the timed CPU baseline.

Restates (CoffeeVampir3/Architecture-Zarelga-Superposition):
  * ZeroCenteredRMSNorm            modeling/zRMSNorm.py:10-17
  * position-RoPE tables           modeling/attention.py:85-104
  * rotate-half RoPE fwd / bwd     modeling/liger_rope.py:98-119
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
