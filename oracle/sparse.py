"""CPU restatement of the reference's sparse input embedding and its optimizer — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
arm may import this module, as the checker or the timed CPU baseline.

Restates (CoffeeVampir3/Architecture-Zarelga-Superposition):
  * MoEModel._embed_tokens, modeling/model.py:71-86: nn.Embedding lookup, the
    f32 bag mean over the last id axis of 3-D ids, x sqrt(d) when untied; its
    gradient as nn.Embedding(sparse=True) returns it (one COO entry per lookup);
  * GramReaperSparse.step, engram/GramReaperSparse.py:18-66: coalesce, per-row
    RMSProp with bias correction, optional unit-L2 projection of touched rows.

Pinned by tests/test_sparse_oracle.py against fixtures made by running the
reference's GramReaperSparse (tests/golden/gen_golden.py, gen_sparse).
"""
from __future__ import annotations

import numpy as np


def embedding_bag(table, ids, scale):
    """f32 [*, d]: scale * mean over the bag axis (3-D ids) of table rows."""
    table = np.asarray(table, np.float32)
    ids = np.asarray(ids)
    rows = table[ids]                                   # [..., (s,) d]
    if ids.ndim == 3:
        rows = (rows.astype(np.float32).sum(axis=-2) * np.float32(1.0 / ids.shape[-1])).astype(np.float32)
    return (rows * np.float32(scale)).astype(np.float32)


def embedding_bag_coo(dy, ids, scale):
    """(rows [n], values [n, d]) of the table gradient, one entry per lookup in lookup order."""
    dy = np.asarray(dy, np.float32)
    ids = np.asarray(ids)
    g = (dy * np.float32(scale)).astype(np.float32)
    if ids.ndim == 3:
        s = ids.shape[-1]
        g = (g / np.float32(s)).astype(np.float32)
        g = np.repeat(g[..., None, :], s, axis=-2)
    return ids.reshape(-1).astype(np.int64), g.reshape(-1, dy.shape[-1])


def sparse_rmsprop_step(p, v, t, rows, values, lr, beta, eps, unit_norm):
    """One GramReaperSparse step on table p (in place, f32) with COO gradient (rows, values).
    Returns the new step count t (unchanged when no row is touched)."""
    rows = np.asarray(rows, np.int64)
    values = np.asarray(values, np.float32)
    if rows.size == 0:
        return t
    uniq, inv = np.unique(rows, return_inverse=True)    # coalesce: one entry per distinct row
    g = np.zeros((uniq.size, values.shape[1]), np.float64)
    np.add.at(g, inv, values.astype(np.float64))
    g = g.astype(np.float32)
    t = t + 1
    f = np.float32
    v[uniq] = f(beta) * v[uniq] + f(1.0 - beta) * (g.astype(np.float64) ** 2).sum(axis=1).astype(np.float32)
    v_hat = v[uniq] / f(1.0 - beta ** t)
    step = f(lr) / (np.sqrt(v_hat) + f(eps))
    row = p[uniq] - step[:, None] * g
    if unit_norm:
        n = np.sqrt((row.astype(np.float64) ** 2).sum(axis=1)).astype(np.float32)
        row = row / np.maximum(n, f(eps))[:, None]
    p[uniq] = row.astype(np.float32)
    return t
