"""CPU restatement of the reference's (multi-target) cut cross entropy — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
arm may import this module, as the checker or the timed CPU baseline.

Restates modeling/mcce_fast.py:21-31 (objective and logit gradient) and
:117-139 (naive formulation); the standard CE of the third-party
linear_cross_entropy (main.py:761) is the s_max = 1 case with ignored rows
dropped (its upstream source, apple/ml-cross-entropy, is not in the
reference tree and is restated from the call's documented meaning: mean
cross entropy over targets != ignore_index).
"""
from __future__ import annotations

import numpy as np


def mcce(hidden, embeddings, labels, s, v_chunk=4096):
    """(loss, dH, dE) in float64.  labels [T, S_MAX] (slots >= s[i] ignored), s [T] >= 0."""
    H = np.asarray(hidden, dtype=np.float64)
    E = np.asarray(embeddings, dtype=np.float64)
    labels = np.asarray(labels, dtype=np.int64)
    s = np.asarray(s, dtype=np.int64)
    T, D = H.shape
    V = E.shape[0]
    S_MAX = labels.shape[1]
    active = np.arange(S_MAX)[None, :] < s[:, None]
    # online log-sum-exp over vocabulary chunks
    m = np.full(T, -np.inf)
    acc = np.zeros(T)
    for v0 in range(0, V, v_chunk):
        z = H @ E[v0:v0 + v_chunk].T
        nm = np.maximum(m, z.max(axis=1))
        acc = acc * np.exp(m - nm) + np.exp(z - nm[:, None]).sum(axis=1)
        m = nm
    lse = m + np.log(acc)
    safe = np.where(active, labels, 0)
    tz = np.einsum("td,tjd->tj", H, E[safe])
    target = (tz * active).sum(axis=1)
    N = s.sum()
    loss = (s * lse - target).sum() / N
    dH = np.zeros_like(H)
    dE = np.zeros_like(E)
    for v0 in range(0, V, v_chunk):
        z = H @ E[v0:v0 + v_chunk].T
        g = (s[:, None] / N) * np.exp(z - lse[:, None])
        dH += g @ E[v0:v0 + v_chunk]
        dE[v0:v0 + v_chunk] += g.T @ H
    for j in range(S_MAX):
        a = active[:, j]
        dH[a] -= E[labels[a, j]] / N
        np.add.at(dE, labels[a, j], -H[a] / N)
    return loss, dH, dE


def cross_entropy(e, c, targets, ignore_index=-100):
    """Mean next-token CE of e @ c^T over targets != ignore_index: (loss, de, dc)."""
    t = np.asarray(targets, dtype=np.int64).reshape(-1)
    active = t != ignore_index
    labels = np.where(active, t, 0)[:, None]
    return mcce(np.asarray(e).reshape(len(t), -1), c, labels, active.astype(np.int64))
