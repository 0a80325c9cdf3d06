"""CPU restatement of the reference's scattermoe expert layer — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
arm may import this module, and only as the checker or the timed CPU
baseline.  The product path (the CUDA library) never calls it.

Restates (CoffeeVampir3/Architecture-Zarelga-Superposition):
  * scatter2scatter          scattermoe/kernels/ops.py:128-190 (+ wrapper :192-209)
  * groupXtY / group_bwd_W   scattermoe/kernels/ops.py:263-271, :320-438
  * group                    scattermoe/kernels/ops.py:449-458, :490-529
  * rowwise_sum_product      scattermoe/kernels/ops.py:9-18, :50-80
  * ParallelLinear fwd/bwd   scattermoe/parallel_experts.py:32-135
  * GLUMLP.forward           scattermoe/mlp.py:74-95 (up half first, gate half second)

Math is float64 on float32 inputs; callers round to the storage dtype where the
reference does (helpers from oracle.routing).
"""
from __future__ import annotations

import numpy as np

from .routing import flatten_sort_count, round_to


def scatter2scatter(X, W, sorted_expert_idxs, sorted_scattered_idxs, k, b=None, x_grouped=False, y_grouped=False):
    """out[out_row(i)] = X[in_row(i)] @ W[e_i] (+ b[e_i]); W is [E, K, N]."""
    X = np.asarray(X, dtype=np.float64)
    W = np.asarray(W, dtype=np.float64)
    sei = np.asarray(sorted_expert_idxs, dtype=np.int64)
    ssi = np.asarray(sorted_scattered_idxs, dtype=np.int64)
    n = sei.shape[0]
    N = W.shape[2]
    out = np.zeros((n, N), dtype=np.float64)
    rows_in = np.arange(n) if x_grouped else ssi // k
    rows_out = np.arange(n) if y_grouped else ssi
    for e in np.unique(sei):
        m = sei == e
        y = X[rows_in[m]] @ W[e]
        if b is not None:
            y = y + np.asarray(b, dtype=np.float64)[e][None, :]
        out[rows_out[m]] = y
    return out


def group_xty(DY, X, expert_offsets, E):
    """DW[e] = X[s:t]^T @ DY[s:t] over each expert's grouped rows; [E, K, N]."""
    DY = np.asarray(DY, dtype=np.float64)
    X = np.asarray(X, dtype=np.float64)
    offs = np.asarray(expert_offsets, dtype=np.int64)
    DW = np.zeros((E, X.shape[1], DY.shape[1]), dtype=np.float64)
    start = 0
    for e in range(E):
        end = int(offs[e])
        if end > start:
            DW[e] = X[start:end].T @ DY[start:end]
        start = end
    return DW


def group_bias(DY, expert_offsets, E):
    DY = np.asarray(DY, dtype=np.float64)
    offs = np.asarray(expert_offsets, dtype=np.int64)
    Db = np.zeros((E, DY.shape[1]), dtype=np.float64)
    start = 0
    for e in range(E):
        end = int(offs[e])
        Db[e] = DY[start:end].sum(axis=0)
        start = end
    return Db


def group(A, sorted_scattered_idxs, fan_out=1, coeff=None):
    """Y[i] = A[ssi[i] // fan_out] (* coeff[ssi[i]])."""
    A = np.asarray(A, dtype=np.float64)
    ssi = np.asarray(sorted_scattered_idxs, dtype=np.int64)
    Y = A[ssi // fan_out]
    if coeff is not None:
        Y = Y * np.asarray(coeff, dtype=np.float64).ravel()[ssi][:, None]
    return Y


def rowwise_sum_product(A, B):
    """out[t, f] = sum_h A[t, f, h] * B[t, h]."""
    return np.einsum("tfh,th->tf", np.asarray(A, dtype=np.float64), np.asarray(B, dtype=np.float64))


def _silu(x):
    return x / (1.0 + np.exp(-x))


def glu_mlp_forward(x, expert_p, expert_idxs, W1, W2, dtype="f32"):
    """GLUMLP.forward (scattermoe/mlp.py:74-95).

    W1 = experts.weight [E, 2f, d] (rows [0, f) "up", [f, 2f) "gate");
    W2 = output_experts.weight [E, d, f].  Intermediate tensors are rounded to
    `dtype` where the reference stores them.  Returns (y, saved) with saved
    tensors for glu_mlp_backward.
    """
    x = np.asarray(x, dtype=np.float64)
    E = W1.shape[0]
    k = expert_idxs.shape[1]
    f = W1.shape[1] // 2
    sei, ssi, offs = flatten_sort_count(expert_idxs, E)
    hfull = round_to(scatter2scatter(x, np.transpose(W1, (0, 2, 1)), sei, ssi, k, y_grouped=True).astype(np.float32), dtype)
    h, g = hfull[:, :f].astype(np.float64), hfull[:, f:].astype(np.float64)
    act = round_to((round_to(_silu(g).astype(np.float32), dtype).astype(np.float64) * h).astype(np.float32), dtype)
    y2 = round_to(scatter2scatter(act, np.transpose(W2, (0, 2, 1)), sei, ssi, 1, x_grouped=True).astype(np.float32), dtype)
    T = x.shape[0]
    p = np.asarray(expert_p, dtype=np.float64)
    y = np.einsum("tj,tjd->td", p, y2.astype(np.float64).reshape(T, k, -1))
    saved = dict(sei=sei, ssi=ssi, offs=offs, hfull=hfull, act=act, y2=y2, k=k, f=f)
    return y, saved


def glu_mlp_backward(dy, x, expert_p, W1, W2, saved, dtype="f32"):
    """Gradients of glu_mlp_forward following ParallelLinear.backward
    (scattermoe/parallel_experts.py:70-135) and autograd through silu(g) * h.
    Returns (dx, d_expert_p, dW1 [E, 2f, d], dW2 [E, d, f])."""
    dy = np.asarray(dy, dtype=np.float64)
    x = np.asarray(x, dtype=np.float64)
    E = W1.shape[0]
    k, f = saved["k"], saved["f"]
    sei, ssi, offs = saved["sei"], saved["ssi"], saved["offs"]
    T = x.shape[0]
    p = np.asarray(expert_p, dtype=np.float64)
    y2 = saved["y2"].astype(np.float64).reshape(T, k, -1)
    d_p = np.einsum("tjd,td->tj", y2, dy)
    dy_g = group(dy, ssi, fan_out=k, coeff=p)          # [n, d]
    act = saved["act"].astype(np.float64)
    dW2t = group_xty(dy_g, act, offs, E)                # [E, f, d]
    dact = scatter2scatter(dy_g, W2, sei, ssi, 1, x_grouped=True, y_grouped=True)  # [n, f]
    hfull = saved["hfull"].astype(np.float64)
    h, g = hfull[:, :f], hfull[:, f:]
    sg = 1.0 / (1.0 + np.exp(-g))
    dh = dact * _silu(g)
    dg = dact * h * sg * (1.0 + g * (1.0 - sg))
    dhfull = np.concatenate([dh, dg], axis=1)
    xg = group(x, ssi, fan_out=k)
    dW1t = group_xty(dhfull, xg, offs, E)               # [E, d, 2f]
    dxg = scatter2scatter(dhfull, W1, sei, ssi, 1, x_grouped=True, y_grouped=False)  # [n, d] at flat rows
    dx = dxg.reshape(T, k, -1).sum(axis=1)
    return dx, d_p, np.transpose(dW1t, (0, 2, 1)), np.transpose(dW2t, (0, 2, 1))
