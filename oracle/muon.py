"""CPU restatement of the reference's Newton-Schulz orthogonalisation — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
arm may import this module, as the checker or the timed CPU baseline.

Restates optimizer/muon.py:6-32 (quintic Newton-Schulz, coefficients
(3.4445, -4.7750, 2.0315), Frobenius pre-normalisation with +1e-7, transpose
of tall matrices), in float64, optionally rounding to bf16 where the
reference's bf16 tensors round.
"""
from __future__ import annotations

import numpy as np

from .routing import round_bf16


def newton_schulz5(G, steps=5, bf16=True):
    a, b, c = 3.4445, -4.7750, 2.0315
    r = round_bf16 if bf16 else (lambda v: np.asarray(v, dtype=np.float64))
    X = r(np.asarray(G, dtype=np.float32)).astype(np.float64)
    tall = X.shape[-2] > X.shape[-1]
    if tall:
        X = np.swapaxes(X, -1, -2)
    nrm = r(np.sqrt((X * X).sum(axis=(-2, -1), keepdims=True)).astype(np.float32)).astype(np.float64)
    X = r((X / r((nrm + 1e-7).astype(np.float32))).astype(np.float32)).astype(np.float64)
    for _ in range(steps):
        A = r((X @ np.swapaxes(X, -1, -2)).astype(np.float32)).astype(np.float64)
        B = r((b * A + c * (A @ A)).astype(np.float32)).astype(np.float64)
        X = r((a * X + B @ X).astype(np.float32)).astype(np.float64)
    if tall:
        X = np.swapaxes(X, -1, -2)
    return X
