"""CPU restatement of the reference's MoE routing — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
arm may import this module, and only as the checker or the timed CPU
baseline.  The product path (the CUDA library) never calls it.

Restates (CoffeeVampir3/Architecture-Zarelga-Superposition):
  * MoEGate.forward top-k + normalisation, modeling/moe_gate.py:26-34
  * compileable_bincount / flatten_sort_count, scattermoe/parallel_experts.py:6-28
  * auxillary_loss_free_update, main.py:161-175

Parity is pinned by tests/test_oracle_golden.py against fixtures produced by
running the reference itself (tests/golden/gen_golden.py); the exact order of
torch.topk(sorted=False) among its k outputs is CUDA behaviour and is pinned on
the GPU against torch.topk in tests/test_routing_gpu.py.
"""
from __future__ import annotations

import numpy as np


def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even), as float32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    bias = ((u >> 16) & 1) + 0x7FFF
    r = ((u + bias) & 0xFFFF0000).astype(np.uint32)
    out = r.view(np.float32).copy()
    nan = np.isnan(x)
    out[nan] = x[nan]
    return out


def round_f16(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bf16":
        return round_bf16(x)
    if dtype == "f16":
        return round_f16(x)
    return np.asarray(x, dtype=np.float32)


def ordered_key(v: np.ndarray) -> np.ndarray:
    """The total order CUDA torch.topk's radix select uses for float32."""
    v = np.ascontiguousarray(v, dtype=np.float32)
    x = v.view(np.uint32)
    key = np.where(x & 0x80000000, ~x, x | 0x80000000).astype(np.uint32)
    key[np.isnan(v)] = 0xFFFFFFFF
    return key


def gate_topk(gate_probs: np.ndarray, expert_biases: np.ndarray, k: int, dtype: str = "bf16"):
    """MoEGate.forward after sigmoid (modeling/moe_gate.py:29-34).

    gate_probs: [T, E] float32 values already representable in `dtype`.
    Returns (topk_idx int64 [T, k], topk_weight float32 [T, k] rounded to dtype).
    Selection: the k largest of probs + bias (f32); at the k-th value, ties go
    to the lowest expert index.  Order: values above the k-th value in index
    order, then the k-th-value ties in index order (CUDA gatherTopK).
    """
    probs = np.asarray(gate_probs, dtype=np.float32)
    T, E = probs.shape
    biased = (probs + np.asarray(expert_biases, dtype=np.float32)[None, :]).astype(np.float32)
    key = ordered_key(biased).astype(np.int64)
    idx = np.arange(E, dtype=np.int64)[None, :]
    comb = (key << 12) | (4095 - idx)
    order = np.argsort(-comb, axis=1, kind="stable")[:, :k]
    sel_keys = np.take_along_axis(key, order, axis=1)
    kth = sel_keys[:, k - 1 : k]
    is_tie = sel_keys == kth
    # sort selected by (tie?, index)
    comb2 = is_tie.astype(np.int64) * 4096 + order
    out_idx = np.take_along_axis(order, np.argsort(comb2, axis=1, kind="stable"), axis=1)
    w = np.take_along_axis(probs, out_idx, axis=1).astype(np.float64)
    denom = round_to(np.abs(w).sum(axis=1, keepdims=True).astype(np.float32), dtype)
    eps = round_to(np.array([1e-12], dtype=np.float32), dtype)[0]
    denom = np.maximum(denom, eps)
    weight = round_to((w.astype(np.float32) / denom).astype(np.float32), dtype)
    return out_idx.astype(np.int64), weight


def bincount(x: np.ndarray, minlength: int) -> np.ndarray:
    """compileable_bincount (scattermoe/parallel_experts.py:6-15)."""
    return np.bincount(np.asarray(x, dtype=np.int64).ravel(), minlength=minlength)[:minlength].astype(np.int64)


def flatten_sort_count(expert_idxs: np.ndarray, num_experts: int):
    """flatten_sort_count (scattermoe/parallel_experts.py:21-28), stable order."""
    flat = np.asarray(expert_idxs, dtype=np.int64).ravel()
    ssi = np.argsort(flat, kind="stable").astype(np.int64)
    sei = flat[ssi]
    offsets = np.cumsum(bincount(flat, num_experts)).astype(np.int64)
    return sei, ssi, offsets


def aux_loss_free_update(expert_biases: np.ndarray, topk_idx: np.ndarray, update_rate: float, valid=None):
    """One layer of auxillary_loss_free_update (main.py:161-175); returns the new bias."""
    topk = np.asarray(topk_idx, dtype=np.int64)
    if valid is not None:
        topk = topk[np.asarray(valid, dtype=bool)]
    bias = np.asarray(expert_biases, dtype=np.float32).copy()
    if topk.size == 0:
        return bias
    E = bias.shape[0]
    counts = bincount(topk.ravel(), E).astype(np.float32)
    mean = np.float32(counts.sum(dtype=np.float32) * np.float32(np.float32(1.0) / np.float32(E)))
    errors = (mean - counts).astype(np.float32)
    return (bias + np.float32(update_rate) * np.sign(errors).astype(np.float32)).astype(np.float32)
