"""MCCE (multi-target cut cross entropy, raw-token mean) on the B200 kernels.

Same public names and signatures as the reference module
(modeling/mcce_fast.py): MCCEKernelConfig, naive_mcce_raw_token_mean
(:117-139), mcce_raw_token_mean (:642-677).  The loss

    N     = sum_i s[i]
    lse_i = logsumexp_v(hidden[i] @ embeddings[v])
    loss  = (sum_i s[i] * lse_i - sum_i sum_{j < s[i]} z[i, labels[i, j]]) / N

runs in libzs.so's fused classifier GEMM (zs_xent_forward / zs_xent_backward):
the [T, V] logits are never stored; the backward recomputes them one
vocabulary slice at a time.  There is no CPU path.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

from zs_b200.xent import DEFAULT_V_CHUNK, fused_linear_cross_entropy


@dataclass(frozen=True)
class MCCEKernelConfig:
    """Accepted for signature compatibility; the B200 kernels pick their own tiles."""

    block_t: int = 16
    block_v: int = 128
    block_d: int = 32
    reduce_block_v: int = 256
    num_warps_lse: int = 4
    num_warps_target: int = 4
    num_warps_finalize: int = 4
    num_warps_backward: int = 8


def _validate_inputs(hidden, embeddings, labels, s, *, check_label_values: bool) -> None:
    if hidden.ndim != 2:
        raise ValueError(f"hidden must be [T, D], got {tuple(hidden.shape)}")
    if embeddings.ndim != 2:
        raise ValueError(f"embeddings must be [V, D], got {tuple(embeddings.shape)}")
    if hidden.shape[1] != embeddings.shape[1]:
        raise ValueError(f"hidden D and embeddings D differ: {hidden.shape[1]} vs {embeddings.shape[1]}")
    if labels.ndim != 2 or labels.shape[0] != hidden.shape[0]:
        raise ValueError(f"labels must be [T, S_MAX], got {tuple(labels.shape)}")
    if s.shape != (hidden.shape[0],):
        raise ValueError(f"s must be [T], got {tuple(s.shape)}")
    if labels.dtype not in (torch.int32, torch.int64):
        raise TypeError(f"labels must be int32 or int64, got {labels.dtype}")
    if s.dtype not in (torch.int16, torch.int32, torch.int64, torch.uint8):
        raise TypeError(f"s must be an integer tensor, got {s.dtype}")
    if not torch.all(s > 0):
        raise ValueError("all sequence granularities s[i] must be positive")
    if not torch.all(s <= labels.shape[1]):
        raise ValueError("all s[i] must be <= S_MAX")
    if labels.shape[1] > 8:
        raise ValueError("S_MAX above 8 is not supported by the B200 kernels")
    if check_label_values:
        cols = torch.arange(labels.shape[1], device=labels.device)[None, :]
        active = labels[cols < s[:, None]]
        V = embeddings.shape[0]
        if active.numel() and not torch.all((active >= 0) & (active < V)):
            raise ValueError("active labels must all be in [0, V)")


def naive_mcce_raw_token_mean(hidden, embeddings, labels, s):
    """Materialising reference formulation (tests only): full [T, V] logits."""
    T, D = hidden.shape
    S_MAX = labels.shape[1]
    logits = hidden.float() @ embeddings.float().T
    lse = torch.logsumexp(logits, dim=-1)
    cols = torch.arange(S_MAX, device=labels.device)[None, :]
    active = cols < s[:, None]
    safe = torch.where(active, labels, torch.zeros_like(labels))
    target_sum = (logits.gather(1, safe) * active.float()).sum(dim=-1)
    s_f = s.float()
    return (s_f.mul(lse).sum() - target_sum.sum()) / s_f.sum()


def mcce_raw_token_mean(hidden, embeddings, labels, s, *, use_triton: bool = True,
                        config: Optional[MCCEKernelConfig] = None, v_chunk_size: int = 8192, debug: bool = False,
                        check_label_values: bool = False):
    """Exact MCCE loss, raw-token mean.  Active labels are labels[i, :s[i]];
    later slots are never read.  `use_triton`, `config` and `v_chunk_size` are
    accepted for compatibility and do not change the computation."""
    if debug:
        _validate_inputs(hidden, embeddings, labels, s, check_label_values=check_label_values)
    return fused_linear_cross_entropy(hidden, embeddings, labels, s, DEFAULT_V_CHUNK)
