"""MCCE v2 entry point on the B200 kernels.

Same public function as the reference (modeling/mcce_fast_v2.py:384-408),
same semantics as modeling.mcce_fast.mcce_raw_token_mean.  The reference's
fused Triton forward / split dH-dE backward are replaced by libzs.so's
classifier GEMM with an online log-sum-exp epilogue (forward) and per-slice
logit-gradient recomputation feeding two tensor-core GEMMs (backward).
"""
from __future__ import annotations

import torch

from . import mcce_fast
from zs_b200.xent import DEFAULT_V_CHUNK, fused_linear_cross_entropy


def mcce_raw_token_mean_v2(hidden: torch.Tensor, embeddings: torch.Tensor, labels: torch.Tensor, s: torch.Tensor, *,
                           use_triton: bool = True, v_chunk_size: int = 8192, debug: bool = False,
                           check_label_values: bool = False) -> torch.Tensor:
    if debug:
        mcce_fast._validate_inputs(hidden, embeddings, labels, s, check_label_values=check_label_values)
    return fused_linear_cross_entropy(hidden, embeddings, labels, s, DEFAULT_V_CHUNK)
