"""Drop-in scattermoe package backed by the B200 kernels of libzs.so.

Same public names as the reference package (scattermoe/__init__.py):
flatten_sort_count, parallel_linear, ParallelExperts and the parallel_experts,
kernels and mlp modules.  The reference's `utils` (HF model monkey-patching,
scattermoe/utils/replace_moe.py) is not part of the training step and is not
provided.
"""
from .parallel_experts import flatten_sort_count, parallel_linear, ParallelExperts
from . import parallel_experts
from . import kernels
from . import mlp

__all__ = ["flatten_sort_count", "parallel_linear", "ParallelExperts", "parallel_experts", "kernels", "mlp"]
