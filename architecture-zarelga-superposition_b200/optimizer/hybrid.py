"""HybridGraphOptimizer (optimizer/hybrid.py:33-117): a dense optimizer whose
step() is captured once into a CUDA graph after `capture_warmup_steps` eager
steps and replayed afterwards, plus an eager sparse optimizer, behind one
torch.optim-like surface (param_groups, state, zero_grad, step, state_dict)."""
from __future__ import annotations

import torch


class HybridGraphOptimizer:
    def __init__(self, dense, sparse, capture_warmup_steps=5, enable_cuda_graph=True):
        self.dense = dense
        self.sparse = sparse
        self.capture_warmup_steps = capture_warmup_steps
        self.enable_cuda_graph = enable_cuda_graph
        self._graph = None
        self._dense_steps = 0

    @property
    def param_groups(self):
        return self.dense.param_groups + self.sparse.param_groups

    @property
    def state(self):
        merged = dict(self.dense.state)
        merged.update(self.sparse.state)
        return merged

    def state_dict(self):
        return {"dense": self.dense.state_dict(), "sparse": self.sparse.state_dict(),
                "dense_steps": self._dense_steps}

    def load_state_dict(self, state):
        self.dense.load_state_dict(state["dense"])
        self.sparse.load_state_dict(state["sparse"])
        self._dense_steps = state.get("dense_steps", self._dense_steps)

    def zero_grad(self, set_to_none=False):
        # dense grads keep their addresses for the captured graph; the sparse
        # COO grad is a new tensor every backward
        self.dense.zero_grad(set_to_none=set_to_none)
        self.sparse.zero_grad(set_to_none=True)

    @torch.no_grad()
    def step(self, closure=None):
        if not self.enable_cuda_graph or not torch.cuda.is_available():
            self.dense.step()
        elif self._graph is not None:
            self._graph.replay()
        elif self._dense_steps >= self.capture_warmup_steps:
            torch.cuda.synchronize()
            self._graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self._graph):
                self.dense.step()
            self._graph.replay()
        else:
            self.dense.step()
        self._dense_steps += 1
        self.sparse.step()
