"""One optimizer surface over the dense step (MuonMD + aux Adam) and the sparse
embedding step, with both replayed from CUDA graphs once warmed up.

Drop-in for the reference's HybridGraphOptimizer (optimizer/hybrid.py:33-117):
constructor (dense, sparse, capture_warmup_steps, enable_cuda_graph), the merged
param_groups (dense groups first, so param_groups[0] is the Muon group a
scheduler anchors on), state, zero_grad (dense gradients keep their buffers,
the sparse COO gradient is dropped), and the checkpoint layout of state_dict
({"dense", "sparse", "dense_steps"}).

Scheduling differs from the reference, where the sparse step has to run
eagerly (coalesce() and a host-synchronising emptiness check every step):

* dense: `capture_warmup_steps` eager steps build the optimizer state, then the
  dense step is recorded once into a CUDA graph and replayed every step (a
  recording does not run the work, so the step that records also replays).
* sparse: the sparse optimizer here (engram.GramReaperSparse) runs on device
  kernels with a device step counter.  From the first graphed step on, its COO
  gradients are staged into fixed buffers (one copy of the row ids and one of
  the values per table) and the update is replayed from a second graph keyed by
  the gradients' sizes.  A fixed batch shape has a fixed lookup count, so every
  step after the first replays; a new size is recorded once (at most
  `max_sparse_graphs` are kept).  A sparse optimizer without stage() (any
  other torch optimizer) simply steps eagerly.

Without CUDA, or with enable_cuda_graph=False, both steps run eagerly; the
numbers are the same either way.
"""
from __future__ import annotations

from collections import OrderedDict

import torch

from zs_b200 import shadow


class HybridGraphOptimizer:
    max_sparse_graphs = 4

    def __init__(self, dense, sparse, capture_warmup_steps=5, enable_cuda_graph=True):
        self.dense = dense
        self.sparse = sparse
        self.capture_warmup_steps = int(capture_warmup_steps)
        self.enable_cuda_graph = bool(enable_cuda_graph)
        self._dense_steps = 0
        self._dense_graph = None
        self._dense_gen = -1
        self._sparse_graphs = OrderedDict()

    # ---------------------------------------------------------- torch.optim surface
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
        self._dense_steps = int(state.get("dense_steps", self._dense_steps))
        # recorded graphs point at the old state tensors: record again on the next step
        self._dense_graph = None
        self._drop_sparse_graphs()

    def zero_grad(self, set_to_none=False):
        """Dense gradients keep their buffers (set_to_none=False) so the recorded step reads
        the same memory every replay; they are zeroed in one multi-tensor launch, except the
        gradients whose producer overwrites them (parameters flagged `_zs_grad_overwrite`:
        the expert weight gradients written straight from the weight-gradient GEMMs, see
        zs_b200.train.enable_fused_weight_grad), which are only marked stale.  A stale
        gradient that no backward wrote is zeroed before the step.  The sparse COO gradient
        is always dropped."""
        if set_to_none:
            self.dense.zero_grad(set_to_none=True)
        else:
            fills = []
            for g in self.dense.param_groups:
                for p in g["params"]:
                    if p.grad is None:
                        continue
                    if getattr(p, "_zs_grad_overwrite", False) and not p.grad.is_sparse:
                        p._zs_grad_stale = True
                    else:
                        if p.grad.grad_fn is not None:
                            p.grad.detach_()
                        fills.append(p.grad)
            if fills:
                torch._foreach_zero_(fills)
        self.sparse.zero_grad(set_to_none=True)

    def _zero_stale(self):
        for g in self.dense.param_groups:
            for p in g["params"]:
                if getattr(p, "_zs_grad_stale", False):
                    p.grad.zero_()
                    p._zs_grad_stale = False

    # ------------------------------------------------------------------------- step
    def _graphs_on(self):
        if not (self.enable_cuda_graph and torch.cuda.is_available()):
            return False
        for g in self.dense.param_groups:
            for p in g["params"]:
                return p.is_cuda
        return False

    @staticmethod
    def _record(fn):
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            fn()
        return graph

    def _drop_sparse_graphs(self):
        release = getattr(self.sparse, "release_static", None)
        for key in list(self._sparse_graphs):
            if release is not None:
                release(key)
        self._sparse_graphs.clear()

    @torch.no_grad()
    def step(self, closure=None):
        self._zero_stale()
        graphed = self._graphs_on() and self._dense_steps >= self.capture_warmup_steps
        if graphed:
            # a bf16 weight shadow allocated after the recording is not written by it
            if self._dense_graph is not None and self._dense_gen != shadow.GEN:
                self._dense_graph = None
            if self._dense_graph is None:
                self._dense_gen = shadow.GEN
                self._dense_graph = self._record(self.dense.step)
            self._dense_graph.replay()
        else:
            self.dense.step()
        self._dense_steps += 1
        if graphed and hasattr(self.sparse, "stage"):
            self._sparse_replay()
        else:
            self.sparse.step()

    def _sparse_replay(self):
        key = self.sparse.stage()
        if key is None:
            return
        graph = self._sparse_graphs.get(key)
        if graph is None:
            graph = self._record(self.sparse.step_staged)
            self._sparse_graphs[key] = graph
            while len(self._sparse_graphs) > self.max_sparse_graphs:
                old, _ = self._sparse_graphs.popitem(last=False)
                if hasattr(self.sparse, "release_static"):
                    self.sparse.release_static(old)
        else:
            self._sparse_graphs.move_to_end(key)
        graph.replay()
