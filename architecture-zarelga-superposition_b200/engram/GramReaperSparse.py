"""Sparse-row RMSProp for embedding tables trained on COO gradients, on the GPU.

Drop-in for the reference's GramReaperSparse (engram/GramReaperSparse.py:7-66):
the same constructor arguments and their validation, the same per-group options
(lr, beta, eps, unit_norm), the same optimizer state per table ("v": f32 [rows],
"t": step count) and the same update of every row the gradient touches:

    g_r   = sum of the gradient entries of row r           (coalesce)
    v_r   = beta * v_r + (1 - beta) * ||g_r||^2
    p_r  -= lr / (sqrt(v_r / (1 - beta^t)) + eps) * g_r
    p_r  /= max(||p_r||, eps)                              (unit_norm)

Here one libzs call per table does all of it on the device
(zs_sparse_rmsprop_step: a stable radix sort of the lookups by row, then one
CTA per distinct row), with no coalesce() and no host synchronisation.  The
step counter "t" is a 0-dim int64 device tensor advanced by the kernels, so
the step can be recorded in a CUDA graph and replayed (stage() +
step_staged(), used by optimizer.hybrid.HybridGraphOptimizer); a checkpoint
that stores "t" as a Python int loads unchanged.  Tables must be f32 CUDA
tensors; gradients of other layouts raise, as in the reference.
"""
from __future__ import annotations

import torch
from torch.optim import Optimizer

from zs_b200 import _lib as Z


def _coo_rows(grad):
    """(rows int64 [n], values [n, d]) of an uncoalesced or coalesced COO gradient."""
    idx = grad._indices()
    vals = grad._values()
    return idx[0], (vals if vals.dim() == 2 else vals.reshape(vals.size(0), -1))


def _passes(num_rows):
    return (max(int(num_rows).bit_length(), 1) + 7) // 8


class GramReaperSparse(Optimizer):
    def __init__(self, params, lr: float = 1e-2, beta: float = 0.9, eps: float = 1e-10, unit_norm: bool = False):
        if lr <= 0:
            raise ValueError(f"lr must be > 0, got {lr}")
        if not (0.0 < beta < 1.0):
            raise ValueError(f"beta must be in (0, 1), got {beta}")
        super().__init__(params, dict(lr=lr, beta=beta, eps=eps, unit_norm=unit_norm))
        self._static = {}       # size signature -> staging buffers of a recorded step
        self._static_key = None
        self._staged = []
        self._lr_dev = {}       # id(group) -> device copy of a float lr (read by recorded kernels)

    # ----------------------------------------------------------------- helpers
    @staticmethod
    def _check(p):
        if p.dim() != 2:
            raise ValueError("GramReaperSparse supports 2-D params [n_rows, dim] only")
        if not p.grad.is_sparse:
            raise ValueError("GramReaperSparse expects a sparse gradient; build the table with "
                             "nn.Embedding(..., sparse=True)")
        Z.require_cuda(p)
        if p.dtype != torch.float32 or p.stride(1) != 1:
            raise Z.ZsError("GramReaperSparse on libzs needs an f32 table with contiguous rows")

    def _state(self, p):
        st = self.state[p]
        if "v" not in st:
            st["v"] = torch.zeros(p.shape[0], dtype=p.dtype, device=p.device)
            st["t"] = torch.zeros((), dtype=torch.int64, device=p.device)
        elif not torch.is_tensor(st["t"]):  # a checkpoint that counted steps on the host
            st["t"] = torch.tensor(int(st["t"]), dtype=torch.int64, device=p.device)
        return st

    def _lr(self, group, device, refresh=True):
        """The group's lr as a device f32 the kernels read: a tensor lr itself, else a
        device copy of the float, refreshed outside any graph recording (a replayed step
        then reads the value the scheduler set for the step being replayed)."""
        lr = group["lr"]
        if torch.is_tensor(lr):
            if lr.dtype != torch.float32 or lr.device != device:
                raise Z.ZsError("a tensor lr must be an f32 tensor on the table's device")
            return lr
        dev = self._lr_dev.get(id(group))
        if dev is None or dev.device != device:
            dev = self._lr_dev[id(group)] = torch.empty((), dtype=torch.float32, device=device)
            refresh = True
        if refresh:
            dev.fill_(float(lr))
        return dev

    def _launch(self, p, group, rows, vals, ws, refresh_lr=True):
        st = self._state(p)
        lr_t = self._lr(group, p.device, refresh_lr)
        Z.count(2 + 3 * _passes(p.shape[0]))
        Z.check(Z.lib().zs_sparse_rmsprop_step(
            p.data_ptr(), p.shape[0], p.shape[1], p.stride(0), st["v"].data_ptr(), st["t"].data_ptr(),
            rows.data_ptr(), vals.data_ptr(), vals.stride(0), rows.numel(), lr_t.data_ptr(), float("nan"),
            float(group["beta"]), float(group["eps"]), int(bool(group["unit_norm"])), ws.data_ptr(), ws.numel(),
            Z.stream_of(p)), "zs_sparse_rmsprop_step")

    @staticmethod
    def _workspace(n, num_rows, device):
        return torch.empty(int(Z.lib().zs_sparse_rmsprop_workspace(n, num_rows)), dtype=torch.uint8, device=device)

    def _entries(self):
        for group in self.param_groups:
            for p in group["params"]:
                if p.grad is None:
                    continue
                self._check(p)
                rows, vals = _coo_rows(p.grad)
                if rows.numel() == 0:
                    continue
                yield group, p, rows, vals

    def state_dict(self):
        """The reference's layout: "t" as a Python int (read from the device counter)."""
        sd = super().state_dict()
        sd["state"] = {k: ({**v, "t": int(v["t"])} if torch.is_tensor(v.get("t")) else v)
                       for k, v in sd["state"].items()}
        return sd

    # ------------------------------------------------------------------ eager
    @torch.no_grad()
    def step(self, closure=None):
        loss = closure() if closure is not None else None
        for group, p, rows, vals in self._entries():
            rows = rows.contiguous()
            if vals.stride(1) != 1 or vals.data_ptr() % 16 or vals.stride(0) % 4:
                vals = vals.contiguous()
            self._launch(p, group, rows, vals, self._workspace(rows.numel(), p.shape[0], p.device))
        return loss

    # ------------------------------------------------ replayable (staged) step
    @torch.no_grad()
    def stage(self):
        """Copy this step's COO gradients into fixed buffers (one copy each for the row
        ids and the values) and return their size signature, or None when no row was
        touched.  step_staged() then runs the update from those buffers, so a CUDA graph
        recorded from it can be replayed on every later step with the same signature."""
        entries = list(self._entries())
        key = tuple((id(p), rows.numel()) for _, p, rows, _ in entries)
        if not key:
            self._static_key = None
            return None
        bufs = self._static.get(key)
        if bufs is None:
            bufs = []
            for _, p, rows, _ in entries:
                n = rows.numel()
                bufs.append((torch.empty(n, dtype=torch.int64, device=p.device),
                             torch.empty((n, p.shape[1]), dtype=torch.float32, device=p.device),
                             self._workspace(n, p.shape[0], p.device)))
            self._static[key] = bufs
        for (group, p, rows, vals), (rb, vb, _) in zip(entries, bufs):
            rb.copy_(rows, non_blocking=True)
            vb.copy_(vals, non_blocking=True)
            self._state(p)
            self._lr(group, p.device)
        self._static_key = key
        self._staged = [(group, p) for group, p, _, _ in entries]
        return key

    @torch.no_grad()
    def step_staged(self):
        for (group, p), (rb, vb, ws) in zip(self._staged, self._static[self._static_key]):
            self._launch(p, group, rb, vb, ws, refresh_lr=False)

    def release_static(self, key):
        self._static.pop(key, None)
