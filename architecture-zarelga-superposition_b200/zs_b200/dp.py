"""Data-parallel plumbing for the training step: one process per GPU, gradients
summed (or averaged) over ranks with bucketed all-reduces that start while the
backward pass is still running.

GradAllReducer registers a post-accumulate-grad hook on every parameter; when
the parameters of a bucket (about bucket_mb of gradients, filled in the order
the backward produces them) all have their gradient, one all-reduce of the
flattened bucket is issued asynchronously on a side stream, overlapping the
rest of the backward.  Code that writes .grad itself (the fused expert
weight-gradient path) reports completion through notify_grad_ready.  finish()
flushes what is left, waits for the collectives and copies the reduced values
back (a bucket dtype group holding one contiguous gradient is reduced in place).  Sparse gradients (the input embedding's COO gradient) are
all-gathered as (indices, values) and concatenated, which is the sum of the
ranks' sparse gradients.

Buckets start in reverse registration order; after the first finish() they are
rebuilt in the order the gradients actually arrived (rank 0's order, broadcast,
so every rank agrees), with parameters that never fire a hook at the end.
Every rank must register the same parameters in the same order and run one
backward pass per finish(): the collectives are issued in bucket order,
identical on every rank.

engine="ce" reduces the dense buckets (after the first step's rebuild) with
CopyEngineAllReduce (zs_b200/ce.py): peer copies on the copy engines instead of
NCCL kernels, so the reduction does not take SMs from the backward GEMMs it
overlaps; the result is bit-identical on every rank.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


_READY = {}   # id(param) -> callback(param), for gradients written outside autograd


def notify_grad_ready(p):
    """Called by code that writes p.grad itself (the fused expert backward): tells a
    GradAllReducer that p's gradient is complete, as autograd's hook would."""
    cb = _READY.get(id(p))
    if cb is not None:
        cb(p)


def all_reduce_counts(counts: torch.Tensor, process_group=None) -> torch.Tensor:
    """Sum per-layer routing counts [L, E] over the data-parallel ranks (in place), so every
    rank applies the same aux-loss-free bias update (main.py:161-175 on the global batch)."""
    if process_group is not None and dist.is_initialized() and dist.get_world_size(process_group) > 1:
        dist.all_reduce(counts, group=process_group)
    return counts


def all_gather_sparse(grad: torch.Tensor, process_group=None) -> torch.Tensor:
    """Sum of every rank's sparse COO gradient (same dense shape), as one uncoalesced COO tensor."""
    world = dist.get_world_size(process_group)
    # duplicates need no coalescing here: the sum over ranks is the concatenation of the
    # ranks' entries, and the sparse-row optimizer sums duplicates itself
    idx, val = grad._indices(), grad._values()
    n = torch.tensor([idx.size(1)], device=idx.device, dtype=torch.long)
    sizes = [torch.zeros_like(n) for _ in range(world)]
    dist.all_gather(sizes, n, group=process_group)
    m = int(max(int(s.item()) for s in sizes))
    pad_idx = torch.zeros((idx.size(0), m), dtype=idx.dtype, device=idx.device)
    pad_val = torch.zeros((m,) + tuple(val.shape[1:]), dtype=val.dtype, device=val.device)
    pad_idx[:, : idx.size(1)] = idx
    pad_val[: val.size(0)] = val
    all_idx = [torch.empty_like(pad_idx) for _ in range(world)]
    all_val = [torch.empty_like(pad_val) for _ in range(world)]
    dist.all_gather(all_idx, pad_idx, group=process_group)
    dist.all_gather(all_val, pad_val, group=process_group)
    cat_idx = torch.cat([a[:, : int(s.item())] for a, s in zip(all_idx, sizes)], dim=1)
    cat_val = torch.cat([a[: int(s.item())] for a, s in zip(all_val, sizes)], dim=0)
    return torch.sparse_coo_tensor(cat_idx, cat_val, grad.shape)


class GradAllReducer:
    def __init__(self, params, process_group=None, bucket_mb=64.0, average=False, engine="nccl"):
        if engine not in ("nccl", "ce"):
            raise ValueError(f"unknown engine {engine!r}")
        self.group = process_group
        self.world = dist.get_world_size(process_group)
        self.average = average
        self.engine = engine
        self._ce = {}             # (bucket, dtype) -> CopyEngineAllReduce
        self._ce_used = False     # a copy-engine all-reduce ran since the last finish()
        self.params = [p for p in params if p.requires_grad]
        self.bucket_bytes = int(bucket_mb * (1 << 20))
        self._hooks = []
        self._index = {id(p): i for i, p in enumerate(self.params)}
        self._arrival = []
        self._rebuilt = False
        # first step: reverse registration order (the backward produces late layers first)
        self._build(list(reversed(range(len(self.params)))))
        self._stream = torch.cuda.Stream() if torch.cuda.is_available() and self.params and \
            self.params[0].is_cuda else None
        self._reset()
        for p in self.params:
            self._hooks.append(p.register_post_accumulate_grad_hook(self._on_grad))
            _READY[id(p)] = self._on_grad

    def _build(self, order):
        self.buckets = []
        cur, size = [], 0
        for i in order:
            p = self.params[i]
            cur.append(p)
            size += p.numel() * p.element_size()
            if size >= self.bucket_bytes:
                self.buckets.append(cur)
                cur, size = [], 0
        if cur:
            self.buckets.append(cur)
        self._bucket_of = {}
        for b, ps in enumerate(self.buckets):
            for p in ps:
                self._bucket_of[id(p)] = b

    def _rebuild_from_arrival(self):
        seen = set(self._arrival)
        order = list(self._arrival) + [i for i in range(len(self.params)) if i not in seen]
        obj = [order]
        dist.broadcast_object_list(obj, src=dist.get_global_rank(self.group, 0) if self.group is not None else 0,
                                   group=self.group)
        self._build(obj[0])
        self._rebuilt = True

    def _reset(self):
        self._ready = [set() for _ in self.buckets]
        self._launched = [False] * len(self.buckets)
        self._next = 0            # buckets are issued strictly in order on every rank
        self._pending = []        # (work, flat, params) of dense buckets
        self._sparse = []         # (param, reduced grad)

    def _close_ce(self):
        for ce in self._ce.values():
            ce.close()
        self._ce = {}

    def _check_peers(self):
        """A copy-engine all-reduce whose wait for a peer expired reduced stale or partial
        chunks: raise instead of handing those gradients to the optimizer, and drop the
        copy-engine state (its step flags no longer agree with the peers')."""
        from . import _lib as Z

        self._ce_used = False
        if torch.cuda.is_available():
            torch.cuda.current_stream().synchronize()
        err = Z.device_error()
        if err & 0x20:  # ZS_DEVERR_TIMEOUT_PEER
            Z.clear_device_error()
            self._close_ce()
            self._reset()
            raise RuntimeError("copy-engine gradient all-reduce: a peer rank did not signal in time "
                               "(ZS_DEVERR_TIMEOUT_PEER); the reduced gradients are invalid")

    def remove(self):
        for h in self._hooks:
            h.remove()
        self._hooks = []
        self._close_ce()
        for p in self.params:
            if _READY.get(id(p)) == self._on_grad:
                del _READY[id(p)]

    def _on_grad(self, p):
        b = self._bucket_of.get(id(p))
        if b is None or id(p) in self._ready[b]:
            return
        if not self._rebuilt:
            self._arrival.append(self._index[id(p)])
        self._ready[b].add(id(p))
        self._launch_ready()

    def _launch_ready(self):
        while self._next < len(self.buckets) and \
                len(self._ready[self._next]) == len(self.buckets[self._next]):
            self._launch(self._next)
            self._next += 1

    def _launch(self, b):
        ps = [p for p in self.buckets[b] if p.grad is not None]
        self._launched[b] = True
        dense = [p for p in ps if not p.grad.is_sparse]
        for p in ps:
            if p.grad.is_sparse:
                self._sparse.append((p, all_gather_sparse(p.grad, self.group)))
        if not dense:
            return
        if self._stream is not None:
            self._stream.wait_stream(torch.cuda.current_stream())
            ctx = torch.cuda.stream(self._stream)
        else:
            ctx = _Null()
        by_dtype = {}
        for p in dense:
            by_dtype.setdefault(p.grad.dtype, []).append(p)
        with ctx:
            for dt in sorted(by_dtype, key=str):   # same order on every rank
                group = by_dtype[dt]
                # a lone contiguous gradient is reduced in place (no flatten copy, no copy back)
                in_place = len(group) == 1 and group[0].grad.is_contiguous()
                flat = group[0].grad.view(-1) if in_place else torch.cat([p.grad.reshape(-1) for p in group])
                if self.engine == "ce" and self._rebuilt and flat.is_cuda and dt in (torch.bfloat16, torch.float32):
                    from .ce import CopyEngineAllReduce

                    key = (b, dt)
                    ce = self._ce.get(key)
                    if ce is not None and ce.count != flat.numel():
                        # the bucket changed size: release the old buffers and peer mappings once
                        # the copies that use them have finished
                        (self._stream or torch.cuda.current_stream()).synchronize()
                        ce.close()
                        ce = None
                    if ce is None:
                        ce = self._ce[key] = CopyEngineAllReduce(flat.numel(), dt, self.group, flat.device)
                    self._ce_used = True
                    ce(flat, scale=(1.0 / self.world) if self.average else 1.0,
                       stream=self._stream or torch.cuda.current_stream())
                    self._pending.append((None, flat, group, in_place))
                    continue
                work = dist.all_reduce(flat, group=self.group, async_op=True)
                self._pending.append((work, flat, group, in_place))

    def finish(self):
        """Issue the remaining buckets, wait, and write the reduced gradients back."""
        for b in range(len(self.buckets)):
            self._ready[b] = {id(p) for p in self.buckets[b]}
        self._launch_ready()
        for work, flat, dense, in_place in self._pending:
            if work is not None:
                work.wait()
            if self._stream is not None:
                torch.cuda.current_stream().wait_stream(self._stream)
                flat.record_stream(torch.cuda.current_stream())
            if self.average and work is not None:
                flat.div_(self.world)
            if in_place:
                continue
            off = 0
            for p in dense:
                n = p.numel()
                p.grad.copy_(flat[off:off + n].view_as(p.grad))
                off += n
        if self._ce_used:
            self._check_peers()
        for p, g in self._sparse:
            p.grad = g / self.world if self.average else g
        self._reset()
        if not self._rebuilt:
            self._rebuild_from_arrival()


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False
