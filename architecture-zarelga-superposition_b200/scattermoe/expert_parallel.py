"""Expert-parallel GLUMLP: the routed experts of one MoE layer sharded over the
ranks of a process group, tokens moved to their experts and back by NCCL
all-to-all over NVLink.

The reference trains on one device and has no expert parallelism; this layer is
the expert-parallel form of its GLUMLP (scattermoe/mlp.py:74-95) that the large
configuration (128 experts, 16 per GPU on 8 GPUs) needs.  Same forward signature
as GLUMLP -- forward(x [T, d], expert_p [T, k], expert_idxs [T, k]) with global
expert ids -- and the same parameter names and per-expert layout
(experts.weight [E_local, 2f, d], output_experts.weight [E_local, d, f]); rank r
holds global experts [r * E_local, (r + 1) * E_local).

One forward, per rank:
  1. flatten_sort_count over the global expert ids: the (token, slot) pairs in
     expert order, which is also destination-rank order (rank = expert // E_local);
  2. the per-expert counts are exchanged with one all-to-all (a [world, E_local]
     int64 table per rank; the split sizes are read on the host once per layer);
  3. dispatch: the slots' token rows (and routing weights) are gathered in that
     order and sent with all_to_all_single;
  4. the received rows -- blocks per source rank, each ordered by local expert --
     run through the fused GLU experts (grouped tcgen05 GEMMs, SwiGLU epilogue)
     with k = 1, each row scaled by its routing weight;
  5. combine: the output rows return with the reverse all_to_all_single, are put
     back in (token, slot) order and summed over the k slots.
The backward mirrors it: the all-to-alls run with swapped splits, the gather's
adjoint is the slot sum and vice versa.  Expert weight gradients stay on their
rank (no data-parallel all-reduce for them); the routing-weight gradient returns
to the token's rank through the dispatch all-to-all's backward.
"""
from __future__ import annotations

import torch
import torch.distributed as dist
from torch import nn

from .parallel_experts import ParallelExperts, flatten_sort_count


def _all_to_all(t, out_splits, in_splits, group, world):
    """_AllToAll, or t itself when the group has one rank (nothing to exchange)."""
    return t if world == 1 else _AllToAll.apply(t, out_splits, in_splits, group)


class _AllToAll(torch.autograd.Function):
    """all_to_all_single with variable splits along dim 0; backward sends the
    gradient back with the splits swapped."""

    @staticmethod
    def forward(ctx, t, out_splits, in_splits, group):
        ctx.splits, ctx.group = (list(out_splits), list(in_splits)), group
        out = t.new_empty((sum(out_splits),) + tuple(t.shape[1:]))
        dist.all_to_all_single(out, t.contiguous(), list(out_splits), list(in_splits), group=group)
        return out

    @staticmethod
    def backward(ctx, g):
        out_splits, in_splits = ctx.splits
        gi = g.new_empty((sum(in_splits),) + tuple(g.shape[1:]))
        dist.all_to_all_single(gi, g.contiguous(), in_splits, out_splits, group=ctx.group)
        return gi, None, None, None


class _SlotGather(torch.autograd.Function):
    """rows[i] = x[ssi[i] // k] (the libzs gather kernel); adjoint: the slot sum."""

    @staticmethod
    def forward(ctx, x, ssi, k):
        from .kernels import ops

        ctx.save_for_backward(ssi)
        ctx.k, ctx.T = k, x.size(0)
        return ops.group(x.contiguous(), ssi, fan_out=k)

    @staticmethod
    def backward(ctx, g):
        (ssi,) = ctx.saved_tensors
        return _slot_sum(g, ssi, ctx.T, ctx.k), None, None


class _SlotSum(torch.autograd.Function):
    """y[t] = sum_j rows[pos(t, j)] with rows in expert order (pos = the inverse of
    ssi); adjoint: the gather."""

    @staticmethod
    def forward(ctx, rows, ssi, T, k):
        ctx.save_for_backward(ssi)
        ctx.k = k
        return _slot_sum(rows, ssi, T, k)

    @staticmethod
    def backward(ctx, g):
        from .kernels import ops

        (ssi,) = ctx.saved_tensors
        return ops.group(g.contiguous(), ssi, fan_out=ctx.k), None, None, None


def _slot_sum(rows, ssi, T, k):
    """y[t] = sum_j rows[pos(t, j)] in one pass (libzs gathered row sum), pos the inverse of ssi."""
    from zs_b200 import _lib as Z

    n = ssi.numel()
    pos = torch.empty_like(ssi)
    pos[ssi] = torch.arange(n, device=ssi.device, dtype=ssi.dtype)
    rows = rows.contiguous()
    C = rows.size(1)
    out = torch.empty((T, C), dtype=rows.dtype, device=rows.device)
    Z.count(1)
    Z.check(Z.lib().zs_gathered_row_sum(out.data_ptr(), out.stride(0), rows.data_ptr(), rows.stride(0), rows.size(0),
                                        pos.data_ptr(), T, k, C, Z.dtype_code(rows.dtype), Z.stream_of(rows)),
            "zs_gathered_row_sum")
    return out


def _glu_experts(x, p, lid, W1, W2, num_local, fuse_wgrad):
    from .mlp import GLUExpertsFunction

    return GLUExpertsFunction.apply(x, p, lid, W1, W2, num_local, 1, fuse_wgrad)


class ExpertParallelGLUMLP(nn.Module):
    """GLUMLP with its num_experts experts split evenly over the ranks of
    process_group (default: the world group).  `kernels` replaces the device
    functions (gather, slot sum, experts, sort); the default is libzs.so."""

    def __init__(self, input_size, hidden_size, num_experts, top_k, process_group=None, bias=False,
                 activation=nn.SiLU(), kernels=None):
        super().__init__()
        if bias or not isinstance(activation, nn.SiLU):
            raise ValueError("ExpertParallelGLUMLP supports bias=False with the SiLU gate (the fused GLU experts)")
        self.group = dist.group.WORLD if process_group is None else process_group
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        if num_experts % self.world:
            raise ValueError(f"{num_experts} experts do not split evenly over {self.world} ranks")
        self.num_experts = num_experts
        self.num_local = num_experts // self.world
        self.first_expert = self.rank * self.num_local
        self.input_size = input_size
        self.hidden_size = hidden_size
        self.top_k = min(top_k, num_experts)
        self.experts = ParallelExperts(self.num_local, input_size, 2 * hidden_size)
        self.output_experts = ParallelExperts(self.num_local, hidden_size, input_size)
        self.fuse_weight_grad = False
        k = kernels or {}
        self._gather = k.get("gather", _SlotGather.apply)
        self._slot_sum = k.get("slot_sum", _SlotSum.apply)
        self._experts = k.get("experts", _glu_experts)
        self._sort = k.get("sort", flatten_sort_count)

    def extra_repr(self):
        return f"k={self.top_k}, experts {self.first_expert}..{self.first_expert + self.num_local - 1} " \
               f"of {self.num_experts}"

    @torch.no_grad()
    def load_from_full(self, glumlp):
        """Copy this rank's slice of a full GLUMLP's expert weights."""
        sl = slice(self.first_expert, self.first_expert + self.num_local)
        self.experts.weight.copy_(glumlp.experts.weight[sl])
        self.output_experts.weight.copy_(glumlp.output_experts.weight[sl])
        return self

    def _splits(self, offs):
        """(send rows per rank, receive rows per rank, receive counts [world, E_local]) from the
        inclusive per-expert offsets of this rank's slots; one all-to-all of the counts."""
        counts = torch.diff(offs, prepend=offs.new_zeros(1))
        if self.world == 1:
            recv = counts
        else:
            recv = torch.empty_like(counts)
            dist.all_to_all_single(recv, counts.contiguous(), group=self.group)
        both = torch.cat([counts, recv]).cpu()  # the one host read per layer: NCCL needs the split sizes
        send_c = both[:self.num_experts].view(self.world, self.num_local)
        recv_c = both[self.num_experts:].view(self.world, self.num_local)
        return send_c.sum(1).tolist(), recv_c.sum(1).tolist(), recv_c

    def forward(self, x: torch.Tensor, expert_p: torch.Tensor, expert_idxs: torch.Tensor):
        shape = x.size()
        x = x.reshape(-1, shape[-1])
        T, d, k = x.size(0), x.size(1), self.top_k
        idx = expert_idxs.reshape(T, k)
        _, ssi, offs = self._sort(idx, self.num_experts)
        send, recv, recv_c = self._splits(offs)
        x_send = self._gather(x, ssi, k)
        p_send = expert_p.reshape(-1)[ssi]
        x_recv = _all_to_all(x_send, recv, send, self.group, self.world)
        p_recv = _all_to_all(p_send, recv, send, self.group, self.world)
        R = x_recv.size(0)
        W1, W2 = self.experts.weight, self.output_experts.weight
        if R:
            lid = torch.repeat_interleave(torch.arange(self.num_local, device=x.device).repeat(self.world),
                                          recv_c.flatten().to(x.device), output_size=R)
            y_recv = self._experts(x_recv, p_recv.view(R, 1), lid.view(R, 1), W1, W2, self.num_local,
                                   self.fuse_weight_grad)
        else:
            # no rows for this rank's experts: zero gradients for its weights; the empty
            # received tensors stay in the graph so every rank runs the same backward
            # all-to-alls in the same order
            y_recv = x_recv.new_zeros((0, d)) + (W1.sum() + W2.sum() + x_recv.sum() + p_recv.sum()).to(x_recv.dtype) * 0
        y_back = _all_to_all(y_recv.to(x.dtype), send, recv, self.group, self.world)
        y = self._slot_sum(y_back, ssi, T, k)
        return y.view(*shape[:-1], y.size(-1))


def shard_experts(model, process_group=None):
    """Replace every GLUMLP in `model` by an ExpertParallelGLUMLP holding this rank's
    slice of its experts (same module names, so parameter names are unchanged; the
    expert weights become [E / world, ...]).  The expert weights are then rank-local:
    a data-parallel gradient reducer must skip them.  Returns the sharded modules."""
    from .mlp import GLUMLP

    out = []
    for parent in list(model.modules()):
        for name, child in list(parent.named_children()):
            if isinstance(child, GLUMLP):
                w = child.experts.weight
                ep = ExpertParallelGLUMLP(child.input_size, child.hidden_size, child.num_experts, child.top_k,
                                          process_group).to(device=w.device, dtype=w.dtype)
                ep.load_from_full(child)
                ep.fuse_weight_grad = child.fuse_weight_grad
                setattr(parent, name, ep)
                out.append(ep)
    return out
