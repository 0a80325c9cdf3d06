"""Trainer-side pieces of the MoE training step (main.py), on this package's
kernels: the MuonMD + aux-Adam + sparse-embedding optimizer grouping
(build_muonmd_optimizer, main.py:354-465), the aux-loss-free router bias
update (main.py:161-175; routing counts optionally all-reduced across
data-parallel ranks so every rank applies the same bias update) and the
next-token loss inputs (main.py:177-185)."""
from __future__ import annotations

import torch

from . import _lib as Z


def build_next_token_loss_inputs(embeddings, input_ids, attention_mask, loss_mask=None, ignore_index=-100):
    source = attention_mask[:, :-1].bool()
    target = attention_mask[:, 1:].bool()
    if loss_mask is not None:
        target = target & loss_mask[:, 1:].bool()
    labels = input_ids[:, 1:].masked_fill(~(source & target), ignore_index)
    return embeddings[:, :-1, :].contiguous(), labels.contiguous()


@torch.no_grad()
def auxillary_loss_free_update(model, all_topk_indices, update_rate, attention_mask=None, process_group=None):
    """bias += update_rate * sign(mean(counts) - counts) per layer; with a
    process group the counts are summed over ranks first (one all-reduce of
    [L, E] int64)."""
    layers = [model.layers[i].mlp.gate for i in range(len(all_topk_indices))]
    if not layers:
        return
    E = layers[0].n_routed_experts
    dev = layers[0].expert_biases.device
    counts = torch.zeros(len(layers), E, dtype=torch.long, device=dev)
    valid = None
    if attention_mask is not None:
        valid = attention_mask.reshape(-1).to(torch.uint8).contiguous()
    for i, topk in enumerate(all_topk_indices):
        t = topk.reshape(-1, topk.size(-1)).to(torch.int64).contiguous()
        Z.count(1)
        Z.check(Z.lib().zs_expert_counts(t.data_ptr(), Z.ptr(valid), t.size(0), t.size(1), E, counts[i].data_ptr(),
                                         Z.stream_of(t)), "zs_expert_counts")
    if process_group is not None:
        from .dp import all_reduce_counts

        all_reduce_counts(counts, process_group)
    for i, gate in enumerate(layers):
        Z.count(1)
        Z.check(Z.lib().zs_bias_sign_update(counts[i].data_ptr(), E, float(update_rate), gate.expert_biases.data_ptr(),
                                            Z.stream_of(counts)), "zs_bias_sign_update")


def enable_fused_weight_grad(model, enabled=True):
    """Let every GLUMLP in the model accumulate its f32 expert weight gradients into .grad
    straight from the weight-gradient GEMMs (training loops that call loss.backward() and
    read param.grad; not for torch.autograd.grad on those weights).  Returns the count."""
    from scattermoe.mlp import GLUMLP

    n = 0
    for m in model.modules():
        if isinstance(m, GLUMLP):
            m.fuse_weight_grad = bool(enabled)
            # the GEMMs can overwrite a stale gradient: HybridGraphOptimizer.zero_grad skips
            # the fill of these buffers
            for w in (m.experts.weight, m.output_experts.weight):
                w._zs_grad_overwrite = bool(enabled)
            n += 1
    return n


def build_muonmd_optimizer(model, device, muon_lr=0.02, adam_lr=3e-4, momentum=0.95, gain_lr=1e-3,
                           adam_betas=(0.9, 0.95), adam_eps=1e-16, embedding_weight_decay=0.1, embedding_lr=3e-3,
                           embedding_beta=0.9, capture_warmup_steps=5, enable_cuda_graph=True, process_group=None):
    """Groups: Muon (Frobenius sphere) for matrices and expert stacks; the router
    on row spheres with column gains and the Muon shape factor; AdamW with weight
    decay for the output head; Adam for 1-D params; GramReaperSparse (unit rows)
    for the sparse input embedding.  Dense LRs are 0-dim device tensors so the
    captured step reads scheduler updates.  With a data-parallel process group the
    dense optimizer is MuonMDWithAuxAdam (Newton-Schulz split over the ranks and
    all-gathered) and runs eagerly, so no CUDA graph holds the collectives."""
    from engram.GramReaperSparse import GramReaperSparse
    from optimizer.hybrid import HybridGraphOptimizer
    from optimizer.muon import MuonMDWithAuxAdam, SingleDeviceMuonMDWithAuxAdam

    emb = model.embedding.weight
    muon, router, head, scalar = [], [], [], []
    for name, p in model.named_parameters():
        if not p.requires_grad or p is emb:
            continue
        if "output_layer" in name:
            head.append(p)
        elif p.ndim >= 2:
            (router if "mlp.gate.weight" in name else muon).append(p)
        else:
            scalar.append(p)
    t = lambda v: torch.tensor(float(v), device=device)  # noqa: E731
    groups = [dict(params=muon, use_muon=True, lr=t(muon_lr), momentum=momentum, gain_lr=gain_lr, capturable=True)]
    if router:
        groups.append(dict(params=router, use_muon=True, lr=t(muon_lr), momentum=momentum, gain_lr=gain_lr,
                           norm_axis="row", gain_mode="col", rescale_mode="muon", capturable=True))
    if head:
        groups.append(dict(params=head, use_muon=False, lr=t(adam_lr), betas=adam_betas, eps=adam_eps,
                           weight_decay=embedding_weight_decay, capturable=True))
    groups.append(dict(params=scalar, use_muon=False, lr=t(adam_lr), betas=adam_betas, eps=adam_eps, weight_decay=0.0,
                       capturable=True))
    sharded = process_group is not None and torch.distributed.get_world_size(process_group) > 1
    dense = MuonMDWithAuxAdam(groups, process_group) if sharded else SingleDeviceMuonMDWithAuxAdam(groups)
    sparse = GramReaperSparse([dict(params=[emb], unit_norm=True)], lr=float(embedding_lr), beta=embedding_beta,
                              unit_norm=True)
    return HybridGraphOptimizer(dense, sparse, capture_warmup_steps=capture_warmup_steps,
                                enable_cuda_graph=enable_cuda_graph and not sharded)


def _lr_value(lr):
    return float(lr.item()) if torch.is_tensor(lr) else float(lr)


class LinearDecayScheduler:
    """Linear LR decay without warmup by default (main.py:512-555): every group's LR is its
    peak times fraction = 1 - (1 - min_lr_ratio) * progress, progress = (step - warmup) /
    (total - warmup) clamped to [0, 1]; with warmup_steps > 0 the first steps ramp linearly.
    0-dim LR tensors are updated in place (fill_), so a CUDA-graph-captured optimizer step
    reads the new LR on every replay; float LRs are replaced.  Returns the first group's LR."""

    def __init__(self, optimizer, total_steps, warmup_steps=0, min_lr_ratio=0.0):
        self.optimizer = optimizer
        self.total_steps = max(1, int(total_steps))
        self.warmup_steps = min(max(0, int(warmup_steps)), self.total_steps)
        self.min_lr_ratio = float(min_lr_ratio)
        self.base_lrs = [_lr_value(g["lr"]) for g in optimizer.param_groups]
        self.step_count = 0
        self.peak_lr = self.base_lrs[0]
        self.min_lr = self.peak_lr * self.min_lr_ratio

    def _fraction(self):
        if self.warmup_steps > 0 and self.step_count < self.warmup_steps:
            return self.step_count / self.warmup_steps
        span = max(1, self.total_steps - self.warmup_steps)
        progress = min(1.0, max(0.0, (self.step_count - self.warmup_steps) / span))
        return 1.0 - (1.0 - self.min_lr_ratio) * progress

    def step(self, increment=1):
        self.step_count += increment
        frac = self._fraction()
        for base, group in zip(self.base_lrs, self.optimizer.param_groups):
            if torch.is_tensor(group["lr"]):
                group["lr"].fill_(base * frac)
            else:
                group["lr"] = base * frac
        return self.base_lrs[0] * frac
