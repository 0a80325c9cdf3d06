"""The MoE language model of the training step, assembled from this package's modules.

The reference defines the model in modeling/model.py (MoEModel:13-142); with a
reference checkout on the import path that file runs unchanged on this
package's modules (the `modeling` package here extends its path to the
reference's).  MoELM is the same network for machines without the reference
(the benchmarks, the GPU tests), written for this package's kernels:

* parameters and buffers carry the reference's names and shapes
  (embedding.weight, layers.{i}.self_attn.*, layers.{i}.mlp.*, norm.weight,
  output_layer.weight), so optimizer grouping (build_muonmd_optimizer) and the
  checkpoint files apply to either model;
* the input embedding is one gather kernel (zs_embedding_bag_forward): table
  rows, the f32 bag mean for token-superposition ids [B, S, s], and the
  sqrt(d) upscale of an untied table, written straight into the f32 residual
  stream; its backward writes the COO gradient nn.Embedding(sparse=True) would
  produce (one value row per lookup, zs_embedding_bag_backward), which the
  sparse-row optimizer consumes without coalescing;
* under bf16 autocast the final zero-centred RMSNorm writes bf16 directly (the
  classifier GEMM's operand type), in the fused norm kernel.

Initialisation follows the reference's recipe: N(0, initializer_range) for
every matrix, embedding rows projected to unit L2 norm, an untied head unless
config.tie_word_embeddings.  The Engram branch is not part of the training
step's hot path and is not provided (config.engram.layers must be empty).
"""
from __future__ import annotations

from functools import partial

import torch
import torch.nn as nn

from . import _lib as Z


class EmbeddingBagFunction(torch.autograd.Function):
    """out[..., :] = scale * mean over the bag of table rows (f32); the table's gradient is
    a COO tensor with one row per lookup (indices = the ids)."""

    @staticmethod
    def forward(ctx, ids, table, scale):
        Z.require_cuda(ids, table)
        if table.dtype != torch.float32 or not table.is_contiguous():
            raise Z.ZsError("the embedding table must be a contiguous f32 tensor")
        bag = ids.size(-1) if ids.dim() == 3 else 1
        lead = ids.shape[:2] if ids.dim() == 3 else ids.shape
        flat = ids.reshape(-1).to(torch.int64).contiguous()
        nb = flat.numel() // bag
        V, d = table.shape
        out = torch.empty(*lead, d, dtype=torch.float32, device=table.device)
        Z.count(1)
        Z.check(Z.lib().zs_embedding_bag_forward(table.data_ptr(), V, d, flat.data_ptr(), nb, bag, float(scale),
                                                 out.data_ptr(), Z.stream_of(table)), "zs_embedding_bag_forward")
        ctx.save_for_backward(flat)
        ctx.meta = (V, d, bag, nb, float(scale))
        return out

    @staticmethod
    def backward(ctx, dy):
        (flat,) = ctx.saved_tensors
        V, d, bag, nb, scale = ctx.meta
        dyc = dy.to(torch.float32).contiguous()
        values = torch.empty(flat.numel(), d, dtype=torch.float32, device=dy.device)
        Z.count(1)
        Z.check(Z.lib().zs_embedding_bag_backward(dyc.data_ptr(), nb, bag, d, scale, values.data_ptr(),
                                                  Z.stream_of(dyc)), "zs_embedding_bag_backward")
        grad = torch.sparse_coo_tensor(flat.view(1, -1), values, (V, d), is_coalesced=False, check_invariants=False)
        return None, grad, None


class MoELM(nn.Module):
    def __init__(self, config):
        super().__init__()
        from modeling.attention import GatedAttention
        from modeling.transformer_block import TransformerBlock
        from modeling.zRMSNorm import ZeroCenteredRMSNorm

        if tuple(getattr(getattr(config, "engram", None), "layers", ()) or ()):
            raise NotImplementedError("MoELM has no Engram branches (config.engram.layers must be empty)")
        self.config = config
        d = config.hidden_size
        self.embedding = nn.Embedding(config.vocab_size, d, sparse=True)
        self.layers = nn.ModuleList(
            TransformerBlock(config, partial(GatedAttention, window_size=w), True)
            for w in config.attention_window_pattern)
        self.norm = ZeroCenteredRMSNorm(d, eps=config.rms_norm_eps)
        self.output_layer = nn.Linear(d, config.vocab_size, bias=False)
        self.tie_word_embeddings = bool(config.tie_word_embeddings)
        self._init_weights()
        if self.tie_word_embeddings:
            self.output_layer.weight = self.embedding.weight

    @torch.no_grad()
    def _init_weights(self):
        std = self.config.initializer_range
        t = self.embedding.weight
        t.normal_(0.0, std)
        t.div_(torch.linalg.vector_norm(t, dim=1, keepdim=True).clamp_min(1e-12))
        if not self.config.tie_word_embeddings:
            self.output_layer.weight.normal_(0.0, std)

    def embed(self, ids):
        """[B, S] ids (or [B, S, s] token-superposition bags) -> f32 [B, S, d]."""
        scale = 1.0 if self.tie_word_embeddings else float(self.config.hidden_size) ** 0.5
        return EmbeddingBagFunction.apply(ids, self.embedding.weight, scale)

    def final_norm(self, h):
        from modeling.zRMSNorm import AddZRMSNormFunction, fused_add_norm_ok

        if (torch.is_autocast_enabled() and torch.get_autocast_dtype("cuda") == torch.bfloat16
                and fused_add_norm_ok(h)):
            return AddZRMSNormFunction.apply(h, None, self.norm.weight, self.norm.eps)
        return self.norm(h)

    def headless_forward(self, x, position_ids=None, cu_seqlens=None, unpad_indices=None, max_seqlen=None):
        """(normed hidden states [B, S, d], per-layer top-k expert ids), as the reference's
        MoEModel.headless_forward (modeling/model.py:134-139)."""
        h = self.embed(x)
        routing = []
        for block in self.layers:
            h, topk = block(h, position_ids=position_ids, cu_seqlens=cu_seqlens, max_seqlen=max_seqlen,
                            unpad_indices=unpad_indices)
            routing.append(topk)
        return self.final_norm(h), routing

    def forward(self, x, position_ids=None, cu_seqlens=None, unpad_indices=None, max_seqlen=None):
        h, routing = self.headless_forward(x, position_ids, cu_seqlens, unpad_indices, max_seqlen)
        return self.output_layer(h), routing

    def get_classifier_weights(self):
        return self.output_layer.weight
