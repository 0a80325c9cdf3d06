"""MoEModel (modeling/model.py:13-142): sparse input embedding (unit-norm rows,
sqrt(d) upscale when untied, bag mean for 3-D token-superposition ids), a
stack of TransformerBlocks with per-layer attention windows, final
zero-centred RMSNorm and an untied (or tied) output head.  Parameter names
match the reference so its optimizer grouping and checkpoints apply.  The
Engram branch (not part of the training step's hot path) is not provided:
config.engram.layers must be empty."""
from __future__ import annotations

from functools import partial

import torch
import torch.nn as nn

from .attention import GatedAttention
from .transformer_block import TransformerBlock
from .zRMSNorm import ZeroCenteredRMSNorm


class MoEModel(nn.Module):
    def __init__(self, config):
        super().__init__()
        if tuple(config.engram.layers):
            raise NotImplementedError("Engram branches are not provided by this package")
        self.config = config
        self.embedding = nn.Embedding(config.vocab_size, config.hidden_size, sparse=True)
        self.layers = nn.ModuleList([TransformerBlock(config, partial(GatedAttention, window_size=w), True)
                                     for w in config.attention_window_pattern])
        self.norm = ZeroCenteredRMSNorm(config.hidden_size, eps=config.rms_norm_eps)
        self.output_layer = nn.Linear(config.hidden_size, config.vocab_size, bias=False)
        self.tie_word_embeddings = config.tie_word_embeddings
        self.engram_layers = ()
        self.engrams = None
        self.reset_parameters()
        if self.tie_word_embeddings:
            self.tie_weights()

    def reset_parameters(self):
        nn.init.normal_(self.embedding.weight, mean=0.0, std=self.config.initializer_range)
        with torch.no_grad():
            self.embedding.weight.div_(self.embedding.weight.norm(dim=1, keepdim=True).clamp_min(1e-12))
        if not self.config.tie_word_embeddings:
            nn.init.normal_(self.output_layer.weight, mean=0.0, std=self.config.initializer_range)

    def tie_weights(self):
        self.output_layer.weight = self.embedding.weight

    def _embed_tokens(self, x):
        if x.ndim == 3:
            bag = self.embedding(x)
            emb = bag.float().mean(dim=-2).to(bag.dtype)
        else:
            emb = self.embedding(x)
        if not self.tie_word_embeddings:
            emb = emb * (self.config.hidden_size ** 0.5)
        return emb

    def _run_layers(self, x, token_ids, position_ids, cu_seqlens, unpad_indices, max_seqlen):
        all_topk = []
        for layer in self.layers:
            x, topk_idx = layer(x, position_ids=position_ids, cu_seqlens=cu_seqlens, max_seqlen=max_seqlen,
                                unpad_indices=unpad_indices)
            all_topk.append(topk_idx)
        return x, all_topk

    def forward(self, x, position_ids=None, cu_seqlens=None, unpad_indices=None, max_seqlen=None):
        h, all_topk = self.headless_forward(x, position_ids, cu_seqlens, unpad_indices, max_seqlen)
        return self.output_layer(h), all_topk

    def headless_forward(self, x, position_ids=None, cu_seqlens=None, unpad_indices=None, max_seqlen=None):
        token_ids = x
        h = self._embed_tokens(x)
        h, all_topk = self._run_layers(h, token_ids, position_ids, cu_seqlens, unpad_indices, max_seqlen)
        return self.norm(h), all_topk

    def get_classifier_weights(self):
        return self.output_layer.weight
