"""ModelConfig: the reference's configuration schema (modeling/model_config.py:45-185),
same field names, defaults, derived fields and validation, so configurations
written for the reference load unchanged.  Engram settings are accepted but
only the disabled form (no layers) is supported by this package's model."""
from __future__ import annotations

import math
from dataclasses import dataclass, field

SUPERPOSITION_REFERENCE_SIZE = 1
SUPERPOSITION_TRAINING_MAX_SIZE = 32


@dataclass
class EngramSettings:
    layers: tuple = ()
    orders: tuple = (2, 3)
    n_heads: int = 4
    rows_per_head: int = 65521
    dim_per_head: int = 64
    alpha_init: float = 0.0
    importance_weighting: bool = False
    head_norm: bool = True
    learned_gate: bool = True


@dataclass
class ModelConfig:
    vocab_size: int = 8192
    embed_size: int = 512
    hidden_size: int = 512
    transformer_depth: int = 8
    intermediate_size: int = 160
    n_experts: int = 34
    n_shared_experts: int = 2
    n_experts_per_token: int = 2
    n_routed_experts: int = field(init=False)
    n_attention_heads: int = 16
    n_key_value_heads: int = 4
    attention_window_pattern: tuple = (256, 256, 256, None, 512, 512, 512, None)
    use_qk_norm: bool = True
    hca_block_size: int = 128
    hca_window_size: int = 128
    rms_norm_eps: float = 1e-6
    max_position_embeddings: int = 4096
    sequence_length: int = 4096
    rope_theta: int = 10000
    do_rope: bool = True
    initializer_range: float = field(init=False)
    tie_word_embeddings: bool = False
    pos_rope_dims: int = 16
    # learned per-head sink key (value 0) in every GatedAttention layer; off keeps the
    # reference's state dict
    attention_sink: bool = False
    superposition_enabled: bool = False
    superposition_max_size: int = field(init=False)
    engram: EngramSettings = field(default_factory=EngramSettings)
    pad_token_id: int = 0

    def __post_init__(self):
        self.superposition_max_size = (SUPERPOSITION_TRAINING_MAX_SIZE if self.superposition_enabled
                                       else SUPERPOSITION_REFERENCE_SIZE)
        self.n_routed_experts = self.n_experts - self.n_shared_experts
        self.initializer_range = 1.0 / math.sqrt(self.hidden_size)
        checks = [
            (self.embed_size == self.hidden_size, "embed_size and hidden_size must match"),
            (self.n_routed_experts > 0, "n_experts must be greater than n_shared_experts."),
            (self.n_experts_per_token > 0, "n_experts_per_token must be positive."),
            (self.n_experts_per_token <= self.n_routed_experts, "n_experts_per_token cannot exceed n_routed_experts."),
            (self.hidden_size % self.n_attention_heads == 0, "hidden_size must be divisible by n_attention_heads."),
            (self.n_attention_heads % self.n_key_value_heads == 0,
             "n_attention_heads must be divisible by n_key_value_heads."),
            (len(self.attention_window_pattern) == self.transformer_depth,
             "attention_window_pattern must have transformer_depth entries"),
            (self.sequence_length <= self.max_position_embeddings,
             "sequence_length cannot exceed max_position_embeddings."),
            (self.pos_rope_dims >= 0 and self.pos_rope_dims % 2 == 0, "pos_rope_dims must be even and >= 0."),
            (self.pos_rope_dims <= self.hidden_size // self.n_attention_heads, "pos_rope_dims cannot exceed head_dim"),
        ]
        for ok, msg in checks:
            if not ok:
                raise ValueError(msg)
        for w in self.attention_window_pattern:
            if w is not None and (not isinstance(w, int) or isinstance(w, bool) or w <= 0):
                raise ValueError(f"attention_window_pattern entries must be None or a positive int, got {w!r}.")
