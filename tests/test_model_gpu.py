"""Whole-model checks on the GPU: causality (no position sees later tokens),
the loss of an untrained model on uniform tokens (~ log V), and agreement of
the fused CCE with a materialised cross entropy on the model's hidden state."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _tiny(layers=2, window=None):
    from modeling.model_config import ModelConfig
    from zs_b200.lm import MoELM as MoEModel

    cfg = ModelConfig(vocab_size=8192, embed_size=256, hidden_size=256, transformer_depth=layers,
                      intermediate_size=512, n_experts=9, n_shared_experts=1, n_experts_per_token=2,
                      n_attention_heads=4, n_key_value_heads=4, attention_window_pattern=(window,) * layers,
                      max_position_embeddings=256, sequence_length=256, pos_rope_dims=32)
    torch.manual_seed(0)
    return cfg, MoEModel(cfg).cuda()


@pytest.mark.parametrize("window", [None, 16])
def test_model_is_causal(window):
    cfg, m = _tiny(window=window)
    ids = torch.randint(0, cfg.vocab_size, (2, 256), device="cuda")
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        h1, _ = m.headless_forward(ids)
        ids2 = ids.clone()
        ids2[:, 100:] = torch.randint(0, cfg.vocab_size, (2, 156), device="cuda")
        h2, _ = m.headless_forward(ids2)
    # positions before 100 must not change when later tokens do
    assert torch.equal(h1[:, :100], h2[:, :100])
    assert not torch.equal(h1[:, 100:], h2[:, 100:])


def test_untrained_loss_is_near_log_vocab_and_matches_materialised_ce():
    from cut_cross_entropy import linear_cross_entropy

    cfg, m = _tiny()
    ids = torch.randint(0, cfg.vocab_size, (4, 256), device="cuda")
    with torch.autocast("cuda", dtype=torch.bfloat16):
        h, _ = m.headless_forward(ids)
        e = h[:, :-1].contiguous()
        t = ids[:, 1:].contiguous()
        loss = linear_cross_entropy(e, m.get_classifier_weights(), t)
    ref = torch.nn.functional.cross_entropy((e.float() @ m.get_classifier_weights().float().T).view(-1, cfg.vocab_size),
                                            t.view(-1))
    assert abs(loss.item() - ref.item()) / ref.item() < 2e-2
    assert abs(loss.item() - math.log(cfg.vocab_size)) < 2.0


def test_fused_add_norm_block_matches_reference_op_sequence():
    """The block's fused residual-add + zRMSNorm path (bf16 norm outputs under autocast)
    against the reference op sequence (add, f32 norm, autocast casts): block output,
    input gradient and every parameter gradient agree to reduction-order rounding."""
    from modeling.transformer_block import TransformerBlock

    cfg, m = _tiny(layers=1)
    blk = m.layers[0]
    with torch.no_grad():
        for n in (blk.input_layernorm, blk.post_attention_layernorm):
            n.weight.normal_(0, 0.1)
    g = torch.Generator(device="cuda").manual_seed(5)
    x0 = torch.randn(2, 256, 256, device="cuda", generator=g)
    dy = torch.randn(2, 256, 256, device="cuda", generator=g)
    outs = []
    for fused in (False, True):
        TransformerBlock.fused_add_norm = fused
        try:
            blk.zero_grad(set_to_none=True)
            x = x0.clone().requires_grad_(True)
            with torch.autocast("cuda", dtype=torch.bfloat16):
                y, _ = blk(x)
            y.backward(dy)
            torch.cuda.synchronize()
            outs.append((y.detach().float(), x.grad.clone(),
                         {n: p.grad.detach().float().clone() for n, p in blk.named_parameters() if p.grad is not None}))
        finally:
            TransformerBlock.fused_add_norm = True
    (ya, xa, ga), (yb, xb, gb) = outs
    assert yb.dtype == ya.dtype
    assert ((ya - yb).norm() / ya.norm()).item() < 5e-3
    cos = lambda a, b: (a.flatten() @ b.flatten() / (a.norm() * b.norm())).item()  # noqa: E731
    assert cos(xa, xb) > 0.9999
    assert ga.keys() == gb.keys()
    for n in ga:
        assert cos(ga[n], gb[n]) > 0.999, n


def test_lazy_zero_grad_of_fused_expert_gradients_matches_filled_buffers():
    """HybridGraphOptimizer.zero_grad marks the expert weight gradients that the weight-
    gradient GEMMs write directly as stale instead of filling them, and the GEMMs overwrite
    them: three full training steps (eager, then graph-replayed optimizer) leave every
    parameter bit-identical to the run whose buffers are zero-filled and accumulated into."""
    from cut_cross_entropy import linear_cross_entropy
    from zs_b200.train import build_muonmd_optimizer, build_next_token_loss_inputs, enable_fused_weight_grad

    runs = []
    for lazy in (True, False):
        cfg, m = _tiny()
        enable_fused_weight_grad(m)
        if not lazy:
            for mod in m.modules():
                for w in (getattr(getattr(mod, "experts", None), "weight", None),
                          getattr(getattr(mod, "output_experts", None), "weight", None)):
                    if w is not None:
                        w._zs_grad_overwrite = False
        opt = build_muonmd_optimizer(m, torch.device("cuda"), capture_warmup_steps=1)
        g = torch.Generator(device="cuda").manual_seed(9)
        for _ in range(3):
            ids = torch.randint(0, cfg.vocab_size, (2, 256), device="cuda", generator=g)
            mask = torch.ones_like(ids)
            opt.zero_grad(set_to_none=False)
            with torch.autocast("cuda", dtype=torch.bfloat16):
                h, _ = m.headless_forward(ids)
                e, t = build_next_token_loss_inputs(h, ids, mask)
                loss = linear_cross_entropy(e, m.get_classifier_weights(), t, ignore_index=-100)
            loss.backward()
            opt.step()
        torch.cuda.synchronize()
        runs.append({n: p.detach().clone() for n, p in m.named_parameters()})
        stale = [n for n, p in m.named_parameters() if getattr(p, "_zs_grad_stale", False)]
        assert not stale, stale
    for n in runs[0]:
        assert torch.equal(runs[0][n], runs[1][n]), n


def test_token_superposition_step_on_bags():
    """BASELINE config 5's input format through the whole model: [B, S, 4] bags of token ids
    (bag-mean embedding, sqrt(d) upscale of an untied table), the next position's bag as the
    4-target MCCE labels; the loss of the untrained model is near log V, the bag embedding equals
    the mean of the table rows, every lookup gets one COO gradient row, and the hidden states'
    gradient and every parameter gradient are finite."""
    from modeling.mcce_fast_v2 import mcce_raw_token_mean_v2

    cfg, m = _tiny()
    B, S, bag = 2, 256, 4
    ids = torch.randint(0, cfg.vocab_size, (B, S, bag), device="cuda")
    emb = m.embed(ids)
    scale = 1.0 if m.tie_word_embeddings else math.sqrt(cfg.hidden_size)
    want = m.embedding.weight[ids].mean(2) * scale
    assert torch.allclose(emb, want, rtol=1e-5, atol=1e-6)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        h, routing = m.headless_forward(ids)
        hidden = h[:, :-1].reshape(-1, h.size(-1))
        labels = ids[:, 1:].reshape(-1, bag)
        s = torch.full((labels.size(0),), bag, dtype=torch.long, device="cuda")
        loss = mcce_raw_token_mean_v2(hidden, m.get_classifier_weights(), labels, s)
    assert abs(float(loss) - math.log(cfg.vocab_size)) < 0.5
    loss.backward()
    g = m.embedding.weight.grad
    assert g.is_sparse and g._nnz() == B * S * bag
    for name, p in m.named_parameters():
        if p.grad is not None and not p.grad.is_sparse:
            assert torch.isfinite(p.grad).all(), name
    assert len(routing) == cfg.transformer_depth
