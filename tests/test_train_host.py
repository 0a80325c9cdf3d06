"""Trainer host logic on CPU: the linear-decay LR schedule (main.py:512-555) on tensor and
float learning rates, and the next-token loss inputs (main.py:177-185)."""
import pytest
import torch


class _Opt:
    def __init__(self):
        self.param_groups = [dict(lr=torch.tensor(0.02)), dict(lr=3e-4)]


@pytest.mark.parametrize("warmup,min_ratio", [(0, 0.0), (4, 0.1)])
def test_linear_decay_schedule(warmup, min_ratio):
    from zs_b200.train import LinearDecayScheduler

    opt = _Opt()
    t0 = opt.param_groups[0]["lr"]
    sch = LinearDecayScheduler(opt, total_steps=20, warmup_steps=warmup, min_lr_ratio=min_ratio)
    seen = []
    for s in range(1, 26):
        lr = sch.step()
        if warmup and s < warmup:
            frac = s / warmup
        else:
            frac = 1.0 - (1.0 - min_ratio) * min(1.0, max(0.0, (s - warmup) / (20 - warmup)))
        assert abs(lr - 0.02 * frac) < 1e-9
        assert abs(float(opt.param_groups[0]["lr"]) - 0.02 * frac) < 1e-7
        assert abs(opt.param_groups[1]["lr"] - 3e-4 * frac) < 1e-12
        seen.append(lr)
    assert opt.param_groups[0]["lr"] is t0          # updated in place (graph-safe)
    assert abs(seen[-1] - 0.02 * min_ratio) < 1e-9


def test_next_token_loss_inputs():
    from zs_b200.train import build_next_token_loss_inputs

    ids = torch.tensor([[5, 6, 7, 8], [1, 2, 3, 0]])
    mask = torch.tensor([[1, 1, 1, 1], [1, 1, 1, 0]])
    emb = torch.randn(2, 4, 3)
    e, labels = build_next_token_loss_inputs(emb, ids, mask)
    assert e.shape == (2, 3, 3) and torch.equal(e, emb[:, :-1])
    assert labels.tolist() == [[6, 7, 8], [2, 3, -100]]
