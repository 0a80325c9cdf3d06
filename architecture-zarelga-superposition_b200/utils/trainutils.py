"""Checkpoints and parameter counts with the reference's interface and on-disk
format (utils/trainutils.py:9-88): the model's state dict as one safetensors
file (the tied output head dropped and re-tied on load) and the trainer state
(optimizer state dict, scheduler fields, global step, epoch) in a torch file
beside it with the suffix `.trainer.pt`.  Parameter names, shapes and the
optimizer state layout are the reference's, so checkpoints written by either
implementation load into the other.

AimLogger (metrics to the `aim` tracker, :91-...) is observability outside the
training step; it is importable so trainers import unchanged, and needs the
`aim` package when constructed.
"""
from __future__ import annotations

from pathlib import Path

import torch


def count_parameters_layerwise(model):
    total = 0
    layer = {}
    for name, p in model.named_parameters():
        if not p.requires_grad:
            continue
        layer[name] = p.numel()
        total += p.numel()
    print("\nModel Parameter Summary:")
    print("-" * 60)
    for name, n in layer.items():
        print(f"{name}: {n:,} parameters")
    print("-" * 60)
    print(f"Total Trainable Parameters: {total:,}\n")
    return total


def _trainer_state_path(filename):
    return Path(filename).with_suffix(".trainer.pt")


def _base(model):
    return model._orig_mod if hasattr(model, "_orig_mod") else model


def save_checkpoint(model, optimizer, filename="checkpoint.safetensors", scheduler=None, global_step=None, epoch=None):
    from safetensors.torch import save_file

    base = _base(model)
    state = {k: v.detach().contiguous() for k, v in base.state_dict().items()}
    if getattr(base, "tie_word_embeddings", False):
        state.pop("output_layer.weight", None)  # shares the embedding's storage
    save_file(state, str(filename))
    trainer = {"optimizer": optimizer.state_dict()}
    if scheduler is not None:
        trainer["scheduler"] = {k: getattr(scheduler, k) for k in
                                ("step_count", "total_steps", "warmup_steps", "peak_lr", "min_lr")}
    if global_step is not None:
        trainer["global_step"] = global_step
    if epoch is not None:
        trainer["epoch"] = epoch
    torch.save(trainer, _trainer_state_path(filename))


def load_checkpoint(model, optimizer, filename="checkpoint.safetensors", scheduler=None):
    from safetensors.torch import load_file

    base = _base(model)
    tied = getattr(base, "tie_word_embeddings", False)
    base.load_state_dict(load_file(str(filename)), strict=not tied)
    if tied:
        base.tie_weights()
    path = _trainer_state_path(filename)
    if not path.exists():
        return {}
    trainer = torch.load(path, map_location="cpu", weights_only=False)
    if "optimizer" in trainer:
        optimizer.load_state_dict(trainer["optimizer"])
    if scheduler is not None and "scheduler" in trainer:
        for k, v in trainer["scheduler"].items():
            setattr(scheduler, k, v)
    return {"global_step": trainer.get("global_step"), "epoch": trainer.get("epoch")}


class AimLogger:
    """Training metrics to an `aim` run (the reference's logger); requires `aim`."""

    def __init__(self, repo="logs/aim", experiment="moe_training", enable_detailed_logging=True,
                 detailed_frequency=10):
        try:
            from aim import Run
        except ImportError as e:  # pragma: no cover - depends on the environment
            raise ImportError("AimLogger needs the `aim` package") from e
        Path(repo).mkdir(parents=True, exist_ok=True)
        self.run = Run(repo=str(repo), experiment=experiment)
        self.enable_detailed_logging = enable_detailed_logging
        self.detailed_frequency = detailed_frequency

    def log_metrics(self, metrics, step=None):
        for name, value in metrics.items():
            self.run.track(float(value), name=name, step=step)

    def close(self):
        self.run.close()
