from pathlib import Path

import numpy as np
import torch

GOLDEN_DIR = Path(__file__).resolve().parent / "golden"


def rel_err(a, b):
    a = torch.as_tensor(a).double().cpu()
    b = torch.as_tensor(b).double().cpu()
    return (a - b).norm().item() / max(b.norm().item(), 1e-30)


def cosine(a, b):
    a = torch.as_tensor(a).double().cpu().flatten()
    b = torch.as_tensor(b).double().cpu().flatten()
    return (a @ b).item() / max(a.norm().item() * b.norm().item(), 1e-30)


def to_np(t):
    return t.detach().float().cpu().numpy()


def bf16_exact(t):
    """float32 numpy copy of a tensor whose values are bf16-representable."""
    return t.detach().to(torch.bfloat16).float().cpu().numpy()
