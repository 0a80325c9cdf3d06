"""Fixed workloads for capturing single kernels under a profiler (one process, one GPU):

    python architecture-zarelga-superposition_b200/zs_b200/profile_workloads.py attention
    python architecture-zarelga-superposition_b200/zs_b200/profile_workloads.py muonmd

attention: config 4's attention shape (B=8, S=4096, H=12, Hkv=4, hd=128, causal, sink key),
two warm-up forward+backward passes, then one more.
muonmd:    one md_decoupled_step on config 4's W1 expert stack [64, 1536, 1536] f32 (gain
mode "both", Frobenius sphere) after one warm-up step.
"""
from __future__ import annotations

import sys
from pathlib import Path

_PKG = Path(__file__).resolve().parents[1]
if str(_PKG) not in sys.path:
    sys.path.insert(0, str(_PKG))

import torch  # noqa: E402


def attention(passes: int = 3) -> None:
    from zs_b200.attn import attention as attn

    B, S, H, Hkv, hd = 8, 4096, 12, 4, 128
    g = torch.Generator(device="cuda").manual_seed(0)
    q = torch.randn(B, S, H, hd, device="cuda", generator=g).bfloat16().requires_grad_(True)
    k = torch.randn(B, S, Hkv, hd, device="cuda", generator=g).bfloat16().requires_grad_(True)
    v = torch.randn(B, S, Hkv, hd, device="cuda", generator=g).bfloat16().requires_grad_(True)
    ks = (torch.randn(H, hd, device="cuda", generator=g) * 0.5).requires_grad_(True)
    do = torch.randn(B, S, H, hd, device="cuda", generator=g).bfloat16()
    for _ in range(passes):
        o = attn(q, k, v, k_sink=ks)
        torch.autograd.grad(o, (q, k, v, ks), do)
    torch.cuda.synchronize()


def muonmd(passes: int = 2) -> None:
    from optimizer.muon import md_decoupled_step

    p = torch.randn(64, 1536, 1536, device="cuda") * 0.02
    state = {}
    lr = torch.tensor(0.02, device="cuda")
    for _ in range(passes):
        md_decoupled_step(p, torch.randn_like(p), state, lr=lr, momentum=0.95, gain_lr=1e-3,
                          gain_betas=(0.9, 0.95), gain_eps=1e-10, gain_mode="both", norm_axis="frobenius",
                          ns_steps=5, capturable=True, rescale_mode="balanced")
    torch.cuda.synchronize()


if __name__ == "__main__":
    which = sys.argv[1] if len(sys.argv) > 1 else "attention"
    {"attention": attention, "muonmd": muonmd}[which]()
    print("ok")
