"""Fixed workloads for capturing single kernels under a profiler (one process, one GPU):

    python architecture-zarelga-superposition_b200/zs_b200/profile_workloads.py attention
    python architecture-zarelga-superposition_b200/zs_b200/profile_workloads.py muonmd

attention: config 4's attention shape (B=8, S=4096, H=12, Hkv=4, hd=128, causal, sink key),
two warm-up forward+backward passes, then one more.
muonmd:    one md_decoupled_step on config 4's W1 expert stack [64, 1536, 1536] f32 (gain
mode "both", Frobenius sphere) after one warm-up step.
attention_timing: CUDA-event times of the attention forward and forward+backward at the
           same shape (mean of 10 calls after 3 warm-ups), beside torch SDPA (cuDNN and flash
           backends, no sink) and flash_attn when importable; prints one JSON line.
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


def _time(fn, n=10):
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(n):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / n


def attention_timing() -> None:
    import json

    import torch.nn.functional as F
    from zs_b200.attn import attention as attn

    B, S, H, Hkv, hd = 8, 4096, 12, 4, 128
    g = torch.Generator(device="cuda").manual_seed(0)
    q = torch.randn(B, S, H, hd, device="cuda", generator=g).bfloat16().requires_grad_(True)
    k = torch.randn(B, S, Hkv, hd, device="cuda", generator=g).bfloat16().requires_grad_(True)
    v = torch.randn(B, S, Hkv, hd, device="cuda", generator=g).bfloat16().requires_grad_(True)
    ks = (torch.randn(H, hd, device="cuda", generator=g) * 0.5).requires_grad_(True)
    do = torch.randn(B, S, H, hd, device="cuda", generator=g).bfloat16()
    res = {}
    f = _time(lambda: attn(q, k, v, k_sink=ks))
    fb = _time(lambda: torch.autograd.grad(attn(q, k, v, k_sink=ks), (q, k, v, ks), do))
    flops = 4 * B * H * S * S / 2 * hd
    res["zs"] = {"fwd_ms": f, "bwd_ms": fb - f, "fwd_tflops": flops / f / 1e9, "bwd_tflops": 2.5 * flops / (fb - f) / 1e9}
    from torch.nn.attention import SDPBackend, sdpa_kernel

    qt, kt, vt = (t.detach().transpose(1, 2).contiguous().requires_grad_(True) for t in (q, k, v))
    dot = do.transpose(1, 2)
    for name, be in (("sdpa_cudnn", SDPBackend.CUDNN_ATTENTION), ("sdpa_flash", SDPBackend.FLASH_ATTENTION)):
        try:
            with sdpa_kernel([be]):
                fn = lambda: F.scaled_dot_product_attention(qt, kt, vt, is_causal=True, enable_gqa=True)  # noqa: E731
                f = _time(fn)
                fb = _time(lambda: torch.autograd.grad(fn(), (qt, kt, vt), dot))
            res[name] = {"fwd_ms": f, "bwd_ms": fb - f}
        except Exception as e:  # backend unavailable on this build
            res[name] = str(e)[:80]
    try:
        from flash_attn import flash_attn_func

        qf, kf, vf = (t.detach().clone().requires_grad_(True) for t in (q, k, v))
        fn = lambda: flash_attn_func(qf, kf, vf, causal=True)  # noqa: E731
        f = _time(fn)
        fb = _time(lambda: torch.autograd.grad(fn(), (qf, kf, vf), do))
        res["flash_attn"] = {"fwd_ms": f, "bwd_ms": fb - f}
    except Exception as e:
        res["flash_attn"] = str(e)[:80]
    print(json.dumps(res))


if __name__ == "__main__":
    which = sys.argv[1] if len(sys.argv) > 1 else "attention"
    {"attention": attention, "muonmd": muonmd, "attention_timing": attention_timing}[which]()
    print("ok")
