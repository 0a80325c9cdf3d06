"""Fixed workloads for capturing single kernels under a profiler (one process, one GPU):

    python architecture-zarelga-superposition_b200/zs_b200/profile_workloads.py attention
    python architecture-zarelga-superposition_b200/zs_b200/profile_workloads.py muonmd

attention: config 4's attention shape (B=8, S=4096, H=12, Hkv=4, hd=128, causal, sink key),
two warm-up forward+backward passes, then one more.
muonmd:    one md_decoupled_step on config 4's W1 expert stack [64, 1536, 1536] f32 (gain
mode "both", Frobenius sphere) after one warm-up step.
norm_rope: zRMSNorm forward + backward on config 4's residual rows [32768, 1536] f32, the
           fused residual add + zRMSNorm (bf16 branch, bf16 output) forward + backward, and
           partial RoPE forward + backward on q [8, 4096, 12, 128] / k [8, 4096, 4, 128] bf16
           (8 of 64 pairs rotated, config 4's pos_rope_dims = 16), two warm-up passes, then one more.
routing:   config 2 routing: sigmoid + biased top-8 of [16384, 64] bf16 probabilities,
           flatten_sort_count, the gate backward; two warm-ups, then one more.
xent:      config 3 cut cross entropy, forward + backward (hidden [16384, 2048], classifier
           [131072, 2048] bf16, 5 % ignored targets); one warm-up, then one more.
newton_schulz: zeropower_via_newtonschulz5 on config 4's W1 expert stack [64, 1536, 1536] and
           W2 stack [64, 1536, 768] (bf16); one warm-up, then one more.
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


def norm_rope(passes: int = 3) -> None:
    from modeling.liger_rope import PartialRopeFunction
    from modeling.zRMSNorm import AddZRMSNormFunction, ZRMSNormFunction

    g = torch.Generator(device="cuda").manual_seed(1)
    x = torch.randn(32768, 1536, device="cuda", generator=g).requires_grad_(True)
    w = (torch.randn(1536, device="cuda", generator=g) * 0.1).requires_grad_(True)
    dy = torch.randn(32768, 1536, device="cuda", generator=g)
    q = torch.randn(8, 4096, 12, 128, device="cuda", generator=g).bfloat16()
    k = torch.randn(8, 4096, 4, 128, device="cuda", generator=g).bfloat16()
    # config 4 keeps ModelConfig's pos_rope_dims = 16: the first 8 of 64 pairs rotate
    ang = torch.arange(4096, device="cuda", dtype=torch.float32)[:, None] * torch.logspace(0, -4, 8, device="cuda")
    cos, sin = ang.cos().expand(8, 4096, 8).contiguous(), ang.sin().expand(8, 4096, 8).contiguous()
    br = torch.randn(32768, 1536, device="cuda", generator=g).bfloat16().requires_grad_(True)
    dyb = dy.bfloat16()
    for _ in range(passes):
        y = ZRMSNormFunction.apply(x, w, 1e-6)
        torch.autograd.grad(y, (x, w), dy)
        # the block's fused residual add + norm with a bf16 output (f32 stream, bf16 branch)
        h, yb = AddZRMSNormFunction.apply(x, br, w, 1e-6)
        torch.autograd.grad((h, yb), (x, br, w), (dy, dyb))
        qq, kk = q.clone().requires_grad_(True), k.clone().requires_grad_(True)
        qo, ko = PartialRopeFunction.apply(qq * 1, kk * 1, cos, sin, 8)
        torch.autograd.grad((qo, ko), (qq, kk), (torch.ones_like(qo), torch.ones_like(ko)))
    torch.cuda.synchronize()


def routing(passes: int = 3) -> None:
    from modeling.moe_gate import GateTopK
    from scattermoe.parallel_experts import flatten_sort_count

    g = torch.Generator(device="cuda").manual_seed(2)
    logits = torch.randn(16384, 64, device="cuda", generator=g).bfloat16().requires_grad_(True)
    bias = torch.randn(64, device="cuda", generator=g) * 0.1
    for _ in range(passes):
        idx, w = GateTopK.apply(torch.sigmoid(logits), bias, 8)
        flatten_sort_count(idx, 64)
        torch.autograd.grad(w, logits, torch.ones_like(w))
    torch.cuda.synchronize()


def xent(passes: int = 2) -> None:
    from cut_cross_entropy import linear_cross_entropy

    g = torch.Generator(device="cuda").manual_seed(3)
    h = torch.randn(16384, 2048, device="cuda", generator=g).bfloat16().requires_grad_(True)
    c = (torch.randn(131072, 2048, device="cuda", generator=g) * 0.02).bfloat16().requires_grad_(True)
    t = torch.randint(0, 131072, (16384,), device="cuda", generator=g)
    t[torch.rand(16384, device="cuda", generator=g) < 0.05] = -100
    for _ in range(passes):
        loss = linear_cross_entropy(h, c, t, ignore_index=-100)
        torch.autograd.grad(loss, (h, c))
    torch.cuda.synchronize()


def newton_schulz(passes: int = 2) -> None:
    from optimizer.muon import zeropower_via_newtonschulz5

    g = torch.Generator(device="cuda").manual_seed(4)
    a = torch.randn(64, 1536, 1536, device="cuda", generator=g).bfloat16()
    b = torch.randn(64, 1536, 768, device="cuda", generator=g).bfloat16()
    for _ in range(passes):
        zeropower_via_newtonschulz5(a, 5)
        zeropower_via_newtonschulz5(b, 5)
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
    {"attention": attention, "muonmd": muonmd, "attention_timing": attention_timing, "norm_rope": norm_rope,
     "routing": routing, "xent": xent, "newton_schulz": newton_schulz}[which]()
    print("ok")
