"""Muon / MuonMD optimizers with the Newton-Schulz orthogonalisation on the
B200 tensor cores.

Same public functions and classes as the reference module (optimizer/muon.py):
zeropower_via_newtonschulz5 (:6-32), muon_update (:35-42), adam_update
(:131-136), md_decoupled_step (:398-508), SingleDeviceMuonMD (:511-571) and
SingleDeviceMuonMDWithAuxAdam (:574-653), with the same arguments, state
layout and defaults.  zeropower_via_newtonschulz5 runs in libzs.so (three
batched tcgen05 GEMMs per iteration with the linear combinations fused into
their epilogues); the magnitude/direction bookkeeping around it is f32 tensor
arithmetic without host syncs, so a whole step can be captured in a CUDA graph.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from zs_b200 import _lib as Z

NS_COEFFS = (3.4445, -4.7750, 2.0315)
_RAW_GAIN_INIT = 0.5413248546129181  # softplus^-1(1): every gain starts at exactly 1


def zeropower_via_newtonschulz5(G: torch.Tensor, steps: int) -> torch.Tensor:
    """Quintic Newton-Schulz orthogonalisation of the trailing two dims of G
    (batched over leading dims), in bf16; returns a bf16 tensor of G's shape."""
    assert G.ndim >= 2
    Z.require_cuda(G)
    X = G.bfloat16()
    tall = G.size(-2) > G.size(-1)
    if tall:
        X = X.mT
    shape = X.shape
    m, n = shape[-2], shape[-1]
    Xc = X.reshape(-1, m, n)
    # Zero rows and columns stay zero through the iteration and change neither
    # X X^T's live block nor the Frobenius norm, so padding to the kernels'
    # 8-element granularity is exact.
    mp, np_ = -(-m // 8) * 8, -(-n // 8) * 8
    if (mp, np_) != (m, n):
        Xc = torch.nn.functional.pad(Xc, (0, np_ - n, 0, mp - m))
    Xc = Xc.contiguous()
    batch = Xc.size(0)
    out = torch.empty_like(Xc)
    ws = torch.empty(int(Z.lib().zs_newton_schulz5_workspace(batch, mp, np_, Z.ZS_BF16)), dtype=torch.uint8,
                     device=G.device)
    a, b, c = NS_COEFFS
    Z.count(1 + 3 * int(steps))
    with Z.timed("newton_schulz5"):
        Z.check(Z.lib().zs_newton_schulz5(Xc.data_ptr(), out.data_ptr(), batch, mp, np_, int(steps), a, b, c,
                                          ws.data_ptr(), ws.numel(), Z.ZS_BF16, Z.stream_of(Xc)),
                "zs_newton_schulz5")
    if (mp, np_) != (m, n):
        out = out[:, :m, :n]
    out = out.reshape(shape)
    return out.mT if tall else out


def muon_update(grad, momentum, beta=0.95, ns_steps=5, nesterov=True):
    momentum.lerp_(grad, 1 - beta)
    update = grad.lerp_(momentum, beta) if nesterov else momentum
    if update.ndim == 4:
        update = update.view(len(update), -1)
    update = zeropower_via_newtonschulz5(update, steps=ns_steps)
    update *= max(1, grad.size(-2) / grad.size(-1)) ** 0.5
    return update


def adam_update(grad, buf1, buf2, step, betas, eps):
    buf1.lerp_(grad, 1 - betas[0])
    buf2.lerp_(grad.square(), 1 - betas[1])
    c1 = buf1 / (1 - betas[0] ** step)
    c2 = buf2 / (1 - betas[1] ** step)
    return c1 / (c2.sqrt() + eps)


def _scaled_add_(dst, src, lr):
    """dst -= lr * src for a float or a 0-dim tensor lr."""
    if torch.is_tensor(lr):
        dst.sub_(lr * src)
    else:
        dst.add_(src, alpha=-lr)


def _softplus_gains(state):
    """softplus of each raw gain present, as (scalar, row, col) broadcastable views."""
    sc = F.softplus(state["g_scalar"]) if "g_scalar" in state else None
    rw = F.softplus(state["g_row"]) if "g_row" in state else None
    cl = F.softplus(state["g_col"]) if "g_col" in state else None
    return ((sc.reshape(sc.shape + (1, 1)) if sc is not None else None),
            (rw.unsqueeze(-1) if rw is not None else None),
            (cl.unsqueeze(-2) if cl is not None else None))


def _gain_product(parts):
    g = None
    for t in parts:
        if t is not None:
            g = t if g is None else g * t
    return g


def _effective_gain(state):
    return _gain_product(_softplus_gains(state))


def _direction_norm(W, norm_axis):
    if norm_axis == "frobenius":
        return W.norm(dim=(-2, -1), keepdim=True)
    if norm_axis == "row":
        return W.norm(dim=-1, keepdim=True)
    if norm_axis == "col":
        return W.norm(dim=-2, keepdim=True)
    raise ValueError(f"unknown norm_axis {norm_axis!r}")


def _project_to_sphere(W_hat, target_norm, norm_axis):
    return W_hat * (target_norm / (_direction_norm(W_hat, norm_axis) + 1e-12))


def _init_md_state(state, W, gain_mode, norm_axis, capturable):
    *lead, m, n = W.shape
    lead = tuple(lead)
    if gain_mode not in ("none", "scalar", "row", "col", "both"):
        raise ValueError(f"unknown gain_mode {gain_mode!r}")
    state["momentum_buffer"] = torch.zeros_like(W)
    if gain_mode == "scalar":
        state["g_scalar"] = W.new_full(lead, _RAW_GAIN_INIT)
    if gain_mode in ("row", "both"):
        state["g_row"] = W.new_full(lead + (m,), _RAW_GAIN_INIT)
    if gain_mode in ("col", "both"):
        state["g_col"] = W.new_full(lead + (n,), _RAW_GAIN_INIT)
    for key in ("g_scalar", "g_row", "g_col"):
        if key in state:
            state[key + "_m1"] = torch.zeros_like(state[key])
            state[key + "_m2"] = torch.zeros_like(state[key])
    state["gain_step"] = W.new_zeros(()) if capturable else 0
    state["target_norm"] = _direction_norm(W, norm_axis)


@torch.no_grad()
def md_decoupled_step(p, grad, state, *, lr, momentum, gain_lr, gain_betas, gain_eps, gain_mode, norm_axis,
                      ns_steps, capturable=False, rescale_mode="balanced"):
    """One magnitude/direction-decoupled Muon step on p (a matrix or a stack of
    matrices over leading dims), in place; f32 bookkeeping, p's dtype on write."""
    W = p.float()
    G = grad.float()
    m, n = W.shape[-2], W.shape[-1]
    if len(state) == 0:
        _init_md_state(state, W, gain_mode, norm_axis, capturable)
    sc, rw, cl = _softplus_gains(state)
    g = _gain_product((sc, rw, cl))
    W_hat = W if g is None else W / g
    G_hat = G if g is None else g * G
    buf = state["momentum_buffer"]
    buf.lerp_(G_hat, 1 - momentum)
    update = zeropower_via_newtonschulz5(G_hat.lerp(buf, momentum), steps=ns_steps).float()
    update.mul_((max(1.0, m / n) ** 0.5) if rescale_mode == "muon" else (max(m, n) / min(m, n)) ** 0.5)
    W_hat = _project_to_sphere(W_hat - lr * update, state["target_norm"], norm_axis)
    if g is not None:
        # gain gradients from the old gains: reduce (W_hat_old * G) times the
        # other gains over the axes each gain does not span, through softplus
        WG = (W / g) * G
        state["gain_step"] += 1
        step = state["gain_step"]
        grads = {}
        if sc is not None:
            grads["g_scalar"] = (WG * _gain_product((rw, cl)) if (rw is not None or cl is not None) else WG).sum(
                dim=(-2, -1)) * torch.sigmoid(state["g_scalar"])
        if rw is not None:
            other = _gain_product((cl, sc))
            grads["g_row"] = (WG * other if other is not None else WG).sum(dim=-1) * torch.sigmoid(state["g_row"])
        if cl is not None:
            other = _gain_product((rw, sc))
            grads["g_col"] = (WG * other if other is not None else WG).sum(dim=-2) * torch.sigmoid(state["g_col"])
        for key in ("g_scalar", "g_row", "g_col"):
            if key in grads:
                upd = adam_update(grads[key], state[key + "_m1"], state[key + "_m2"], step, gain_betas, gain_eps)
                _scaled_add_(state[key], upd, gain_lr)
    g_new = _effective_gain(state)
    p.copy_((W_hat if g_new is None else g_new * W_hat).to(p.dtype))


_MD_KEYS = {"params", "lr", "momentum", "gain_lr", "gain_betas", "gain_eps", "gain_mode", "norm_axis", "ns_steps",
            "capturable", "rescale_mode"}


class SingleDeviceMuonMD(torch.optim.Optimizer):
    def __init__(self, params, lr=0.02, momentum=0.95, gain_lr=1e-3, gain_betas=(0.9, 0.95), gain_eps=1e-10,
                 gain_mode="both", norm_axis="frobenius", ns_steps=5, capturable=False, rescale_mode="balanced"):
        super().__init__(params, dict(lr=lr, momentum=momentum, gain_lr=gain_lr, gain_betas=gain_betas,
                                      gain_eps=gain_eps, gain_mode=gain_mode, norm_axis=norm_axis,
                                      ns_steps=ns_steps, capturable=capturable, rescale_mode=rescale_mode))

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for group in self.param_groups:
            for p in group["params"]:
                if p.grad is None:
                    continue
                assert p.ndim >= 2, "MD decoupling needs a matrix or a stack of matrices (>=2D)"
                md_decoupled_step(p, p.grad, self.state[p], **{k: group[k] for k in _MD_KEYS if k != "params"})
        return loss


class SingleDeviceMuonMDWithAuxAdam(torch.optim.Optimizer):
    """MuonMD for groups with use_muon=True, AdamW (decoupled weight decay) for the rest."""

    def __init__(self, param_groups):
        for group in param_groups:
            assert "use_muon" in group
            if group["use_muon"]:
                for k, v in dict(lr=0.02, momentum=0.95, gain_lr=1e-3, gain_betas=(0.9, 0.95), gain_eps=1e-10,
                                 gain_mode="both", norm_axis="frobenius", ns_steps=5, capturable=False,
                                 rescale_mode="balanced").items():
                    group.setdefault(k, v)
                assert set(group.keys()) == _MD_KEYS | {"use_muon"}
            else:
                for k, v in dict(lr=3e-4, betas=(0.9, 0.95), eps=1e-10, weight_decay=0, capturable=False).items():
                    group.setdefault(k, v)
                assert set(group.keys()) == {"params", "lr", "betas", "eps", "weight_decay", "capturable", "use_muon"}
        super().__init__(param_groups, dict())

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for group in self.param_groups:
            for p in group["params"]:
                if p.grad is None:
                    continue
                if group["use_muon"]:
                    md_decoupled_step(p, p.grad, self.state[p], **{k: group[k] for k in _MD_KEYS if k != "params"})
                    continue
                state = self.state[p]
                if len(state) == 0:
                    state["exp_avg"] = torch.zeros_like(p)
                    state["exp_avg_sq"] = torch.zeros_like(p)
                    state["step"] = (torch.zeros((), dtype=torch.float32, device=p.device) if group["capturable"]
                                     else 0)
                state["step"] += 1
                update = adam_update(p.grad, state["exp_avg"], state["exp_avg_sq"], state["step"], group["betas"],
                                     group["eps"])
                p.mul_(1 - group["lr"] * group["weight_decay"])
                _scaled_add_(p, update, group["lr"])
        return loss
