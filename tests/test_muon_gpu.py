"""Newton-Schulz on the tensor cores and the MuonMD step on the GPU, against
the reference's CPU fixtures, the oracle, and the reference formula in torch
bf16 on the GPU (cfg 4 expert-stack shapes).  bf16 tolerance (five chained bf16 iterations): relative error
<= 5e-2 and cosine >= 0.999 on the orthogonalised update; parameters after a
MuonMD steps within 5e-3 relative, update direction cosine >= 0.998."""
import numpy as np
import pytest
import torch

from _util import cosine, rel_err
from oracle import muon as M

pytestmark = pytest.mark.gpu


def _torch_ns5(G, steps=5):
    a, b, c = (3.4445, -4.7750, 2.0315)
    X = G.bfloat16()
    tall = G.size(-2) > G.size(-1)
    if tall:
        X = X.mT
    X = X / (X.norm(dim=(-2, -1), keepdim=True) + 1e-7)
    for _ in range(steps):
        A = X @ X.mT
        B = b * A + c * A @ A
        X = a * X + B @ X
    return X.mT if tall else X


def test_ns5_reference_fixture(golden):
    from optimizer.muon import zeropower_via_newtonschulz5

    g = golden("ns5")
    for G, X in ((g["G_wide"], g["X_wide"]), (g["G_tall"], g["X_tall"])):
        out = zeropower_via_newtonschulz5(torch.tensor(G, device="cuda"), 5)
        assert out.dtype == torch.bfloat16 and tuple(out.shape) == X.shape
        assert cosine(out, X) > 0.999 and rel_err(out, X) < 5e-2


@pytest.mark.parametrize("shape", [(64, 1536, 1536), (64, 1536, 768), (1536, 1536), (64, 1536), (12, 256, 512),
                                   (3, 8, 16), (12, 1536), (5, 37, 20), (1, 1, 9)])
def test_ns5_matches_torch_formula(shape):
    from optimizer.muon import zeropower_via_newtonschulz5

    g = torch.Generator(device="cuda").manual_seed(sum(shape))
    G = torch.randn(*shape, device="cuda", generator=g)
    out = zeropower_via_newtonschulz5(G, 5)
    ref = _torch_ns5(G, 5)
    assert out.shape == G.shape
    assert cosine(out, ref) > 0.999 and rel_err(out, ref) < 5e-2
    if G.numel() < 200000:
        o = M.newton_schulz5(G.cpu().numpy(), 5)
        assert cosine(out, o) > 0.999


@pytest.mark.parametrize("case,gain_mode,norm_axis,rescale", [
    ("md_both_frobenius", "both", "frobenius", "balanced"), ("md_col_row", "col", "row", "muon"),
    ("md_scalar_frobenius", "scalar", "frobenius", "balanced"), ("md_none_col", "none", "col", "balanced")])
def test_md_decoupled_step_reference_fixture(golden, case, gain_mode, norm_axis, rescale):
    from optimizer.muon import md_decoupled_step

    gd = golden(case)
    p = torch.tensor(gd["W0"], device="cuda")
    state = {}
    for key in ("grad0", "grad1"):
        md_decoupled_step(p, torch.tensor(gd[key], device="cuda"), state, lr=0.02, momentum=0.95, gain_lr=1e-3,
                          gain_betas=(0.9, 0.95), gain_eps=1e-10, gain_mode=gain_mode, norm_axis=norm_axis,
                          ns_steps=5, rescale_mode=rescale)
    # two steps of lr 0.02 with a bf16 orthogonalised update (~5e-2 relative
    # apart from the reference's bf16 CPU run) move p by ~4e-2; 5e-3 bounds it
    assert rel_err(p, gd["W2"]) < 5e-3
    w0 = torch.tensor(gd["W0"], device="cuda")
    assert cosine(p - w0, torch.tensor(gd["W2"], device="cuda") - w0) > 0.998
    assert rel_err(state["momentum_buffer"], gd["momentum"]) < 1e-5
    for key in ("g_scalar", "g_row", "g_col"):
        if key in gd:
            assert rel_err(state[key], gd[key]) < 1e-3


def _torch_md_step(p, grad, state, *, lr, momentum, gain_lr, gain_betas, gain_eps, gain_mode, norm_axis, ns_steps,
                   capturable=False, rescale_mode="balanced", U=None, X_fused=None):
    """optimizer/muon.py:398-508 restated with torch f32 ops on the GPU.  With U given, that
    orthogonalised update replaces the Newton-Schulz call (so both sides share it); with
    X_fused given, the restatement's own Newton-Schulz input is checked against it."""
    import torch.nn.functional as F
    from optimizer.muon import _direction_norm, _init_md_state, zeropower_via_newtonschulz5

    def eff(st):
        g = None
        if "g_scalar" in st:
            gs = F.softplus(st["g_scalar"])
            g = gs.reshape(gs.shape + (1, 1))
        if "g_row" in st:
            gr = F.softplus(st["g_row"]).unsqueeze(-1)
            g = gr if g is None else g * gr
        if "g_col" in st:
            gc = F.softplus(st["g_col"]).unsqueeze(-2)
            g = gc if g is None else g * gc
        return g

    def adam(grad, b1, b2, step):
        b1.lerp_(grad, 1 - gain_betas[0])
        b2.lerp_(grad.square(), 1 - gain_betas[1])
        return (b1 / (1 - gain_betas[0] ** step)) / ((b2 / (1 - gain_betas[1] ** step)).sqrt() + gain_eps)

    W, G = p.float(), grad.float()
    m, n = W.shape[-2:]
    if len(state) == 0:
        _init_md_state(state, W, gain_mode, norm_axis, capturable)
    g = eff(state)
    W_hat = W if g is None else W / g
    G_hat = G if g is None else g * G
    WG = None if g is None else W_hat * G
    buf = state["momentum_buffer"]
    buf.lerp_(G_hat, 1 - momentum)
    X = G_hat.lerp(buf, momentum).bfloat16()
    if X_fused is not None:
        # f32 lerps that differ in the last bit (fma contraction) round a few values to the
        # neighbouring bf16 (at most 1e-3 of them); the lerp subtracts values of the
        # momentum's size, so near-zero results carry an absolute f32 error on top
        diff = (X.float() - X_fused.float()).abs()
        assert (X != X_fused).float().mean().item() < 1e-3
        assert (diff <= X.float().abs() * 2 ** -7 + 1e-6 * X.float().abs().max()).all()
    upd = (zeropower_via_newtonschulz5(X, steps=ns_steps) if U is None else U).float()
    upd.mul_((max(1.0, m / n) ** 0.5) if rescale_mode == "muon" else (max(m, n) / min(m, n)) ** 0.5)
    W_hat = W_hat - lr * upd
    W_hat = W_hat * (state["target_norm"] / (_direction_norm(W_hat, norm_axis) + 1e-12))
    if g is not None:
        state["gain_step"] += 1
        step = state["gain_step"]
        sp = {k: F.softplus(state[k]) for k in ("g_scalar", "g_row", "g_col") if k in state}
        sb = {"g_scalar": (lambda t: t.reshape(t.shape + (1, 1))), "g_row": (lambda t: t.unsqueeze(-1)),
              "g_col": (lambda t: t.unsqueeze(-2))}
        grads = {}
        for key, dims in (("g_scalar", (-2, -1)), ("g_row", -1), ("g_col", -2)):
            if key in state:
                red = WG
                for other in ("g_row", "g_col", "g_scalar"):
                    if other != key and other in sp:
                        red = red * sb[other](sp[other])
                grads[key] = red.sum(dim=dims) * torch.sigmoid(state[key])
        for key, gr in grads.items():
            u = adam(gr, state[key + "_m1"], state[key + "_m2"], step)
            state[key].add_(u, alpha=-gain_lr)
    g_new = eff(state)
    p.copy_((W_hat if g_new is None else g_new * W_hat).to(p.dtype))


MD_SHAPES = [(64, 256, 512), (1536, 1536), (12, 1536), (5, 37, 20), (3, 96, 40), (200, 72)]


@pytest.mark.parametrize("shape", MD_SHAPES)
@pytest.mark.parametrize("gain_mode,norm_axis,rescale", [("both", "frobenius", "balanced"), ("col", "row", "muon"),
                                                         ("scalar", "col", "balanced"), ("row", "row", "balanced"),
                                                         ("none", "frobenius", "muon")])
def test_fused_md_step_matches_torch_formula(shape, gain_mode, norm_axis, rescale):
    from optimizer.muon import _md_post, _md_pre, zeropower_via_newtonschulz5

    gen = torch.Generator(device="cuda").manual_seed(len(shape) * 1000 + shape[-1])
    W0 = torch.randn(*shape, device="cuda", generator=gen) * 0.05
    grads = [torch.randn(*shape, device="cuda", generator=gen) for _ in range(3)]
    pa, pb = W0.clone(), W0.clone()
    sa, sb = {}, {}
    lr = torch.tensor(0.02, device="cuda")
    kw = dict(lr=lr, momentum=0.95, gain_lr=1e-2, gain_betas=(0.9, 0.95), gain_eps=1e-10, gain_mode=gain_mode,
              norm_axis=norm_axis, ns_steps=5, capturable=True, rescale_mode=rescale)
    # The bf16 Newton-Schulz amplifies a one-ulp change of a few inputs to ~0.5 % of its
    # output, so both sides share the fused path's orthogonalised update; the
    # restatement's own input is checked against the fused one.  What remains differs by
    # f32 rounding and reduction order only.
    for gr in grads:
        W, red, X = _md_pre(pa, gr, sa, momentum=0.95, gain_mode=gain_mode, norm_axis=norm_axis, capturable=True)
        U = zeropower_via_newtonschulz5(X, 5)
        _md_post(pa, W, red, U, sa, lr=lr, gain_lr=1e-2, gain_betas=(0.9, 0.95), gain_eps=1e-10,
                 norm_axis=norm_axis, rescale_mode=rescale)
        _torch_md_step(pb, gr, sb, U=U, X_fused=X, **kw)
        torch.cuda.synchronize()
        assert rel_err(pa, pb) < 2e-6
    assert rel_err(sa["momentum_buffer"], sb["momentum_buffer"]) < 1e-6
    for key in ("g_scalar", "g_row", "g_col", "g_scalar_m1", "g_row_m2", "g_col_m1"):
        if key in sb:
            assert rel_err(sa[key], sb[key]) < 1e-5, key
    assert float(sa["gain_step"]) == float(sb["gain_step"]) == (0.0 if gain_mode == "none" else 3.0)


def test_fused_md_step_bf16_param_and_float_lr():
    from optimizer.muon import _md_post, _md_pre, md_decoupled_step, zeropower_via_newtonschulz5

    gen = torch.Generator(device="cuda").manual_seed(9)
    W0 = (torch.randn(4, 64, 128, device="cuda", generator=gen) * 0.05).bfloat16()
    pa, pb = W0.clone(), W0.clone()
    sa, sb = {}, {}
    kw = dict(lr=0.01, momentum=0.9, gain_lr=1e-3, gain_betas=(0.9, 0.95), gain_eps=1e-10, gain_mode="both",
              norm_axis="frobenius", ns_steps=5, capturable=False, rescale_mode="balanced")
    for _ in range(2):
        gr = torch.randn(4, 64, 128, device="cuda", generator=gen).bfloat16()
        W, red, X = _md_pre(pa, gr, sa, momentum=0.9, gain_mode="both", norm_axis="frobenius", capturable=False)
        U = zeropower_via_newtonschulz5(X, 5)
        _md_post(pa, W, red, U, sa, lr=0.01, gain_lr=1e-3, gain_betas=(0.9, 0.95), gain_eps=1e-10,
                 norm_axis="frobenius", rescale_mode="balanced")
        _torch_md_step(pb, gr, sb, U=U, **kw)
        # p is stored in bf16 on both sides: agreement to a bf16 rounding of the update
        assert rel_err(pa, pb) < 2e-3
    assert pa.dtype == torch.bfloat16 and sa["gain_step"] == sb["gain_step"] == 2
    md_decoupled_step(pa, gr, sa, **kw)
    assert sa["gain_step"] == 3


def test_batched_optimizer_matches_per_parameter_steps():
    """SingleDeviceMuonMDWithAuxAdam batches Newton-Schulz across same-shape matrices,
    writing each parameter's input into its slice of the batch (transposed for a tall
    stack, partial 64 x 256 tiles included) and reading the update back from there; the
    result equals stepping each parameter alone."""
    from optimizer.muon import SingleDeviceMuonMDWithAuxAdam, md_decoupled_step

    gen = torch.Generator(device="cuda").manual_seed(3)
    shapes = [(256, 512), (256, 512), (512, 256), (4, 256, 512), (64, 512), (12, 128), (200, 72), (3, 96, 40),
              (2, 72, 200), (12, 128), (40, 33), (3, 200, 72)]
    ps = [torch.nn.Parameter(torch.randn(*s, device="cuda", generator=gen) * 0.05) for s in shapes]
    ref = [p.detach().clone() for p in ps]
    lr = torch.tensor(0.02, device="cuda")
    opt = SingleDeviceMuonMDWithAuxAdam([
        dict(params=ps[:9], use_muon=True, lr=lr, momentum=0.95, gain_lr=1e-3, capturable=True),
        dict(params=ps[9:], use_muon=True, lr=lr, momentum=0.95, gain_lr=1e-3, norm_axis="row", gain_mode="col",
             rescale_mode="muon", capturable=True)])
    states = [{} for _ in ps]
    for _ in range(2):
        gs = [torch.randn(*s, device="cuda", generator=gen) for s in shapes]
        for p, g in zip(ps, gs):
            p.grad = g
        opt.step()
        for i, (r, g) in enumerate(zip(ref, gs)):
            group = opt.param_groups[0] if i < 9 else opt.param_groups[1]
            md_decoupled_step(r, g, states[i], lr=lr, momentum=0.95, gain_lr=1e-3, gain_betas=group["gain_betas"],
                              gain_eps=group["gain_eps"], gain_mode=group["gain_mode"], norm_axis=group["norm_axis"],
                              ns_steps=5, capturable=True, rescale_mode=group["rescale_mode"])
    # same kernels, same inputs, Newton-Schulz per matrix independent of the batching (its
    # norm is reduced in a fixed order): equal up to the gain reductions' atomic order
    for p, r in zip(ps, ref):
        assert rel_err(p.detach(), r) < 1e-6


@pytest.mark.parametrize("gain_mode,norm_axis", [("both", "frobenius"), ("col", "row"), ("row", "col"),
                                                 ("scalar", "frobenius")])
def test_md_step_is_deterministic(gain_mode, norm_axis):
    """Two runs of the fused MuonMD step on the same inputs give bit-identical parameters
    and state (fixed-order reductions), which keeps data-parallel replicas in sync."""
    from optimizer.muon import md_decoupled_step

    gen = torch.Generator(device="cuda").manual_seed(17)
    W0 = torch.randn(8, 384, 640, device="cuda", generator=gen) * 0.05
    grads = [torch.randn(8, 384, 640, device="cuda", generator=gen) for _ in range(2)]
    runs = []
    for _ in range(2):
        p, st = W0.clone(), {}
        for gr in grads:
            md_decoupled_step(p, gr.clone(), st, lr=0.02, momentum=0.95, gain_lr=1e-2, gain_betas=(0.9, 0.95),
                              gain_eps=1e-10, gain_mode=gain_mode, norm_axis=norm_axis, ns_steps=5, capturable=True,
                              rescale_mode="balanced")
        torch.cuda.synchronize()
        runs.append((p, st))
    (pa, sa), (pb, sb) = runs
    assert torch.equal(pa, pb)
    for k, v in sa.items():
        if torch.is_tensor(v):
            assert torch.equal(v, sb[k]), k
