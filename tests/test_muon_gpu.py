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
