"""zRMSNorm and RoPE kernels on the GPU: reference fixtures, oracle, and the
reference's torch formulation at model sizes (f32 exactness; bf16 within one
bf16 ulp-level relative error)."""
import numpy as np
import pytest
import torch

from _util import bf16_exact, cosine, rel_err
from oracle import attention as A

pytestmark = pytest.mark.gpu


def _torch_zrms(x, w, eps):
    xf = x.float()
    out = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (out * (1.0 + w.float())).to(x.dtype)


@pytest.mark.parametrize("case", ["zrms_d64", "zrms_d256"])
def test_zrmsnorm_fixture(golden, case):
    from modeling.zRMSNorm import ZeroCenteredRMSNorm

    g = golden(case)
    d = g["x"].shape[1]
    m = ZeroCenteredRMSNorm(d).cuda()
    with torch.no_grad():
        m.weight.copy_(torch.tensor(g["w"]))
    x = torch.tensor(g["x"], device="cuda", requires_grad=True)
    y = m(x)
    y.backward(torch.tensor(g["dy"], device="cuda"))
    np.testing.assert_allclose(y.detach().cpu().numpy(), g["y"], rtol=2e-6, atol=2e-6)
    np.testing.assert_allclose(x.grad.cpu().numpy(), g["dx"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(m.weight.grad.cpu().numpy(), g["dw"], rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("shape,dtype", [((32768, 1536), torch.float32), ((32768, 1536), torch.bfloat16),
                                         ((8, 4096, 12, 128), torch.bfloat16), ((3, 5, 2048), torch.float16),
                                         ((1, 7), torch.float32)])
def test_zrmsnorm_matches_reference_formula(shape, dtype):
    from modeling.zRMSNorm import ZeroCenteredRMSNorm

    d = shape[-1]
    g = torch.Generator(device="cuda").manual_seed(d)
    m = ZeroCenteredRMSNorm(d).cuda()
    with torch.no_grad():
        m.weight.copy_(torch.randn(d, device="cuda", generator=g) * 0.1)
    x0 = (torch.randn(*shape, device="cuda", generator=g) * 3).to(dtype)
    x1 = x0.clone().requires_grad_(True)
    y = m(x1)
    dy = torch.randn(*shape, device="cuda", generator=g).to(dtype)
    y.backward(dy)
    w2 = m.weight.detach().clone().requires_grad_(True)
    x2 = x0.clone().requires_grad_(True)
    y2 = _torch_zrms(x2, w2, 1e-6)
    y2.backward(dy)
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    assert y.dtype == dtype and rel_err(y, y2) < tol
    assert rel_err(x1.grad, x2.grad) < tol and cosine(x1.grad, x2.grad) > 0.9999
    assert rel_err(m.weight.grad, w2.grad) < max(tol, 1e-4)


@pytest.mark.parametrize("B,S,Hq,Hk,hd,dtype,pairs", [(8, 4096, 12, 4, 128, torch.bfloat16, 32),
                                                      (4, 256, 4, 4, 64, torch.float32, 16),
                                                      (2, 11, 4, 2, 64, torch.bfloat16, 0)])
def test_rope_forward_backward(B, S, Hq, Hk, hd, dtype, pairs):
    from modeling.liger_rope import LigerRopeFunction

    g = torch.Generator(device="cuda").manual_seed(S)
    cos_t, sin_t = A.rope_tables(S + 5, hd, 10000.0, 2 * pairs)
    pos = torch.randint(0, S + 5, (B, S), device="cuda", generator=g)
    cos = torch.tensor(cos_t, device="cuda")[pos]
    sin = torch.tensor(sin_t, device="cuda")[pos]
    q = torch.randn(B, S, Hq, hd, device="cuda", generator=g).to(dtype)
    k = torch.randn(B, S, Hk, hd, device="cuda", generator=g).to(dtype)
    q_np, k_np = q.float().cpu().numpy(), k.float().cpu().numpy()
    qo, ko = LigerRopeFunction.apply(q, k, cos, sin, cos, sin)
    rq = A.rope(q_np, cos.cpu().numpy(), sin.cpu().numpy())
    rk = A.rope(k_np, cos.cpu().numpy(), sin.cpu().numpy())
    tol = 1e-6 if dtype == torch.float32 else 5e-3
    assert rel_err(qo, rq) < tol and rel_err(ko, rk) < tol
    if pairs == 0:
        assert torch.equal(qo.cpu(), torch.tensor(q_np).to(dtype))
    # backward is the inverse rotation
    from modeling.liger_rope import rope_backward
    dq, dk = rope_backward(qo.clone(), ko.clone(), cos, sin, cos, sin)
    assert rel_err(dq, q_np) < 2 * tol and rel_err(dk, k_np) < 2 * tol


def test_rope_reference_fixture(golden):
    from modeling.liger_rope import LigerRopeFunction, rope_backward

    gd = golden("rope")
    pos = torch.tensor(gd["pos"], device="cuda")
    cos = torch.tensor(gd["cos_table"], device="cuda")[pos]
    sin = torch.tensor(gd["sin_table"], device="cuda")[pos]
    q = torch.tensor(gd["q"], device="cuda")
    k = torch.tensor(gd["k"], device="cuda")
    qo, ko = LigerRopeFunction.apply(q, k, cos, sin, cos, sin)
    np.testing.assert_allclose(qo.cpu().numpy(), gd["q_out"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(ko.cpu().numpy(), gd["k_out"], rtol=1e-5, atol=1e-6)
    dq, dk = rope_backward(torch.tensor(gd["dq"], device="cuda"), torch.tensor(gd["dk"], device="cuda"), cos, sin, cos,
                           sin)
    np.testing.assert_allclose(dq.cpu().numpy(), gd["dq_out"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(dk.cpu().numpy(), gd["dk_out"], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("rot", [8, 16, 32, 64])
def test_partial_rope_equals_full_rope_with_identity_tail(rot):
    """PartialRopeFunction (rotates the first `rot` pairs only) gives bit-identical
    outputs and gradients to LigerRopeFunction on tables whose pairs beyond `rot` are
    the identity (cos 1, sin 0), as GatedAttention builds them."""
    from modeling.liger_rope import LigerRopeFunction, PartialRopeFunction

    g = torch.Generator(device="cuda").manual_seed(rot)
    B, S, H, Hk, hd = 2, 96, 6, 2, 128
    q = torch.randn(B, S, H, hd, device="cuda", generator=g).bfloat16()
    k = torch.randn(B, S, Hk, hd, device="cuda", generator=g).bfloat16()
    ang = torch.rand(B, S, rot, device="cuda", generator=g) * 6.0
    cos_full = torch.ones(B, S, hd // 2, device="cuda")
    sin_full = torch.zeros(B, S, hd // 2, device="cuda")
    cos_full[..., :rot], sin_full[..., :rot] = ang.cos(), ang.sin()
    dq = torch.randn_like(q)
    dk = torch.randn_like(k)
    outs = []
    for partial in (False, True):
        qq, kk = q.clone().requires_grad_(True), k.clone().requires_grad_(True)
        if partial:
            a, b = PartialRopeFunction.apply(qq * 1, kk * 1, ang.cos(), ang.sin(), rot)
        else:
            a, b = LigerRopeFunction.apply(qq * 1, kk * 1, cos_full, sin_full, cos_full, sin_full)
        # the backward rotates the incoming gradients in place: give each run its own copy
        gq, gk = torch.autograd.grad((a, b), (qq, kk), (dq.clone(), dk.clone()))
        outs.append((a.detach(), b.detach(), gq, gk))
    for x, y in zip(*outs):
        assert torch.equal(x, y)
