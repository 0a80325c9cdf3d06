"""Dense projections on the grouped GEMM (zs_b200.dense) against f32 PyTorch:
the concatenated q/k/v/head-gate product with zero padding columns, the output
projection, and the shared expert's fused SwiGLU MLP, forward and every
gradient, at row counts that are and are not tile multiples."""
import pytest
import torch
import torch.nn.functional as F

from _util import cosine, rel_err

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("T", [4096, 1000])
def test_dense_linear_concat_pad_matches_torch(T):
    from zs_b200.dense import dense_linear

    torch.manual_seed(0)
    d, qd, kd, H = 512, 512, 128, 8
    x = torch.randn(2, T // 2, d, device="cuda").bfloat16().requires_grad_(True)
    ws = [(torch.randn(n, d, device="cuda") * d ** -0.5).requires_grad_(True) for n in (qd, kd, kd, H)]
    pad = -(qd + 2 * kd + H) % 16
    y = dense_linear(x, ws, tag="proj_test", pad=pad)
    assert y.shape == (2, T // 2, qd + 2 * kd + H + pad) and y.dtype == torch.bfloat16
    assert torch.all(y[..., qd + 2 * kd + H:] == 0)
    xr = x.detach().float().requires_grad_(True)
    wr = [w.detach().bfloat16().float().requires_grad_(True) for w in ws]
    yr = xr @ torch.cat(wr, 0).T
    assert rel_err(y[..., :yr.size(-1)], yr) < 1e-2
    dy = torch.randn_like(yr)
    y[..., :yr.size(-1)].float().backward(dy)
    yr.backward(dy)
    assert cosine(x.grad, xr.grad) > 0.9999
    for w, r in zip(ws, wr):
        assert w.grad.dtype == torch.float32
        assert cosine(w.grad, r.grad) > 0.9999 and rel_err(w.grad, r.grad) < 1e-2


def test_dense_swiglu_matches_torch():
    from zs_b200.dense import dense_swiglu

    torch.manual_seed(1)
    T, d, f = 3000, 512, 384
    x = torch.randn(T, d, device="cuda").bfloat16().requires_grad_(True)
    wg, wu = [(torch.randn(f, d, device="cuda") * 0.05).requires_grad_(True) for _ in range(2)]
    wd = (torch.randn(d, f, device="cuda") * 0.05).requires_grad_(True)
    y = dense_swiglu(x, wg, wu, wd)
    xr = x.detach().float().requires_grad_(True)
    rs = [w.detach().bfloat16().float().requires_grad_(True) for w in (wg, wu, wd)]
    yr = (F.silu(xr @ rs[0].T) * (xr @ rs[1].T)) @ rs[2].T
    assert rel_err(y, yr) < 1e-2
    dy = torch.randn_like(yr)
    y.float().backward(dy)
    yr.backward(dy)
    assert cosine(x.grad, xr.grad) > 0.999
    for w, r in zip((wg, wu, wd), rs):
        assert cosine(w.grad, r.grad) > 0.999, (cosine(w.grad, r.grad))
