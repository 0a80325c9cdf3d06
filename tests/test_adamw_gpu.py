"""The fused AdamW step (zs_adamw_step) against the reference's tensor formulation
(optimizer/muon.py:131-136 adam_update, :616-650 the aux-Adam group of
SingleDeviceMuonMDWithAuxAdam) run with torch ops on the same GPU: device step and
learning rate (the capturable groups the trainer builds), host step and learning
rate, weight decay on and off, sizes that are and are not multiples of the vector
width, more tensors than one launch takes, parameters without a gradient, and the
optional bf16 copy of the new weights."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _torch_adamw(ps, grads, states, lr, betas, eps, wd, capturable):
    from optimizer.muon import _scaled_add_, adam_update

    for p, g in zip(ps, grads):
        st = states.setdefault(p, {})
        if not st:
            st["exp_avg"] = torch.zeros_like(p)
            st["exp_avg_sq"] = torch.zeros_like(p)
            st["step"] = torch.zeros((), device=p.device) if capturable else 0
        st["step"] += 1
        u = adam_update(g, st["exp_avg"], st["exp_avg_sq"], st["step"], betas, eps)
        p.mul_(1 - lr * wd)
        _scaled_add_(p, u, lr)


@pytest.mark.parametrize("capturable", [True, False])
@pytest.mark.parametrize("wd", [0.0, 0.1])
def test_fused_adamw_matches_torch_formulation(capturable, wd):
    from optimizer.muon import _adam_steps

    torch.manual_seed(0)
    sizes = [1, 3, 5, 8, 1536, 4097, 12345, 65536 * 3 + 7] + [17] * 100   # > 96 tensors: two launches
    ps = [torch.randn(n, device="cuda") for n in sizes]
    ref = [p.clone() for p in ps]
    lr = torch.tensor(3e-4, device="cuda") if capturable else 3e-4
    betas, eps = (0.9, 0.95), 1e-16
    group = dict(params=ps, lr=lr, betas=betas, eps=eps, weight_decay=wd)
    states, rstates = {}, {}
    for step in range(4):
        grads = [torch.randn_like(p) * (10.0 ** (step - 2)) for p in ps]
        for p, g in zip(ps, grads):
            p.grad = g.clone()
        _adam_steps(group, states, capturable=capturable)
        _torch_adamw(ref, grads, rstates, lr, betas, eps, wd, capturable)
        if capturable:
            lr.mul_(0.5)   # a scheduler update read by the next launch
    torch.cuda.synchronize()
    worst = max(float(((a - b).abs() / (b.abs() + 1e-30)).max()) for a, b in zip(ps, ref))
    assert worst < 1e-6, worst
    for p, r in zip(ps, ref):
        st, rs = states[p], rstates[r]
        torch.testing.assert_close(st["exp_avg"], rs["exp_avg"], rtol=1e-6, atol=0)
        torch.testing.assert_close(st["exp_avg_sq"], rs["exp_avg_sq"], rtol=1e-6, atol=0)
        assert float(st["step"]) == float(rs["step"]) == 4


def test_fused_adamw_writes_bf16_shadow_and_skips_gradless_params():
    from optimizer.muon import SingleDeviceMuonMDWithAuxAdam
    from zs_b200 import _lib as Z

    torch.manual_seed(1)
    a = torch.nn.Parameter(torch.randn(1000, 24, device="cuda"))
    b = torch.nn.Parameter(torch.randn(77, device="cuda"))
    opt = SingleDeviceMuonMDWithAuxAdam([dict(params=[a, b], use_muon=False, lr=1e-2, capturable=True)])
    a.grad = torch.randn_like(a)
    before_b = b.detach().clone()
    opt.step()
    assert torch.equal(b, before_b) and len(opt.state[b]) == 0
    assert float(opt.state[a]["step"]) == 1
    # the kernel's optional bf16 copy of the updated weights
    p = torch.randn(4099, device="cuda")
    g, m1, m2 = torch.randn_like(p), torch.zeros_like(p), torch.zeros_like(p)
    shadow = torch.empty(4099, dtype=torch.bfloat16, device="cuda")
    d = Z.AdamWTensor()
    d.p, d.g, d.m1, d.m2, d.step_dev = p.data_ptr(), g.data_ptr(), m1.data_ptr(), m2.data_ptr(), None
    d.inv_bc1_host, d.inv_bc2_host, d.shadow_bf16, d.n = 10.0, 20.0, shadow.data_ptr(), p.numel()
    arr = (Z.AdamWTensor * 1)(d)
    Z.check(Z.lib().zs_adamw_step(arr, 1, None, 1e-3, 1.0, 0.9, 0.95, 0.1, 0.05, 1e-8, 0.0, None), "zs_adamw_step")
    torch.cuda.synchronize()
    assert torch.equal(shadow, p.bfloat16())
