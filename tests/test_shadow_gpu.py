"""bf16 weight shadows (zs_b200.shadow): the optimizer kernels keep them equal to the bf16
rounding of the f32 weights they write, every reader refreshes a shadow whose weight
changed through torch ops, concatenated shadows are row slices of one buffer, and a
recorded optimizer step is recorded again when a shadow appears after the recording."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _params():
    torch.manual_seed(0)
    mats = [torch.nn.Parameter(torch.randn(*s, device="cuda") * 0.05)
            for s in [(4, 256, 512), (512, 256), (384, 384), (64, 256)]]
    vecs = [torch.nn.Parameter(torch.randn(300, 64, device="cuda") * 0.05),
            torch.nn.Parameter(torch.randn(77, device="cuda"))]
    return mats, vecs


def test_optimizer_kernels_write_shadows_equal_to_weight_rounding():
    from optimizer.muon import SingleDeviceMuonMDWithAuxAdam
    from zs_b200.shadow import bf16_shadow, concat_shadow

    mats, vecs = _params()
    lr = torch.tensor(0.02, device="cuda")
    opt = SingleDeviceMuonMDWithAuxAdam([
        dict(params=mats, use_muon=True, lr=lr, momentum=0.95, gain_lr=1e-3, capturable=True),
        dict(params=vecs, use_muon=False, lr=torch.tensor(3e-4, device="cuda"), weight_decay=0.1, capturable=True)])
    shadows = [bf16_shadow(p) for p in mats[:2] + mats[3:] + vecs]
    cat = concat_shadow([mats[2]], pad=16)   # a concatenated buffer (one weight and zero rows)
    for _ in range(3):
        for p in mats + vecs:
            p.grad = torch.randn_like(p)
        opt.step()
    torch.cuda.synchronize()
    for p, sh in zip(mats[:2] + mats[3:] + vecs, shadows):
        assert bf16_shadow(p) is sh                      # still valid: no re-cast
        assert torch.equal(sh, p.detach().bfloat16())
    assert torch.equal(cat[:384], mats[2].detach().bfloat16()) and torch.all(cat[384:] == 0)
    assert concat_shadow([mats[2]], pad=16) is cat


def test_torch_inplace_change_refreshes_shadow():
    from zs_b200.shadow import bf16_shadow, concat_shadow

    p = torch.nn.Parameter(torch.randn(128, 64, device="cuda"))
    q = torch.nn.Parameter(torch.randn(32, 64, device="cuda"))
    sh = bf16_shadow(p)
    buf = concat_shadow([p, q], pad=0)
    with torch.no_grad():
        p.mul_(2.0)
        q.add_(1.0)
    assert torch.equal(bf16_shadow(p), p.detach().bfloat16())
    buf2 = concat_shadow([p, q], pad=0)
    assert buf2 is buf and torch.equal(buf2, torch.cat([p, q]).detach().bfloat16())
    assert sh.dtype == torch.bfloat16


def test_graph_recorded_step_is_recorded_again_for_a_new_shadow():
    from optimizer.hybrid import HybridGraphOptimizer
    from optimizer.muon import SingleDeviceMuonMDWithAuxAdam
    from engram.GramReaperSparse import GramReaperSparse
    from zs_b200.shadow import bf16_shadow

    mats, _ = _params()
    emb = torch.nn.Parameter(torch.nn.functional.normalize(torch.randn(50, 16, device="cuda"), dim=1))
    dense = SingleDeviceMuonMDWithAuxAdam([dict(params=mats, use_muon=True, lr=torch.tensor(0.02, device="cuda"),
                                                momentum=0.95, gain_lr=1e-3, capturable=True)])
    sparse = GramReaperSparse([dict(params=[emb], unit_norm=True)], lr=1e-2, beta=0.9, unit_norm=True)
    opt = HybridGraphOptimizer(dense, sparse, capture_warmup_steps=1)
    sh = None
    for step in range(4):
        for p in mats:
            p.grad = torch.randn_like(p)
        if step == 2:
            sh = bf16_shadow(mats[0])     # appears after the step was recorded (step 1)
        opt.step()
    torch.cuda.synchronize()
    assert torch.equal(sh, mats[0].detach().bfloat16())
