"""tcgen05 grouped expert GEMMs and the scattermoe drop-in on the GPU, against
the CPU oracle (small sizes) and a per-expert torch f32 computation (BASELINE
config 2 sizes).  bf16 tolerance: relative L2 error <= 1e-2 per output and
per-parameter gradient cosine >= 0.999."""
import numpy as np
import pytest
import torch

from _util import bf16_exact, cosine, rel_err, to_np
from oracle import routing as R
from oracle import scattermoe as S

pytestmark = pytest.mark.gpu
BF = torch.bfloat16
TOL = 1e-2


def _route(T, E, k, g, skew=0.0):
    logits = torch.randn(T, E, device="cuda", generator=g) + skew * torch.randn(E, device="cuda", generator=g)
    idx = torch.topk(logits, k, dim=-1).indices
    p = torch.softmax(torch.randn(T, k, device="cuda", generator=g), -1)
    return idx, p


def _sort(idx, E):
    from scattermoe.parallel_experts import flatten_sort_count

    return flatten_sort_count(idx, E)


@pytest.mark.parametrize("T,d,E,k,N", [(45, 64, 6, 3, 80), (300, 256, 8, 2, 384), (1000, 512, 16, 4, 256),
                                       (513, 192, 64, 8, 320), (1, 64, 4, 2, 64)])
@pytest.mark.parametrize("x_grouped,y_grouped", [(False, True), (False, False), (True, True), (True, False)])
def test_scatter2scatter_kmajor_weight(T, d, E, k, N, x_grouped, y_grouped):
    from scattermoe.kernels import ops

    g = torch.Generator(device="cuda").manual_seed(T * 7 + N)
    idx, _ = _route(T, E, k, g, skew=1.0)
    sei, ssi, off = _sort(idx, E)
    Wt = (torch.randn(E, N, d, device="cuda", generator=g) * 0.05).to(BF)   # weight [E, out, in]
    rows = T * k if x_grouped else T
    fan = 1 if x_grouped else k
    X = torch.randn(rows, d, device="cuda", generator=g).to(BF)
    out = ops.scatter2scatter(X, Wt.permute(0, 2, 1), sei, ssi, fan, x_grouped=x_grouped, y_grouped=y_grouped)
    ref = S.scatter2scatter(bf16_exact(X), np.transpose(bf16_exact(Wt), (0, 2, 1)), sei.cpu().numpy(),
                            ssi.cpu().numpy(), fan, x_grouped=x_grouped, y_grouped=y_grouped)
    assert rel_err(out, ref) < TOL


@pytest.mark.parametrize("T,d,E,k,N", [(45, 80, 6, 3, 64), (700, 256, 8, 2, 512), (333, 1024, 64, 8, 512)])
def test_scatter2scatter_mn_major_weight(T, d, E, k, N):
    """W = weight [E, K, N] with N contiguous, as the input-gradient GEMM uses it."""
    from scattermoe.kernels import ops

    g = torch.Generator(device="cuda").manual_seed(T + d)
    idx, _ = _route(T, E, k, g)
    sei, ssi, off = _sort(idx, E)
    W = (torch.randn(E, d, N, device="cuda", generator=g) * 0.05).to(BF)
    X = torch.randn(T * k, d, device="cuda", generator=g).to(BF)
    out = ops.scatter2scatter(X, W, sei, ssi, 1, x_grouped=True, y_grouped=False)
    ref = S.scatter2scatter(bf16_exact(X), bf16_exact(W), sei.cpu().numpy(), ssi.cpu().numpy(), 1, x_grouped=True)
    assert rel_err(out, ref) < TOL


def test_scatter2scatter_bias(golden):
    from scattermoe.kernels import ops

    gd = golden("ops_f32")
    k = int(gd["k"])
    dev = "cuda"
    X = torch.tensor(gd["X"], device=dev)
    Wt = torch.tensor(gd["Wt"], device=dev)
    sei = torch.tensor(gd["sorted_expert_idxs"], device=dev)
    ssi = torch.tensor(gd["sorted_scattered_idxs"], device=dev)
    b = torch.tensor(gd["bias"], device=dev)
    out = ops.scatter2scatter(X.to(BF), Wt.to(BF).permute(0, 2, 1), sei, ssi, k, b=b.to(BF), y_grouped=True)
    assert rel_err(out, gd["s2s_bias"]) < TOL
    # f32 operands go through the bf16 contraction and keep their dtype
    out32 = ops.scatter2scatter(X, Wt.permute(0, 2, 1), sei, ssi, k, x_grouped=False, y_grouped=False)
    assert out32.dtype == torch.float32 and rel_err(out32, gd["s2s_xg0_yg0"]) < TOL


@pytest.mark.parametrize("n_per,E,K,N,empty", [(40, 6, 64, 80, False), (300, 8, 256, 512, True),
                                               (2048, 4, 1024, 1024, False), (70, 64, 512, 1024, True)])
def test_group_xty(n_per, E, K, N, empty):
    from scattermoe.kernels import ops

    g = torch.Generator(device="cuda").manual_seed(E * K + N)
    counts = torch.randint(0, 2 * n_per, (E,), device="cuda", generator=g)
    if empty:
        counts[::3] = 0
    off = counts.cumsum(0)
    n = int(off[-1])
    DY = torch.randn(n, N, device="cuda", generator=g).to(BF)
    X = torch.randn(n, K, device="cuda", generator=g).to(BF)
    DW, Db = ops.group_bwd_W(DY, X, off, E, has_bias=True)
    ref = S.group_xty(bf16_exact(DY), bf16_exact(X), off.cpu().numpy(), E)
    assert rel_err(DW, ref) < TOL
    for e in range(E):
        if counts[e] == 0:
            assert DW[e].abs().max().item() == 0
        else:
            assert cosine(DW[e], ref[e]) > 0.999
    assert rel_err(Db, S.group_bias(bf16_exact(DY), off.cpu().numpy(), E)) < TOL


def test_group_and_rowwise(golden):
    from scattermoe.kernels import ops

    gd = golden("ops_f32")
    k = int(gd["k"])
    X = torch.tensor(gd["X"], device="cuda")
    ssi = torch.tensor(gd["sorted_scattered_idxs"], device="cuda")
    p = torch.tensor(gd["p"], device="cuda")
    assert torch.equal(ops.group(X, ssi, fan_out=k).cpu(), torch.tensor(gd["group"]))
    np.testing.assert_allclose(to_np(ops.group(X, ssi, fan_out=k, coeff=p.flatten())), gd["group_coeff"], rtol=1e-6)
    Xb = X.to(BF)
    np.testing.assert_array_equal(to_np(ops.group(Xb, ssi, fan_out=k, coeff=p.flatten().to(BF))),
                                  R.round_bf16(bf16_exact(Xb)[ssi.cpu().numpy() // k] *
                                               bf16_exact(p.flatten())[ssi.cpu().numpy()][:, None]))
    A3 = torch.tensor(gd["A3"], device="cuda")
    B2 = torch.tensor(gd["B2"], device="cuda")
    np.testing.assert_allclose(to_np(ops.rowwise_sum_product(A3, B2)), gd["rsp"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(to_np(ops.rowwise_sum_product(A3.to(BF), B2.to(BF), dtype=torch.float32)),
                               S.rowwise_sum_product(bf16_exact(A3), bf16_exact(B2)), rtol=1e-4, atol=1e-4)


def _glu_case(T, d, E, k, f, seed, dtype=BF, skew=1.0):
    from scattermoe.mlp import GLUMLP

    g = torch.Generator(device="cuda").manual_seed(seed)
    m = GLUMLP(d, f, E, k).cuda()
    with torch.no_grad():
        m.experts.weight.copy_(torch.randn(E, 2 * f, d, device="cuda", generator=g) * 0.02)
        m.output_experts.weight.copy_(torch.randn(E, d, f, device="cuda", generator=g) * 0.02)
    m = m.to(dtype)
    idx, p = _route(T, E, k, g, skew=skew)
    x = torch.randn(T, d, device="cuda", generator=g).to(dtype).requires_grad_(True)
    p = p.to(dtype).requires_grad_(True)
    dy = torch.randn(T, d, device="cuda", generator=g).to(dtype)
    return m, x, p, idx, dy


@pytest.mark.parametrize("T,d,E,k,f", [(33, 64, 4, 2, 32), (257, 256, 8, 2, 192), (1024, 1024, 64, 8, 512)])
def test_glumlp_fused_matches_oracle(T, d, E, k, f):
    m, x, p, idx, dy = _glu_case(T, d, E, k, f, seed=T + f)
    y = m(x, p, idx)
    y.backward(dy)
    W1, W2 = bf16_exact(m.experts.weight), bf16_exact(m.output_experts.weight)
    ry, saved = S.glu_mlp_forward(bf16_exact(x), bf16_exact(p), idx.cpu().numpy(), W1, W2, dtype="bf16")
    dx, dp, dW1, dW2 = S.glu_mlp_backward(bf16_exact(dy), bf16_exact(x), bf16_exact(p), W1, W2, saved, dtype="bf16")
    assert rel_err(y, ry) < TOL
    assert rel_err(x.grad, dx) < TOL and cosine(x.grad, dx) > 0.999
    assert rel_err(p.grad, dp) < TOL and cosine(p.grad, dp) > 0.999
    assert cosine(m.experts.weight.grad, dW1) > 0.999 and rel_err(m.experts.weight.grad, dW1) < TOL
    assert cosine(m.output_experts.weight.grad, dW2) > 0.999 and rel_err(m.output_experts.weight.grad, dW2) < TOL


def test_glumlp_fused_equals_op_level_path():
    """The fused GLUMLP autograd function and the reference-structured path
    through ParallelExperts / ParallelLinear give the same results."""
    m, x, p, idx, dy = _glu_case(600, 256, 16, 4, 128, seed=5)
    y1 = m(x, p, idx)
    y1.backward(dy)
    g1 = [x.grad.clone(), p.grad.clone(), m.experts.weight.grad.clone(), m.output_experts.weight.grad.clone()]
    for t in (x, p, m.experts.weight, m.output_experts.weight):
        t.grad = None
    m._fused_ok = lambda: False
    y2 = m(x, p, idx)
    y2.backward(dy)
    g2 = [x.grad, p.grad, m.experts.weight.grad, m.output_experts.weight.grad]
    assert rel_err(y1, y2) < TOL
    for a, b in zip(g1, g2):
        assert cosine(a, b) > 0.999 and rel_err(a, b) < TOL


def test_glumlp_golden_fixture(golden):
    """Reference outputs (f32, Triton interpreter) vs the bf16 kernels."""
    from scattermoe.mlp import GLUMLP

    gd = golden("glu_e8")
    E, f2, d = gd["W1"].shape
    k = int(gd["k"])
    m = GLUMLP(d, f2 // 2, E, k).cuda()
    with torch.no_grad():
        m.experts.weight.copy_(torch.tensor(gd["W1"]))
        m.output_experts.weight.copy_(torch.tensor(gd["W2"]))
    x = torch.tensor(gd["x"], device="cuda", requires_grad=True)
    p = torch.tensor(gd["expert_p"], device="cuda", requires_grad=True)
    y = m(x, p, torch.tensor(gd["expert_idxs"], device="cuda"))
    y.backward(torch.tensor(gd["dy"], device="cuda"))
    assert y.dtype == torch.float32
    assert rel_err(y, gd["y"]) < 2e-2
    for got, ref in ((x.grad, gd["dx"]), (p.grad, gd["dp"]), (m.experts.weight.grad, gd["dW1"]),
                     (m.output_experts.weight.grad, gd["dW2"])):
        assert cosine(got, ref) > 0.999


def test_glumlp_config2_full_size():
    """BASELINE config 2 shapes: 16384 tokens, d 1024, 64 experts, f 512,
    top-8, skewed loads.  Checked per expert against torch f32 on the GPU."""
    T, d, E, k, f = 16384, 1024, 64, 8, 512
    m, x, p, idx, dy = _glu_case(T, d, E, k, f, seed=2, skew=0.5)
    y = m(x, p, idx)
    y.backward(dy)
    W1 = m.experts.weight.detach().float()
    W2 = m.output_experts.weight.detach().float()
    xf, pf, dyf = x.detach().float(), p.detach().float(), dy.float()
    # f32 reference with autograd
    xr = xf.clone().requires_grad_(True)
    pr = pf.clone().requires_grad_(True)
    W1r = W1.clone().requires_grad_(True)
    W2r = W2.clone().requires_grad_(True)
    yr = torch.zeros(T, d, device="cuda")
    flat = idx.flatten()
    for e in range(E):
        sel = (flat == e).nonzero().flatten()
        if sel.numel() == 0:
            continue
        t, j = sel // k, sel % k
        hfull = xr[t] @ W1r[e].T
        h, gt = hfull[:, :f], hfull[:, f:]
        a = torch.nn.functional.silu(gt) * h
        yr = yr.index_add(0, t, (a @ W2r[e].T) * pr[t, j][:, None])
    yr.backward(dyf)
    assert rel_err(y, yr) < TOL
    assert cosine(x.grad, xr.grad) > 0.999 and rel_err(x.grad, xr.grad) < TOL
    assert cosine(p.grad, pr.grad) > 0.999
    assert cosine(m.experts.weight.grad, W1r.grad) > 0.999
    assert cosine(m.output_experts.weight.grad, W2r.grad) > 0.999
    from zs_b200 import device_error
    assert device_error() == 0


@pytest.mark.parametrize("n_per,E,d,f", [(50, 6, 64, 48), (700, 8, 256, 192), (2000, 64, 1024, 512)])
def test_up_swiglu_and_down_dswiglu_kernels(n_per, E, d, f):
    """The fused-epilogue GEMMs against the oracle's SwiGLU forward/backward."""
    from scattermoe.mlp import down_dswiglu, up_swiglu

    g = torch.Generator(device="cuda").manual_seed(n_per + f)
    counts = torch.randint(0, 2 * n_per, (E,), device="cuda", generator=g)
    counts[1] = 0
    off = counts.cumsum(0)
    n = int(off[-1])
    sei = torch.repeat_interleave(torch.arange(E, device="cuda"), counts)
    xg = torch.randn(n, d, device="cuda", generator=g).to(BF)
    W1 = (torch.randn(E, 2 * f, d, device="cuda", generator=g) * 0.05).to(BF)
    W2 = (torch.randn(E, d, f, device="cuda", generator=g) * 0.05).to(BF)
    act, hfull = up_swiglu(xg, W1, sei, off)
    hf_ref = np.zeros((n, 2 * f))
    sei_np = sei.cpu().numpy()
    xg_np, W1_np, W2_np = bf16_exact(xg), bf16_exact(W1), bf16_exact(W2)
    for e in range(E):
        m = sei_np == e
        hf_ref[m] = xg_np[m].astype(np.float64) @ W1_np[e].T.astype(np.float64)
    assert rel_err(hfull, hf_ref) < TOL
    hf = hfull.float().cpu().numpy().astype(np.float64)
    h, gt = hf[:, :f], hf[:, f:]
    act_ref = h * gt / (1 + np.exp(-gt))
    assert rel_err(act, act_ref) < TOL
    dyg = torch.randn(n, d, device="cuda", generator=g).to(BF)
    dh = down_dswiglu(dyg, W2, hfull, sei, off)
    dyg_np = bf16_exact(dyg).astype(np.float64)
    dact = np.zeros((n, f))
    for e in range(E):
        m = sei_np == e
        dact[m] = dyg_np[m] @ W2_np[e].astype(np.float64)
    sg = 1 / (1 + np.exp(-gt))
    ref = np.concatenate([dact * gt * sg, dact * h * sg * (1 + gt * (1 - sg))], axis=1)
    assert rel_err(dh, ref) < TOL
    from zs_b200 import device_error
    assert device_error() == 0


@pytest.mark.parametrize("set_to_none,wdtype", [(True, torch.float32), (False, torch.float32),
                                                (True, torch.bfloat16), (False, torch.bfloat16)])
def test_glumlp_fused_weight_grad_accumulation(set_to_none, wdtype):
    """fuse_weight_grad: the f32 expert grads come straight from the GEMM epilogue into .grad
    (accumulated over two backward passes) and equal the unfused bf16-dW-then-cast path to
    bf16 rounding of dW; the input and gate gradients are unchanged."""
    from scattermoe.mlp import GLUMLP

    torch.manual_seed(0)
    T, d, E, k, f = 1000, 256, 16, 4, 192
    ref = GLUMLP(d, f, E, k).cuda()
    fus = GLUMLP(d, f, E, k).cuda()
    fus.load_state_dict(ref.state_dict())
    ref, fus = ref.to(wdtype), fus.to(wdtype)
    fus.fuse_weight_grad = True
    x = torch.randn(T, d, device="cuda")
    logits = torch.randn(T, E, device="cuda")
    p, idx = torch.topk(torch.softmax(logits, -1), k)
    for m in (ref, fus):
        for prm in m.parameters():
            prm.grad = None if set_to_none else torch.full_like(prm, 0.25)
    outs = []
    for m in (ref, fus):
        xs, ps = x.clone().requires_grad_(True), p.clone().requires_grad_(True)
        for rep in range(2):
            with torch.autocast("cuda", dtype=torch.bfloat16):
                y = m(xs, ps, idx)
            (y.float() * torch.linspace(-1, 1, d, device="cuda")).sum().backward()
        outs.append((xs.grad, ps.grad))
    for a, b in ((ref.experts.weight, fus.experts.weight), (ref.output_experts.weight, fus.output_experts.weight)):
        assert b.grad.dtype == wdtype and b.grad.is_contiguous()
        assert rel_err(b.grad, a.grad) < 5e-3 and cosine(b.grad, a.grad) > 0.99999
    assert rel_err(outs[1][0], outs[0][0]) < 1e-6 and rel_err(outs[1][1], outs[0][1]) < 1e-6


@pytest.mark.parametrize("T,k,C", [(1000, 8, 1024), (257, 3, 72), (64, 1, 40)])
def test_gathered_row_sum(T, k, C):
    """out[t] = sum_j rows[pos[t*k + j]] (the expert-parallel combine): bit-exact against
    the f32 sum in slot order rounded once; a row index out of range contributes zero
    and is recorded as ZS_DEVERR_INDEX."""
    from scattermoe.expert_parallel import _slot_sum
    from zs_b200 import _lib as Z
    from zs_b200 import clear_device_error, device_error

    g = torch.Generator(device="cuda").manual_seed(T + C)
    n = T * k
    rows = torch.randn(n, C, device="cuda", generator=g).bfloat16()
    ssi = torch.randperm(n, device="cuda", generator=g)
    out = _slot_sum(rows, ssi, T, k)
    pos = torch.empty_like(ssi)
    pos[ssi] = torch.arange(n, device="cuda")
    acc = torch.zeros(T, C, device="cuda")
    for j in range(k):
        acc = acc + rows[pos.view(T, k)[:, j]].float()
    assert torch.equal(out, acc.bfloat16())
    assert device_error() == 0
    bad = pos.clone()
    bad[0] = n + 5
    out2 = torch.empty(T, C, device="cuda", dtype=torch.bfloat16)
    Z.check(Z.lib().zs_gathered_row_sum(out2.data_ptr(), C, rows.data_ptr(), C, n, bad.data_ptr(), T, k, C,
                                        Z.ZS_BF16, torch.cuda.current_stream().cuda_stream), "zs_gathered_row_sum")
    torch.cuda.synchronize()
    ref0 = torch.zeros(C, device="cuda")
    for j in range(1, k):
        ref0 = ref0 + rows[pos[j]].float()
    assert torch.equal(out2[0], ref0.bfloat16()) and torch.equal(out2[1:], out[1:])
    assert device_error() & 0x10
    clear_device_error()
