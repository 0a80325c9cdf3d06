"""Routing kernels on the GPU: bit-exact against CUDA torch (the runtime the
reference trains on) and against the oracle."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import routing as R

pytestmark = pytest.mark.gpu


def _probs(T, E, dtype, seed, bias_std):
    g = torch.Generator(device="cuda").manual_seed(seed)
    logits = torch.randn(T, E, generator=g, device="cuda")
    probs = torch.sigmoid(logits.to(dtype))
    bias = torch.randn(E, generator=g, device="cuda") * bias_std
    return probs, bias


@pytest.mark.parametrize("T,E,k,dtype,bias_std", [
    (16384, 64, 8, torch.bfloat16, 0.1),    # BASELINE config 2 routing
    (16384, 64, 8, torch.bfloat16, 0.0),    # zero bias: ~12% of tokens tie at the k-th value
    (32768, 64, 6, torch.bfloat16, 0.0),    # config 4 shape
    (4096, 128, 8, torch.bfloat16, 0.05),   # config 5 shape
    (1024, 8, 2, torch.float32, 0.0),       # config 1 shape
    (777, 9, 3, torch.float16, 0.02),
    (64, 1024, 32, torch.bfloat16, 0.0),    # largest supported
    (1, 4, 4, torch.float32, 0.0),
])
def test_gate_topk_matches_cuda_torch(T, E, k, dtype, bias_std):
    from modeling.moe_gate import gate_topk

    probs, bias = _probs(T, E, dtype, 1234 + E + k, bias_std)
    idx, w = gate_topk(probs, bias, k)
    ref_idx = torch.topk(probs + bias, k=k, dim=-1, sorted=False)[1]
    assert torch.equal(idx, ref_idx), (idx != ref_idx).any(1).float().mean().item()
    ref_w = F.normalize(probs.gather(-1, ref_idx), p=1, dim=-1)
    assert torch.equal(w, ref_w), (w.float() - ref_w.float()).abs().max().item()
    o_idx, o_w = R.gate_topk(probs.float().cpu().numpy(), bias.cpu().numpy(), k,
                             dtype={torch.bfloat16: "bf16", torch.float16: "f16", torch.float32: "f32"}[dtype])
    assert np.array_equal(idx.cpu().numpy(), o_idx)


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-5), (torch.bfloat16, 2e-2)])
def test_gate_module_gradient_matches_reference_formula(dtype, tol):
    from modeling.moe_gate import GateTopK

    probs, bias = _probs(512, 64, dtype, 7, 0.1)
    p1 = probs.clone().requires_grad_(True)
    idx, w = GateTopK.apply(p1, bias, 8)
    gw = torch.randn_like(w)
    (w.float() * gw.float()).sum().backward()
    p2 = probs.clone().requires_grad_(True)
    ref_idx = torch.topk(p2 + bias, k=8, dim=-1, sorted=False)[1]
    ref_w = F.normalize(p2.gather(-1, ref_idx), p=1, dim=-1)
    (ref_w.float() * gw.float()).sum().backward()
    torch.testing.assert_close(p1.grad.float(), p2.grad.float(), rtol=tol, atol=tol * 0.1)


@pytest.mark.parametrize("n,E", [(131072, 64), (196608, 64), (262144, 128), (74, 8), (4097, 5), (1, 3)])
def test_flatten_sort_count_exact(n, E):
    from scattermoe.parallel_experts import flatten_sort_count

    g = torch.Generator(device="cuda").manual_seed(n + E)
    w = torch.softmax(torch.randn(E, device="cuda", generator=g) * 2, 0)
    ids = torch.multinomial(w, n, replacement=True, generator=g)
    sei, ssi, off = flatten_sort_count(ids.view(-1, 1), E)
    ref_sei, ref_ssi = torch.sort(ids, stable=True)
    assert torch.equal(sei, ref_sei)
    assert torch.equal(ssi, ref_ssi)
    assert torch.equal(off, torch.bincount(ids, minlength=E).cumsum(0))
    o_sei, o_ssi, o_off = R.flatten_sort_count(ids.cpu().numpy(), E)
    assert np.array_equal(ssi.cpu().numpy(), o_ssi) and np.array_equal(off.cpu().numpy(), o_off)


def test_flatten_sort_count_empty_experts_and_single_expert():
    from scattermoe.parallel_experts import flatten_sort_count

    ids = torch.full((1000, 2), 5, dtype=torch.long, device="cuda")
    sei, ssi, off = flatten_sort_count(ids, 16)
    assert torch.equal(ssi, torch.arange(2000, device="cuda"))
    assert off.tolist() == [0] * 5 + [2000] * 11


def test_bincount_and_bias_update(golden):
    from scattermoe.parallel_experts import compileable_bincount
    from zs_b200 import _lib as Z

    g = torch.Generator(device="cuda").manual_seed(3)
    T, k, E = 4096, 6, 64
    topk = torch.randint(0, E, (T, k), device="cuda", generator=g)
    assert torch.equal(compileable_bincount(topk.flatten(), E), torch.bincount(topk.flatten(), minlength=E))
    valid = (torch.rand(T, device="cuda", generator=g) > 0.3).to(torch.uint8)
    counts = torch.zeros(E, dtype=torch.long, device="cuda")
    Z.check(Z.lib().zs_expert_counts(topk.data_ptr(), valid.data_ptr(), T, k, E, counts.data_ptr(),
                                     Z.stream_of(topk)), "counts")
    ref_counts = torch.bincount(topk[valid.bool()].flatten(), minlength=E)
    assert torch.equal(counts, ref_counts)
    bias = torch.randn(E, device="cuda", generator=g) * 0.01
    ref = bias.clone()
    errors = ref_counts.float().mean() - ref_counts.float()
    ref.add_(1e-3 * torch.sign(errors))
    Z.check(Z.lib().zs_bias_sign_update(counts.data_ptr(), E, 1e-3, bias.data_ptr(), Z.stream_of(bias)), "bias")
    assert torch.equal(bias, ref)
    assert Z.device_error() == 0
