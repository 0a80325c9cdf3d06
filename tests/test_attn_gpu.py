"""tcgen05 flash attention (zs_attention_forward / zs_attention_backward)
against the float64 oracle on the same bf16 inputs: causal, window, GQA,
packed sequences with padding, the sink key, head_dim 64 and 128, ragged
sequence lengths; then the model shape (cfg4: B=2 of S=4096, H=12, Hkv=4,
hd=128) against PyTorch SDPA on the GPU.

Tolerances: the kernel keeps P and dS in bf16 for the tensor-core products
(as flash-attn does), so outputs are compared by relative Frobenius error
(forward < 1e-2, gradients < 3e-2) and cosine (> 0.9995 / > 0.999)."""
import math

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from _util import cosine, rel_err
from oracle import attention as A

pytestmark = pytest.mark.gpu

CASES = [
    # B, S, H, Hkv, hd, window, packed, sink, q_gain
    (2, 300, 4, 2, 64, 0, False, None, 1.0),
    (1, 512, 4, 4, 128, 0, False, None, 1.0),
    (2, 256, 6, 2, 128, 100, False, None, 1.0),
    (2, 333, 4, 1, 64, 0, True, torch.float32, 1.0),
    (1, 200, 2, 2, 128, 37, True, torch.bfloat16, 1.0),
    (1, 640, 4, 2, 128, 0, False, torch.float32, 4.0),   # large logits: lazy rescale path
    (3, 130, 2, 1, 64, 64, False, None, 4.0),
]


def _inputs(B, S, H, Hkv, hd, packed, sink, gain, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = (torch.randn(B, S, H, hd, device="cuda", generator=g) * gain).bfloat16()
    k = torch.randn(B, S, Hkv, hd, device="cuda", generator=g).bfloat16()
    v = torch.randn(B, S, Hkv, hd, device="cuda", generator=g).bfloat16()
    do = torch.randn(B, S, H, hd, device="cuda", generator=g).bfloat16()
    ks = (torch.randn(H, hd, device="cuda", generator=g) * 0.5).to(sink) if sink is not None else None
    seq_ids = None
    if packed:
        seq_ids = torch.full((B, S), -1, dtype=torch.long, device="cuda")
        for b in range(B):
            # ragged documents back to back, then padding
            cuts = [0, S // 5, S // 5 + 7, S // 2 + 3, S - 11 - b]
            for i in range(len(cuts) - 1):
                seq_ids[b, cuts[i]:cuts[i + 1]] = 10 * b + i
    return q, k, v, do, ks, seq_ids


@pytest.mark.parametrize("case", CASES, ids=lambda c: "-".join(str(x) for x in c))
def test_attention_matches_oracle(case):
    from zs_b200 import _lib as Z
    from zs_b200.attn import attention, seg_start_from_seq_ids

    B, S, H, Hkv, hd, window, packed, sink, gain = case
    q, k, v, do, ks, seq_ids = _inputs(B, S, H, Hkv, hd, packed, sink, gain, seed=S + hd)
    Z.clear_device_error()
    qr, kr, vr = (t.clone().requires_grad_(True) for t in (q, k, v))
    ksr = ks.clone().requires_grad_(True) if ks is not None else None
    o = attention(qr, kr, vr, window=window or None, seq_ids=seq_ids, k_sink=ksr)
    o.backward(do)
    torch.cuda.synchronize()
    assert Z.device_error() == 0

    npf = lambda t: t.detach().float().cpu().numpy()
    seg = seg_start_from_seq_ids(seq_ids).cpu().numpy() if seq_ids is not None else None
    ks_np = npf(ks) if ks is not None else None
    ro, _ = A.attention_forward(npf(q), npf(k), npf(v), window=window, seg_start=seg, k_sink=ks_np)
    dq, dk, dv, dks = A.attention_backward(npf(do), npf(q), npf(k), npf(v), window=window, seg_start=seg,
                                           k_sink=ks_np)
    assert rel_err(o, ro) < 1e-2 and cosine(o, ro) > 0.9995
    for got, ref in ((qr.grad, dq), (kr.grad, dk), (vr.grad, dv)):
        assert rel_err(got, ref) < 3e-2 and cosine(got, ref) > 0.999
    if ks is not None:
        assert ksr.grad.dtype == ks.dtype
        assert rel_err(ksr.grad, dks) < 3e-2 and cosine(ksr.grad, dks) > 0.999
    if seq_ids is not None:
        pad = (seq_ids < 0).cpu()
        assert torch.all(o.detach().cpu()[pad] == 0)


def test_attention_lse_matches_oracle():
    from zs_b200 import _lib as Z

    B, S, H, Hkv, hd = 2, 257, 4, 2, 128
    q, k, v, _, ks, _ = _inputs(B, S, H, Hkv, hd, False, torch.float32, 2.0, seed=3)
    o = torch.empty_like(q)
    lse = torch.empty(B, H, S, device="cuda")
    Z.check(Z.lib().zs_attention_forward(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(),
                                         B, S, H, Hkv, hd, 0, None, ks.data_ptr(), Z.ZS_F32, 1 / math.sqrt(hd),
                                         torch.cuda.current_stream().cuda_stream), "fwd")
    torch.cuda.synchronize()
    npf = lambda t: t.detach().float().cpu().numpy()
    _, rl = A.attention_forward(npf(q), npf(k), npf(v), k_sink=npf(ks))
    np.testing.assert_allclose(lse.cpu().numpy(), rl, atol=2e-2, rtol=0)


def test_attention_model_shape_vs_sdpa():
    """cfg4 attention shape against PyTorch SDPA (bf16 inputs, causal, GQA)."""
    from zs_b200 import _lib as Z
    from zs_b200.attn import attention

    B, S, H, Hkv, hd = 2, 4096, 12, 4, 128
    q, k, v, do, _, _ = _inputs(B, S, H, Hkv, hd, False, None, 1.0, seed=4)
    Z.clear_device_error()
    qa, ka, va = (t.clone().requires_grad_(True) for t in (q, k, v))
    o = attention(qa, ka, va)
    o.backward(do)
    qb, kb, vb = (t.clone().requires_grad_(True) for t in (q, k, v))
    ref = F.scaled_dot_product_attention(qb.transpose(1, 2), kb.transpose(1, 2), vb.transpose(1, 2),
                                         is_causal=True, enable_gqa=True).transpose(1, 2)
    ref.backward(do)
    torch.cuda.synchronize()
    assert Z.device_error() == 0
    assert rel_err(o, ref) < 1e-2 and cosine(o, ref) > 0.9995
    for a, b in ((qa.grad, qb.grad), (ka.grad, kb.grad), (va.grad, vb.grad)):
        assert rel_err(a, b) < 3e-2 and cosine(a, b) > 0.999


def test_attention_rejects_unsupported():
    from zs_b200 import _lib as Z
    from zs_b200.attn import attention

    q = torch.zeros(1, 8, 2, 32, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(Z.ZsError):
        attention(q, q, q)
    q = torch.zeros(1, 8, 2, 64, device="cuda", dtype=torch.float32)
    with pytest.raises(Z.ZsError):
        attention(q, q, q)
    with pytest.raises(Z.ZsError):
        attention(q.cpu(), q.cpu(), q.cpu())
