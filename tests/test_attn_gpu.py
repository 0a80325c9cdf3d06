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


GATED_CASES = [
    # hidden, H, Hkv, window, packed, sink, pos_rope_dims
    (256, 4, 4, None, False, False, 32),
    (1536, 12, 4, None, False, True, 16),
    (512, 4, 2, 64, True, False, 16),
    (768, 6, 2, None, True, True, 128),
]


@pytest.mark.parametrize("case", GATED_CASES, ids=lambda c: "-".join(str(x) for x in c))
def test_fused_gated_attention_core_matches_stepwise_path(case):
    """GatedAttention's fused core (q/k norm + RoPE kernel, attention reading v and the gate
    logits in place with the sigmoid gate in its epilogue, the backward writing the
    projection's gradient) against the same module's step-by-step path (split, norms, RoPE,
    attention, torch gate): output, input gradient and every parameter gradient."""
    from modeling.attention import GatedAttention
    from modeling.model_config import ModelConfig
    from zs_b200 import _lib as Z

    hidden, H, Hkv, window, packed, sink, prd = case
    B, S = 2, 384
    cfg = ModelConfig(vocab_size=256, embed_size=hidden, hidden_size=hidden, transformer_depth=1,
                      intermediate_size=64, n_experts=3, n_shared_experts=1, n_experts_per_token=1,
                      n_attention_heads=H, n_key_value_heads=Hkv, attention_window_pattern=(window,),
                      max_position_embeddings=S, sequence_length=S, pos_rope_dims=prd, attention_sink=sink)
    torch.manual_seed(hidden + H)
    m = GatedAttention(cfg, window_size=window).cuda()
    with torch.no_grad():
        m.q_norm.weight.normal_(0, 0.1)
        m.k_norm.weight.normal_(0, 0.1)
        m.head_gate_proj.weight.normal_(0, 0.2)
    x = torch.randn(B, S, hidden, device="cuda")
    cu, unpad = None, None
    if packed:
        lens = [100, 150, 84, 200, 40]   # two rows: 100+150+84 = 334 (+50 pad), 200+40 = 240 (+144 pad)
        starts = [0, 100, 250, S, S + 200]
        unpad = torch.cat([torch.arange(s, s + n) for s, n in zip(starts, lens)]).cuda()
        cu = torch.tensor([0] + list(torch.cumsum(torch.tensor(lens), 0)), dtype=torch.int32, device="cuda")
    dy = torch.randn(B, S, hidden, device="cuda")
    outs = []
    for fused in (True, False):
        m.fused_core = fused
        m.zero_grad(set_to_none=True)
        xi = x.clone().requires_grad_(True)
        Z.clear_device_error()
        with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
            y = m(xi, cu_seqlens=cu, unpad_indices=unpad, max_seqlen=None)
        y.float().backward(dy)
        torch.cuda.synchronize()
        assert Z.device_error() == 0
        outs.append((y.float(), xi.grad, {n: p.grad.float() for n, p in m.named_parameters() if p.grad is not None}))
    (yf, gxf, gpf), (ys, gxs, gps) = outs
    if packed:   # padding positions are not attended to by anything; compare real tokens
        yf, ys = yf.reshape(-1, hidden)[unpad], ys.reshape(-1, hidden)[unpad]
    assert rel_err(yf, ys) < 2e-2 and cosine(yf, ys) > 0.9995
    assert rel_err(gxf, gxs) < 3e-2 and cosine(gxf, gxs) > 0.999
    assert set(gpf) == set(gps)
    for n in gps:
        assert cosine(gpf[n], gps[n]) > 0.999 and rel_err(gpf[n], gps[n]) < 3e-2, n


def test_fused_gated_attention_core_matches_f32_torch():
    """The fused core against an f32 PyTorch restatement of GatedAttention between its
    projections: per-head zero-centred RMSNorm of q and k, partial rotate-half RoPE, causal
    GQA softmax attention, o * sigmoid(gate logits)."""
    from zs_b200.attn import gated_attention_core

    torch.manual_seed(3)
    B, S, H, Hkv, hd, rp = 2, 512, 8, 2, 128, 8
    pad = -((H + 2 * Hkv) * hd + H) % 16
    qkvg = (torch.randn(B, S, (H + 2 * Hkv) * hd + H + pad, device="cuda")).bfloat16()
    qkvg[..., (H + 2 * Hkv) * hd + H:] = 0
    qkvg.requires_grad_(True)
    wq = (torch.randn(hd, device="cuda") * 0.1).requires_grad_(True)
    wk = (torch.randn(hd, device="cuda") * 0.1).requires_grad_(True)
    inv = 1.0 / (10000 ** (torch.arange(0, 2 * rp, 2, device="cuda").float() / (2 * rp)))
    ang = torch.outer(torch.arange(S, device="cuda").float(), inv)
    cos, sin = ang.cos()[None], ang.sin()[None]
    o = gated_attention_core(qkvg, wq, wk, n_heads=H, n_kv_heads=Hkv, head_dim=hd, cos=cos, sin=sin, rot_pairs=rp,
                             eps=1e-6, pad=pad)
    do = torch.randn_like(o)
    o.backward(do)

    xr = qkvg.detach().float().requires_grad_(True)
    wqr, wkr = wq.detach().clone().requires_grad_(True), wk.detach().clone().requires_grad_(True)
    q = xr[..., : H * hd].reshape(B, S, H, hd)
    k = xr[..., H * hd:(H + Hkv) * hd].reshape(B, S, Hkv, hd)
    v = xr[..., (H + Hkv) * hd:(H + 2 * Hkv) * hd].reshape(B, S, Hkv, hd)
    gl = xr[..., (H + 2 * Hkv) * hd:(H + 2 * Hkv) * hd + H]

    def norm(t, w):
        return t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + 1e-6) * (1 + w)

    def rope(t):
        c, s_ = cos[:, :, None, :], sin[:, :, None, :]
        x1, x2 = t[..., :rp], t[..., hd // 2: hd // 2 + rp]
        out = t.clone()
        out[..., :rp] = x1 * c - x2 * s_
        out[..., hd // 2: hd // 2 + rp] = x2 * c + x1 * s_
        return out

    qn, kn = rope(norm(q, wqr)), rope(norm(k, wkr))
    a = F.scaled_dot_product_attention(qn.transpose(1, 2), kn.transpose(1, 2), v.transpose(1, 2), is_causal=True,
                                       enable_gqa=True).transpose(1, 2)
    ref = (a * torch.sigmoid(gl)[..., None]).reshape(B, S, H * hd)
    ref.backward(do.float())
    assert rel_err(o, ref) < 1e-2 and cosine(o, ref) > 0.9995
    W = (H + 2 * Hkv) * hd + H
    assert rel_err(qkvg.grad[..., :W], xr.grad[..., :W]) < 3e-2 and cosine(qkvg.grad[..., :W], xr.grad[..., :W]) > 0.999
    assert torch.all(qkvg.grad[..., W:] == 0)
    for a_, b_ in ((wq.grad, wqr.grad), (wk.grad, wkr.grad)):
        assert cosine(a_, b_) > 0.999 and rel_err(a_, b_) < 3e-2


@pytest.mark.parametrize("B,S,H,hd,extra", [(2, 300, 4, 64, 0), (1, 4096, 12, 128, 1024), (3, 17, 2, 128, 8)])
def test_sink_key_gradient_kernel(B, S, H, hd, extra):
    """zs_attention_sink_grad against the f64 sum over (batch, position), q read from rows wider
    than the heads (the fused q|k buffer), and bit-identical on a second run."""
    from zs_b200.attn import sink_grad

    g = torch.Generator(device="cuda").manual_seed(S + hd)
    ld = H * hd + extra
    qbuf = torch.randn(B, S, ld, device="cuda", generator=g).bfloat16()
    ds = torch.randn(B, H, S, device="cuda", generator=g)
    got = sink_grad(ds, qbuf, ld, B, S, H, hd, 0.125)
    q = qbuf[..., : H * hd].reshape(B, S, H, hd).double()
    want = torch.einsum("bhs,bshd->hd", ds.double(), q) * 0.125
    assert (got.double() - want).norm() / want.norm() < 1e-6
    assert torch.equal(sink_grad(ds, qbuf, ld, B, S, H, hd, 0.125), got)
