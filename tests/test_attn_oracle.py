"""The attention oracle pinned to PyTorch's scaled_dot_product_attention on the
CPU: per-sequence causal SDPA for packed sequences (flash_attn_varlen_func's
semantics, modeling/attention.py:131-169), a banded mask for the window, GQA
by repeating K/V heads, and the sink appended as hca.py:264-298 does (k_sink
row with a zero value row, always visible).  Also the host-side seg_start
construction."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from _util import rel_err
from oracle import attention as A


def _sdpa_varlen(q, k, v, cu, window, k_sink):
    """Reference semantics on flattened packed tokens: each [cu[i], cu[i+1]) span is one sequence."""
    T, H, hd = q.shape
    G = H // k.shape[1]
    outs = []
    for i in range(len(cu) - 1):
        a, b = cu[i], cu[i + 1]
        n = b - a
        qs = q[a:b].transpose(0, 1)[None]
        ks = k[a:b].repeat_interleave(G, dim=1).transpose(0, 1)[None]
        vs = v[a:b].repeat_interleave(G, dim=1).transpose(0, 1)[None]
        idx = torch.arange(n)
        mask = idx[None, :] <= idx[:, None]
        if window:
            mask &= idx[:, None] - idx[None, :] < window
        if k_sink is not None:
            ks = torch.cat([ks, k_sink.view(1, H, 1, hd)], dim=2)
            vs = torch.cat([vs, torch.zeros(1, H, 1, hd, dtype=vs.dtype)], dim=2)
            mask = torch.cat([mask, torch.ones(n, 1, dtype=torch.bool)], dim=1)
        outs.append(F.scaled_dot_product_attention(qs, ks, vs, attn_mask=mask)[0].transpose(0, 1))
    return torch.cat(outs, 0)


@pytest.mark.parametrize("window,sink", [(0, False), (5, False), (0, True), (7, True)])
def test_oracle_matches_sdpa_packed(window, sink):
    g = torch.Generator().manual_seed(11 + window)
    B, S, H, Hkv, hd = 2, 24, 4, 2, 16
    q = torch.randn(B, S, H, hd, generator=g, dtype=torch.float64)
    k = torch.randn(B, S, Hkv, hd, generator=g, dtype=torch.float64)
    v = torch.randn(B, S, Hkv, hd, generator=g, dtype=torch.float64)
    ksink = torch.randn(H, hd, generator=g, dtype=torch.float64) if sink else None
    # row 0: sequences of 9 and 11 then 4 padding; row 1: one sequence of 17 then padding
    seq_ids = torch.full((B, S), -1, dtype=torch.long)
    seq_ids[0, :9] = 0
    seq_ids[0, 9:20] = 1
    seq_ids[1, :17] = 2
    from zs_b200.attn import seg_start_from_seq_ids

    seg = seg_start_from_seq_ids(seq_ids)
    assert seg[0, :9].tolist() == [0] * 9 and seg[0, 9:20].tolist() == [9] * 11
    assert seg[0, 20:].tolist() == [-1] * 4 and seg[1, 16].item() == 0 and seg[1, 17].item() == -1
    o, lse = A.attention_forward(q.numpy(), k.numpy(), v.numpy(), window=window, seg_start=seg.numpy(),
                                 k_sink=None if ksink is None else ksink.numpy())
    valid = (seq_ids >= 0).flatten()
    qf, kf, vf = (t.reshape(B * S, -1, hd)[valid] for t in (q, k, v))
    ref = _sdpa_varlen(qf, kf, vf, [0, 9, 20, 37], window, ksink)
    got = torch.from_numpy(o).reshape(B * S, H, hd)[valid]
    assert rel_err(got, ref) < 1e-12
    # padding rows: zero output; lse -inf without a sink, the sink logit with one
    assert np.all(o.reshape(B * S, H, hd)[~valid.numpy()] == 0)
    if not sink:
        assert np.all(np.isneginf(lse[0, :, 20:]))


@pytest.mark.parametrize("window,sink", [(0, False), (6, True)])
def test_oracle_backward_matches_autograd(window, sink):
    g = torch.Generator().manual_seed(5)
    B, S, H, Hkv, hd = 1, 20, 4, 1, 8
    q = torch.randn(B, S, H, hd, generator=g, dtype=torch.float64, requires_grad=True)
    k = torch.randn(B, S, Hkv, hd, generator=g, dtype=torch.float64, requires_grad=True)
    v = torch.randn(B, S, Hkv, hd, generator=g, dtype=torch.float64, requires_grad=True)
    ks = torch.randn(H, hd, generator=g, dtype=torch.float64, requires_grad=True) if sink else None
    do = torch.randn(B, S, H, hd, generator=g, dtype=torch.float64)
    ref = _sdpa_varlen(q[0], k[0], v[0], [0, S], window, ks)
    (ref * do[0]).sum().backward()
    dq, dk, dv, dks = A.attention_backward(do.numpy(), q.detach().numpy(), k.detach().numpy(), v.detach().numpy(),
                                           window=window, k_sink=None if ks is None else ks.detach().numpy())
    assert rel_err(dq, q.grad) < 1e-12 and rel_err(dk, k.grad) < 1e-12 and rel_err(dv, v.grad) < 1e-12
    if sink:
        assert rel_err(dks, ks.grad) < 1e-12
