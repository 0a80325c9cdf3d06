"""Generate golden fixtures by running the reference implementation itself.

Run once in a container that has the reference checked out (read-only) at
$ZS_REFERENCE (default /root/reference):

    python tests/golden/gen_golden.py

The reference's Triton kernels (scattermoe/kernels/ops.py) run on the CPU
through Triton's interpreter (TRITON_INTERPRET=1); MoEGate and
flatten_sort_count run as plain CPU PyTorch.  Outputs are small .npz files next
to this script; the tests read only those files and never the reference.
"""
from __future__ import annotations

import os
import sys
import types
import zlib
from pathlib import Path

os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np
import torch

REF = os.environ.get("ZS_REFERENCE", "/root/reference")
OUT = Path(__file__).resolve().parent


def _import_reference():
    sys.path.insert(0, REF)
    from scattermoe.kernels import ops  # noqa: F401
    from scattermoe import parallel_experts, mlp  # noqa: F401
    from modeling import moe_gate  # noqa: F401
    return ops, parallel_experts, mlp, moe_gate


def _np(t):
    return t.detach().float().cpu().numpy() if t.is_floating_point() else t.detach().cpu().numpy()


def gen_gate(moe_gate):
    cases = {}
    for name, (T, d, E, k, bias_std, seed) in {
        "gate_e8_k2": (64, 32, 8, 2, 0.0, 11),
        "gate_e64_k8": (300, 48, 64, 8, 0.1, 12),
        "gate_e128_k8": (97, 40, 128, 8, 0.1, 13),
    }.items():
        g = torch.Generator().manual_seed(seed)
        cfg = types.SimpleNamespace(n_experts_per_token=k, n_routed_experts=E, hidden_size=d, initializer_range=0.2)
        gate = moe_gate.MoEGate(cfg)
        with torch.no_grad():
            gate.weight.copy_(torch.randn(E, d, generator=g) * 0.2)
            gate.expert_biases.copy_(torch.randn(E, generator=g) * bias_std)
        hidden = torch.randn(1, T, d, generator=g)
        with torch.no_grad():
            idx, w = gate(hidden)
            probs = torch.sigmoid(torch.nn.functional.linear(hidden.view(-1, d), gate.weight))
        cases[name] = dict(hidden=_np(hidden.view(T, d)), weight=_np(gate.weight), bias=_np(gate.expert_biases),
                           probs=_np(probs), topk_idx=_np(idx.view(T, k)), topk_weight=_np(w.view(T, k)), k=k)
    return cases


def gen_fsc(parallel_experts):
    cases = {}
    for name, (T, k, E, seed) in {"fsc_small": (37, 2, 8, 21), "fsc_e64": (1500, 8, 64, 22),
                                  "fsc_skew": (700, 6, 64, 23)}.items():
        g = torch.Generator().manual_seed(seed)
        if name == "fsc_skew":
            probs = torch.softmax(torch.randn(E, generator=g) * 3, 0)
            idx = torch.multinomial(probs.expand(T, E), k, replacement=False, generator=g)
        else:
            idx = torch.randint(0, E, (T, k), generator=g)
        sei, ssi, off = parallel_experts.flatten_sort_count(idx, num_experts=E)
        cases[name] = dict(expert_idxs=_np(idx), sorted_expert_idxs=_np(sei), sorted_scattered_idxs=_np(ssi),
                           expert_offsets=_np(off), num_experts=E)
    return cases


def _routing(T, k, E, g):
    scores = torch.rand(T, E, generator=g)
    idx = torch.topk(scores, k, dim=-1).indices
    p = torch.softmax(torch.randn(T, k, generator=g), -1)
    return idx, p


def gen_ops(ops, parallel_experts):
    cases = {}
    T, d, E, k, N = 45, 64, 6, 3, 80
    g = torch.Generator().manual_seed(31)
    X = torch.randn(T, d, generator=g)
    Wt = torch.randn(E, N, d, generator=g) * 0.1          # weight [E, out, in]
    idx, p = _routing(T, k, E, g)
    sei, ssi, off = parallel_experts.flatten_sort_count(idx, num_experts=E)
    base = dict(X=_np(X), Wt=_np(Wt), expert_idxs=_np(idx), p=_np(p), sorted_expert_idxs=_np(sei),
                sorted_scattered_idxs=_np(ssi), expert_offsets=_np(off), k=k)
    # scatter2scatter, x ungrouped -> y grouped and y scattered
    base["s2s_xg0_yg1"] = _np(ops.scatter2scatter(X, Wt.permute(0, 2, 1), sei, ssi, k, x_grouped=False, y_grouped=True))
    base["s2s_xg0_yg0"] = _np(ops.scatter2scatter(X, Wt.permute(0, 2, 1), sei, ssi, k, x_grouped=False, y_grouped=False))
    Xg = torch.randn(T * k, d, generator=g)
    base["Xg"] = _np(Xg)
    base["s2s_xg1_yg1"] = _np(ops.scatter2scatter(Xg, Wt.permute(0, 2, 1), sei, ssi, 1, x_grouped=True, y_grouped=True))
    base["s2s_xg1_yg0"] = _np(ops.scatter2scatter(Xg, Wt.permute(0, 2, 1), sei, ssi, 1, x_grouped=True, y_grouped=False))
    # the transposed weight as used for input gradients (N contiguous)
    DYg = torch.randn(T * k, N, generator=g)
    base["DYg"] = _np(DYg)
    base["s2s_wT"] = _np(ops.scatter2scatter(DYg, Wt, sei, ssi, 1, x_grouped=True, y_grouped=False))
    bias = torch.randn(E, N, generator=g)
    base["bias"] = _np(bias)
    base["s2s_bias"] = _np(ops.scatter2scatter(X, Wt.permute(0, 2, 1), sei, ssi, k, b=bias, x_grouped=False,
                                               y_grouped=True))
    dw, db = ops.group_bwd_W(DYg, Xg, off, E, has_bias=True)
    base["xty_dw"] = _np(dw)
    base["xty_db"] = _np(db)
    base["group"] = _np(ops.group(X, ssi, fan_out=k))
    base["group_coeff"] = _np(ops.group(X, ssi, fan_out=k, coeff=p.flatten()))
    A3 = torch.randn(T, k, d, generator=g)
    B2 = torch.randn(T, d, generator=g)
    base["A3"] = _np(A3)
    base["B2"] = _np(B2)
    base["rsp"] = _np(ops.rowwise_sum_product(A3, B2))
    cases["ops_f32"] = base
    return cases


def gen_glu(mlp):
    cases = {}
    for name, (T, d, E, k, f, seed) in {"glu_small": (33, 64, 4, 2, 32, 41), "glu_e8": (70, 96, 8, 3, 48, 42)}.items():
        g = torch.Generator().manual_seed(seed)
        torch.manual_seed(seed)
        m = mlp.GLUMLP(d, f, E, k)
        with torch.no_grad():
            m.experts.weight.copy_(torch.randn(E, 2 * f, d, generator=g) * 0.1)
            m.output_experts.weight.copy_(torch.randn(E, d, f, generator=g) * 0.1)
        x = torch.randn(T, d, generator=g, requires_grad=True)
        idx, p = _routing(T, k, E, g)
        p = p.clone().requires_grad_(True)
        y = m(x, p, idx)
        dy = torch.randn(T, d, generator=g)
        y.backward(dy)
        cases[name] = dict(x=_np(x), expert_p=_np(p), expert_idxs=_np(idx), W1=_np(m.experts.weight),
                           W2=_np(m.output_experts.weight), y=_np(y), dy=_np(dy), dx=_np(x.grad), dp=_np(p.grad),
                           dW1=_np(m.experts.weight.grad), dW2=_np(m.output_experts.weight.grad), k=k)
    return cases


def main():
    ops, parallel_experts, mlp, moe_gate = _import_reference()
    all_cases = {}
    all_cases.update(gen_gate(moe_gate))
    all_cases.update(gen_fsc(parallel_experts))
    all_cases.update(gen_ops(ops, parallel_experts))
    all_cases.update(gen_glu(mlp))
    all_cases.update(gen_mcce())
    all_cases.update(gen_norm_rope())
    all_cases.update(gen_muon())
    all_cases.update(gen_data())
    all_cases.update(gen_sparse())
    all_cases.update(gen_step())
    for name, arrs in all_cases.items():
        np.savez_compressed(OUT / f"{name}.npz", **{kk: np.asarray(v) for kk, v in arrs.items()})
        print("wrote", name, sorted(arrs.keys()))




def gen_mcce():
    """MCCE fixtures from the reference's own CPU paths: the naive formulation
    (modeling/mcce_fast.py:117-139) for the loss and autograd gradients, and
    the chunked exact path (:147-249) as a second opinion."""
    from modeling import mcce_fast

    cases = {}
    shapes = {"mcce_selftest": (17, 64, 1009, 4, 123), "mcce_t1": (1, 16, 33, 1, 5), "mcce_t7": (7, 32, 127, 2, 6),
              "mcce_t33": (33, 64, 2099, 8, 7)}
    for name, (T, D, V, S_MAX, seed) in shapes.items():
        g = torch.Generator().manual_seed(seed)
        hidden = torch.randn(T, D, generator=g) / D ** 0.5
        emb = torch.randn(V, D, generator=g) / D ** 0.5 * (3.0 if name == "mcce_selftest" else 1.0)
        s = torch.randint(1, S_MAX + 1, (T,), generator=g, dtype=torch.int32)
        labels = torch.randint(0, V, (T, S_MAX), generator=g, dtype=torch.int64)
        if S_MAX >= 2:
            labels[:, 1] = labels[:, 0]                       # duplicate labels count twice
        cols = torch.arange(S_MAX)[None, :]
        labels = torch.where(cols < s[:, None].long(), labels, torch.full_like(labels, V + 777))  # never read
        h1 = hidden.clone().requires_grad_(True)
        e1 = emb.clone().requires_grad_(True)
        loss = mcce_fast.naive_mcce_raw_token_mean(h1, e1, labels, s)
        loss.backward()
        h2 = hidden.clone().requires_grad_(True)
        e2 = emb.clone().requires_grad_(True)
        loss2 = mcce_fast.mcce_raw_token_mean(h2, e2, labels, s, use_triton=False, v_chunk_size=128)
        loss2.backward()
        # the reference's two CPU paths agree with each other
        assert torch.allclose(loss, loss2, rtol=1e-5, atol=1e-6)
        assert torch.allclose(h1.grad, h2.grad, rtol=1e-4, atol=1e-6)
        assert torch.allclose(e1.grad, e2.grad, rtol=1e-4, atol=1e-6)
        cases[name] = dict(hidden=_np(hidden), emb=_np(emb), labels=_np(labels), s=_np(s), loss=_np(loss),
                           dH=_np(h1.grad), dE=_np(e1.grad))
    # standard CE with ignore_index, as F.cross_entropy defines it
    g = torch.Generator().manual_seed(9)
    T, D, V = 50, 48, 777
    e = torch.randn(T, D, generator=g) / D ** 0.5
    c = torch.randn(V, D, generator=g)
    t = torch.randint(0, V, (T,), generator=g)
    t[::7] = -100
    e1 = e.clone().requires_grad_(True)
    c1 = c.clone().requires_grad_(True)
    loss = torch.nn.functional.cross_entropy(e1 @ c1.T, t, ignore_index=-100)
    loss.backward()
    cases["cce_ignore"] = dict(e=_np(e), c=_np(c), targets=_np(t), loss=_np(loss), de=_np(e1.grad), dc=_np(c1.grad))
    return cases


if __name__ == "__main__" and os.environ.get("ZS_GOLDEN_ONLY") == "mcce":
    sys.path.insert(0, REF)
    for name, arrs in gen_mcce().items():
        np.savez_compressed(OUT / f"{name}.npz", **{kk: np.asarray(v) for kk, v in arrs.items()})
        print("wrote", name)




def gen_norm_rope():
    """zRMSNorm from the reference module (CPU autograd); Liger RoPE from the
    reference's Triton kernel under the interpreter; RoPE tables from the
    reference's own table builder."""
    from modeling.zRMSNorm import ZeroCenteredRMSNorm
    from modeling import liger_rope
    from modeling.attention import GatedAttention

    cases = {}
    g = torch.Generator().manual_seed(51)
    for name, (rows, d) in {"zrms_d64": (37, 64), "zrms_d256": (20, 256)}.items():
        m = ZeroCenteredRMSNorm(d, eps=1e-6)
        with torch.no_grad():
            m.weight.copy_(torch.randn(d, generator=g) * 0.1)
        x = (torch.randn(rows, d, generator=g) * 2).requires_grad_(True)
        y = m(x)
        dy = torch.randn(rows, d, generator=g)
        y.backward(dy)
        cases[name] = dict(x=_np(x), w=_np(m.weight), y=_np(y), dy=_np(dy), dx=_np(x.grad), dw=_np(m.weight.grad))
    fake = types.SimpleNamespace(pos_rope_pairs=16, pos_rope_dims=32)
    cos_t, sin_t = GatedAttention._build_pos_rope_tables(fake, 300, 64, 10000.0, torch.float32, "cpu")
    B, S, Hq, Hk, hd = 2, 11, 4, 2, 64
    pos = torch.randint(0, 300, (B, S), generator=g)
    cos, sin = cos_t[pos], sin_t[pos]
    q = torch.randn(B, S, Hq, hd, generator=g)
    k = torch.randn(B, S, Hk, hd, generator=g)
    q_out, k_out = liger_rope.LigerRopeFunction.apply(q.clone(), k.clone(), cos, sin, cos, sin)
    dq = torch.randn(B, S, Hq, hd, generator=g)
    dk = torch.randn(B, S, Hk, hd, generator=g)
    dq_out, dk_out = liger_rope.rope_backward(dq.clone(), dk.clone(), cos, sin, cos, sin)
    cases["rope"] = dict(cos_table=_np(cos_t), sin_table=_np(sin_t), pos=_np(pos), q=_np(q), k=_np(k),
                         q_out=_np(q_out), k_out=_np(k_out), dq=_np(dq), dk=_np(dk), dq_out=_np(dq_out),
                         dk_out=_np(dk_out))
    return cases


if __name__ == "__main__" and os.environ.get("ZS_GOLDEN_ONLY") == "norm_rope":
    sys.path.insert(0, REF)
    for name, arrs in gen_norm_rope().items():
        np.savez_compressed(OUT / f"{name}.npz", **{kk: np.asarray(v) for kk, v in arrs.items()})
        print("wrote", name)


def gen_muon():
    """Newton-Schulz output and two MuonMD steps from the reference optimizer on CPU."""
    from optimizer import muon

    cases = {}
    g = torch.Generator().manual_seed(61)
    Gw = torch.randn(3, 64, 128, generator=g)
    Gt = torch.randn(2, 96, 64, generator=g)
    cases["ns5"] = dict(G_wide=_np(Gw), X_wide=_np(muon.zeropower_via_newtonschulz5(Gw, 5).float()),
                        G_tall=_np(Gt), X_tall=_np(muon.zeropower_via_newtonschulz5(Gt, 5).float()))
    for gain_mode, norm_axis, rescale in [("both", "frobenius", "balanced"), ("col", "row", "muon"),
                                          ("scalar", "frobenius", "balanced"), ("none", "col", "balanced")]:
        W0 = torch.randn(4, 64, 96, generator=g) * 0.05
        p = W0.clone()
        state = {}
        grads = [torch.randn(4, 64, 96, generator=g) * 0.01 for _ in range(2)]
        for gr in grads:
            muon.md_decoupled_step(p, gr.clone(), state, lr=0.02, momentum=0.95, gain_lr=1e-3,
                                   gain_betas=(0.9, 0.95), gain_eps=1e-10, gain_mode=gain_mode, norm_axis=norm_axis,
                                   ns_steps=5, rescale_mode=rescale)
        out = dict(W0=_np(W0), grad0=_np(grads[0]), grad1=_np(grads[1]), W2=_np(p),
                   momentum=_np(state["momentum_buffer"]))
        for key in ("g_scalar", "g_row", "g_col"):
            if key in state:
                out[key] = _np(state[key])
        cases[f"md_{gain_mode}_{norm_axis}"] = out
    return cases


if __name__ == "__main__" and os.environ.get("ZS_GOLDEN_ONLY") == "muon":
    sys.path.insert(0, REF)
    for name, arrs in gen_muon().items():
        np.savez_compressed(OUT / f"{name}.npz", **{kk: np.asarray(v) for kk, v in arrs.items()})
        print("wrote", name)


def _import_reference_main():
    """The reference trainer module (main.py) with stand-ins for the two modules it
    imports that are absent here (aim, cut_cross_entropy); only its data functions
    are called."""
    sys.path.insert(0, REF)
    for name, attrs in (("aim", ("Distribution", "Run")), ("cut_cross_entropy", ("linear_cross_entropy",))):
        if name not in sys.modules:
            mod = types.ModuleType(name)
            for a in attrs:
                setattr(mod, a, None)
            sys.modules[name] = mod
    import main as ref_main  # noqa: E402
    return ref_main


def gen_data():
    """Packed-batch and TST-batch fixtures from the reference's PackedTokenizedCollator
    (main.py:57-129), build_token_superposition_batch (:243-352) and
    bag_label_entropy_floor (:187-215) on seeded synthetic token lists."""
    ref = _import_reference_main()
    g = np.random.default_rng(11)
    cases = {}
    # lengths include empty, single-token, exactly max_length and over-long examples
    for name, L, lens in (("pack_a", 64, [5, 0, 64, 30, 30, 3, 1, 70, 12, 40, 25, 2, 17, 9]),
                          ("pack_b", 128, list(g.integers(1, 90, size=40)))):
        examples = [{"token_ids": [int(t) for t in g.integers(2, 1000, size=n)]} for n in lens]
        out = ref.PackedTokenizedCollator(L, 0)(examples)
        arrs = {k: (v.numpy() if torch.is_tensor(v) else np.asarray(v)) for k, v in out.items()}
        arrs["lens"] = np.asarray(lens)
        arrs["tokens"] = np.concatenate([np.asarray(e["token_ids"], np.int64) for e in examples] or [np.zeros(0)])
        arrs["L"] = np.asarray(L)
        cases[name] = arrs
        for sname, s_bag, latent in (("tst_a", 4, 8), ("tst_b", 3, 40)):
            if name != "pack_b" and sname == "tst_b":
                continue
            tb = ref.build_token_superposition_batch(out, s_bag, latent, 0)
            t = {k: (v.numpy() if torch.is_tensor(v) else np.asarray(v)) for k, v in tb.items()}
            t["floor"] = ref.bag_label_entropy_floor(tb["labels"], tb["s"]).numpy()
            t["src"] = name
            t["s_bag"], t["latent"] = np.asarray(s_bag), np.asarray(latent)
            cases[f"{sname}_{name}"] = t
    return cases


if __name__ == "__main__" and os.environ.get("ZS_GOLDEN_ONLY") == "data":
    for name, arrs in gen_data().items():
        np.savez_compressed(OUT / f"{name}.npz", **{kk: np.asarray(v) for kk, v in arrs.items()})
        print("wrote", name)


def gen_sparse():
    """Three GramReaperSparse steps (engram/GramReaperSparse.py:18-66) of the reference on
    seeded COO gradients with duplicate rows, with and without the unit-norm projection;
    the middle step's gradient touches no row."""
    sys.path.insert(0, REF)
    from engram.GramReaperSparse import GramReaperSparse

    cases = {}
    g = torch.Generator().manual_seed(71)
    for name, unit in (("sparse_unit", True), ("sparse_plain", False)):
        V, d = 50, 16
        W0 = torch.randn(V, d, generator=g)
        if unit:
            W0 = W0 / W0.norm(dim=1, keepdim=True)
        p = torch.nn.Parameter(W0.clone())
        opt = GramReaperSparse([dict(params=[p], unit_norm=unit)], lr=3e-2, beta=0.9, unit_norm=unit)
        out = dict(W0=_np(W0).copy())
        for k, n in enumerate((40, 0, 25)):
            rows = torch.randint(0, V, (n,), generator=g)
            if n:
                rows[: n // 4] = rows[0]                      # a row hit several times
            vals = torch.randn(n, d, generator=g)
            p.grad = torch.sparse_coo_tensor(rows.view(1, -1), vals, (V, d))
            opt.step()
            # copies: the parameter keeps changing in place
            out[f"rows{k}"], out[f"vals{k}"], out[f"W{k + 1}"] = _np(rows), _np(vals), _np(p).copy()
        st = opt.state[p]
        out["v"], out["t"] = _np(st["v"]).copy(), np.asarray(st["t"])
        cases[name] = out
    return cases


if __name__ == "__main__" and os.environ.get("ZS_GOLDEN_ONLY") == "sparse":
    for name, arrs in gen_sparse().items():
        np.savez_compressed(OUT / f"{name}.npz", **{kk: np.asarray(v) for kk, v in arrs.items()})
        print("wrote", name)


def _sdpa_varlen(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, dropout_p=0.0, causal=True,
                 window_size=(-1, -1), **_):
    """CPU stand-in for flash_attn_varlen_func (CUDA only): exact causal GQA softmax
    attention per packed sequence (q head h reads kv head h // (H / Hkv))."""
    assert causal and tuple(window_size) == (-1, -1)
    out = torch.empty_like(q)
    rep = q.size(1) // k.size(1)
    cu = cu_seqlens_q.tolist()
    for a, b in zip(cu[:-1], cu[1:]):
        qq = q[a:b].transpose(0, 1)
        kk = k[a:b].repeat_interleave(rep, dim=1).transpose(0, 1)
        vv = v[a:b].repeat_interleave(rep, dim=1).transpose(0, 1)
        out[a:b] = torch.nn.functional.scaled_dot_product_attention(qq, kk, vv, is_causal=True).transpose(0, 1)
    return out


STEP_SAMPLES = 4096


def _sample_idx(name, numel, rows=None, width=None):
    """Seeded flat indices (sorted) of up to STEP_SAMPLES elements of a parameter; for the
    embedding only inside the touched rows."""
    g = torch.Generator().manual_seed(zlib.crc32(name.encode()))
    if rows is not None:
        r = rows[torch.randint(0, rows.numel(), (STEP_SAMPLES,), generator=g)]
        c = torch.randint(0, width, (STEP_SAMPLES,), generator=g)
        return torch.unique(r * width + c)
    if numel <= STEP_SAMPLES:
        return torch.arange(numel)
    return torch.unique(torch.randint(0, numel, (STEP_SAMPLES,), generator=g))


def gen_step():
    """One full training step of the reference at BASELINE config 1's shapes on the CPU
    (main.py:723-815 with s == 1): its own MoEModel, build_muonmd_optimizer and
    auxillary_loss_free_update, on weights from oracle.model_step.canonical_params (N(0, 0.02),
    unit-norm embedding rows, zero norm gains and biases) and seeded ids [4, 256].  The
    reference's scattermoe and Liger RoPE Triton kernels run under Triton's interpreter,
    flash_attn_varlen_func is replaced by exact SDPA (_sdpa_varlen), linear_cross_entropy by
    F.cross_entropy over h @ W^T.  Stored: the loss, every layer's routing and gate
    probabilities, layer outputs, and for every parameter the gradient and the weights after
    the optimizer step at up to 4096 seeded positions plus their full norms and sums."""
    ref = _import_reference_main()
    sys.path.insert(0, str(OUT.parents[1]))
    from oracle.model_step import canonical_ids, canonical_params, config1
    import modeling.attention as ref_attn
    from modeling.model import MoEModel
    from modeling.model_config import ModelConfig

    ref_attn.flash_attn_varlen_func = _sdpa_varlen
    c1 = config1()
    cfg = ModelConfig(vocab_size=c1["vocab_size"], embed_size=c1["hidden_size"], hidden_size=c1["hidden_size"],
                      transformer_depth=c1["transformer_depth"], intermediate_size=c1["intermediate_size"],
                      n_experts=c1["n_routed_experts"] + 1, n_shared_experts=1,
                      n_experts_per_token=c1["n_experts_per_token"], n_attention_heads=c1["n_attention_heads"],
                      n_key_value_heads=c1["n_key_value_heads"], attention_window_pattern=(None, None),
                      max_position_embeddings=c1["max_position_embeddings"], sequence_length=256,
                      pos_rope_dims=c1["pos_rope_dims"])
    torch.manual_seed(0)
    model = MoEModel(cfg)
    P = canonical_params(c1, 0)
    sd = model.state_dict()
    missing = set(P) ^ {k for k in sd if not k.endswith("expert_biases")}
    assert not missing, missing
    with torch.no_grad():
        for k, v in P.items():
            sd[k].copy_(v)
    ids = canonical_ids(c1, 4, 256, 1)
    mask = torch.ones_like(ids)
    opt = ref.build_muonmd_optimizer(model, torch.device("cpu"))
    keep = {}
    hooks = []
    for i, layer in enumerate(model.layers):
        hooks.append(layer.self_attn.register_forward_hook(
            lambda m, a, o, i=i: keep.__setitem__(f"attn{i}", o.detach().clone())))
        hooks.append(layer.mlp.register_forward_hook(
            lambda m, a, o, i=i: keep.update({f"moe{i}": o[0].detach().clone(),
                                              f"probs{i}": torch.sigmoid(a[0].reshape(-1, a[0].size(-1))
                                                                         @ m.gate.weight.T).detach().clone()})))
        hooks.append(layer.register_forward_hook(lambda m, a, o, i=i: keep.__setitem__(f"out{i}", o[0].detach().clone())))
    opt.zero_grad(set_to_none=False)
    emb, topk = model.headless_forward(ids)
    le, labels = ref.build_next_token_loss_inputs(emb, ids, mask)
    loss = torch.nn.functional.cross_entropy(le.reshape(-1, le.size(-1)) @ model.get_classifier_weights().T,
                                             labels.reshape(-1), ignore_index=-100)
    loss.backward()
    for h in hooks:
        h.remove()
    grads = {n: (p.grad.to_dense() if p.grad.is_sparse else p.grad).detach().clone()
             for n, p in model.named_parameters()}
    before = {n: p.detach().clone() for n, p in model.named_parameters()}
    opt.step()
    ref.auxillary_loss_free_update(model, topk, 1e-3, mask)
    out = dict(loss=_np(loss), ids=_np(ids))
    touched = torch.unique(ids)
    for n, p in model.named_parameters():
        rows = touched if n == "embedding.weight" else None
        idx = _sample_idx(n, p.numel(), rows, p.size(-1))
        out[f"idx:{n}"] = idx.numpy().astype(np.int64)
        out[f"grad:{n}"] = _np(grads[n].reshape(-1)[idx]).copy()
        out[f"after:{n}"] = _np(p.detach().reshape(-1)[idx]).copy()
        out[f"delta:{n}"] = _np((p.detach() - before[n]).reshape(-1)[idx]).copy()
        out[f"gnorm:{n}"] = np.asarray(float(grads[n].norm()))
        out[f"dnorm:{n}"] = np.asarray(float((p.detach() - before[n]).norm()))
    for i, layer in enumerate(model.layers):
        out[f"topk{i}"] = _np(topk[i]).copy()
        out[f"probs{i}"] = _np(keep[f"probs{i}"]).copy()
        out[f"bias_after{i}"] = _np(layer.mlp.gate.expert_biases).copy()
        for key in ("attn", "moe", "out"):
            t = keep[f"{key}{i}"].reshape(-1)
            sel = _sample_idx(f"{key}{i}", t.numel())
            out[f"{key}{i}"] = _np(t[sel]).copy()
            out[f"{key}{i}_idx"] = sel.numpy().astype(np.int64)
            out[f"{key}{i}_norm"] = np.asarray(float(t.norm()))
    return {"step_cfg1": out}


if __name__ == "__main__" and os.environ.get("ZS_GOLDEN_ONLY") == "step":
    for name, arrs in gen_step().items():
        np.savez_compressed(OUT / f"{name}.npz", **{kk: np.asarray(v) for kk, v in arrs.items()})
        print("wrote", name, len(arrs))


CKPT_CONFIG = dict(vocab_size=128, embed_size=32, hidden_size=32, transformer_depth=2, intermediate_size=16,
                   n_experts=5, n_shared_experts=1, n_experts_per_token=2, n_attention_heads=2, n_key_value_heads=1,
                   attention_window_pattern=(None, None), max_position_embeddings=32, sequence_length=32,
                   pos_rope_dims=8)


def gen_ckpt():
    """A checkpoint written by the reference's save_checkpoint (utils/trainutils.py:34-59)
    for a tiny MoEModel after one step of its build_muonmd_optimizer optimizer
    (main.py:354-465) on seeded synthetic gradients (the model's forward needs
    flash-attn on a GPU, so the gradients are set directly)."""
    ref = _import_reference_main()
    from modeling.model import MoEModel
    from modeling.model_config import ModelConfig
    from utils.trainutils import save_checkpoint

    torch.manual_seed(21)
    model = MoEModel(ModelConfig(**CKPT_CONFIG))
    opt = ref.build_muonmd_optimizer(model, torch.device("cpu"))
    g = torch.Generator().manual_seed(22)
    emb = model.embedding.weight
    for p in model.parameters():
        if p is emb:
            rows = torch.tensor([[1, 5, 9, 77]])
            p.grad = torch.sparse_coo_tensor(rows, torch.randn(4, p.size(1), generator=g), p.shape)
        else:
            p.grad = torch.randn(p.shape, generator=g) * 0.01
    opt.step()
    save_checkpoint(model, opt, str(OUT / "ckpt_ref.safetensors"), global_step=1, epoch=0)
    print("wrote ckpt_ref.safetensors / ckpt_ref.trainer.pt")


if __name__ == "__main__" and os.environ.get("ZS_GOLDEN_ONLY") == "ckpt":
    gen_ckpt()


if __name__ == "__main__" and os.environ.get("ZS_GOLDEN_ONLY") is None:
    main()
    gen_ckpt()
