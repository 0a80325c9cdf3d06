"""CPU restatement of the reference's whole MoE training step — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py (its cpu_baseline leg and its
--impl reference arm) may import this module, as the checker or as the timed
CPU baseline.  Nothing in the product path imports it.

Restates, in PyTorch on the CPU (f32; the Newton-Schulz in bf16 as the
reference computes it), the step body of main.py:723-815 for s == 1:

  * embedding: modeling/model.py:71-86 (lookup, x sqrt(d) when untied);
  * TransformerBlock: modeling/transformer_block.py:19-46 (pre-norm residual);
  * ZeroCenteredRMSNorm: modeling/zRMSNorm.py:10-17;
  * GatedAttention: modeling/attention.py:172-226 (q/k/v projections, per-head
    QK-norm, partial rotate-half RoPE with the tables of :85-104, causal GQA
    softmax attention in place of flash_attn_varlen_func, sigmoid head gate,
    o_proj);
  * MoELayer: modeling/moe_layer.py:38-58 with MoEGate (moe_gate.py:19-35:
    sigmoid scores, biased top-k, L1-normalised weights), the shared ExpertMLP
    (expert_layer.py:23-24) and GLUMLP (scattermoe/mlp.py:74-95: first half of
    experts.weight = up, second half = gate, weighted k-way sum);
  * final norm, next-token labels (main.py:177-185), mean cross entropy over
    non-ignored targets (the linear_cross_entropy call at main.py:755-761);
  * backward (autograd), then the optimizer of build_muonmd_optimizer
    (main.py:354-465): MuonMD (optimizer/muon.py:339-508) on matrices and
    expert stacks, the router on row spheres with column gains and the Muon
    shape factor, AdamW for the head (wd 0.1) and Adam for 1-D parameters
    (muon.py:620-653), GramReaperSparse on the embedding rows
    (engram/GramReaperSparse.py:18-66);
  * auxillary_loss_free_update (main.py:161-175).

Parameters are a dict keyed by the reference's parameter names, generated from
(name, seed) by canonical_params(), so a test and the fixture generator build
identical weights without storing them.  Pinned by tests/test_step_oracle.py
against one step of the reference itself (tests/golden/gen_golden.py,
gen_step).
"""
from __future__ import annotations

import math
import os
import time
import zlib

import torch
import torch.nn.functional as F

NS = (3.4445, -4.7750, 2.0315)
RAW_GAIN_INIT = 0.5413248546129181   # softplus^-1(1)


def config1():
    """the tiny MoE LM whose full step runs on the CPU."""
    return dict(vocab_size=8192, hidden_size=256, transformer_depth=2, intermediate_size=512, n_routed_experts=8,
                n_shared_experts=1, n_experts_per_token=2, n_attention_heads=4, n_key_value_heads=4,
                rms_norm_eps=1e-6, rope_theta=10000, pos_rope_dims=32, max_position_embeddings=256,
                initializer_range=0.02)


# --------------------------------------------------------------- parameters

def param_shapes(cfg):
    """{name: (shape, init)} in the reference's naming; init in {"normal", "zeros", "unit_rows"}."""
    d, V, f = cfg["hidden_size"], cfg["vocab_size"], cfg["intermediate_size"]
    H, Hkv = cfg["n_attention_heads"], cfg["n_key_value_heads"]
    hd = d // H
    E = cfg["n_routed_experts"]
    fs = f * cfg["n_shared_experts"]
    out = {"embedding.weight": ((V, d), "unit_rows")}
    for i in range(cfg["transformer_depth"]):
        p = f"layers.{i}."
        out[p + "input_layernorm.weight"] = ((d,), "zeros")
        out[p + "self_attn.q_proj.weight"] = ((H * hd, d), "normal")
        out[p + "self_attn.k_proj.weight"] = ((Hkv * hd, d), "normal")
        out[p + "self_attn.v_proj.weight"] = ((Hkv * hd, d), "normal")
        out[p + "self_attn.o_proj.weight"] = ((d, H * hd), "normal")
        out[p + "self_attn.head_gate_proj.weight"] = ((H, d), "normal")
        out[p + "self_attn.q_norm.weight"] = ((hd,), "zeros")
        out[p + "self_attn.k_norm.weight"] = ((hd,), "zeros")
        out[p + "post_attention_layernorm.weight"] = ((d,), "zeros")
        out[p + "mlp.gate.weight"] = ((E, d), "normal")
        out[p + "mlp.shared_experts.gate_proj.weight"] = ((fs, d), "normal")
        out[p + "mlp.shared_experts.up_proj.weight"] = ((fs, d), "normal")
        out[p + "mlp.shared_experts.down_proj.weight"] = ((d, fs), "normal")
        out[p + "mlp.routed_experts.experts.weight"] = ((E, 2 * f, d), "normal")
        out[p + "mlp.routed_experts.output_experts.weight"] = ((E, d, f), "normal")
    out["norm.weight"] = ((d,), "zeros")
    out["output_layer.weight"] = ((V, d), "normal")
    return out


def canonical_params(cfg, seed):
    """Seeded f32 weights per parameter name (independent of construction order)."""
    std = cfg["initializer_range"]
    P = {}
    for name, (shape, kind) in param_shapes(cfg).items():
        g = torch.Generator().manual_seed((seed * 1000003 + zlib.crc32(name.encode())) % (2 ** 63))
        if kind == "zeros":
            P[name] = torch.zeros(shape)
        else:
            t = torch.randn(shape, generator=g) * std
            if kind == "unit_rows":
                t = t / t.norm(dim=1, keepdim=True).clamp_min(1e-12)
            P[name] = t
    return P


def canonical_ids(cfg, batch, seq, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, cfg["vocab_size"], (batch, seq), generator=g)


# ------------------------------------------------------------------ forward

def zrms(x, w, eps):
    xf = x.float()
    return xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * (1.0 + w.float())


def rope_tables(cfg, hd):
    half = hd // 2
    maxp = cfg["max_position_embeddings"]
    cos = torch.ones(maxp, half)
    sin = torch.zeros(maxp, half)
    pairs = cfg["pos_rope_dims"] // 2
    if pairs:
        inv = 1.0 / (cfg["rope_theta"] ** (torch.arange(0, cfg["pos_rope_dims"], 2, dtype=torch.float32)
                                           / cfg["pos_rope_dims"]))
        fr = torch.outer(torch.arange(maxp, dtype=torch.float32), inv)
        cos[:, :pairs] = fr.cos()
        sin[:, :pairs] = fr.sin()
    return cos, sin


def rope(x, cos, sin):
    """Rotate-half pairs (i, i + hd/2) of x [B, S, H, hd] by tables [B, S, hd/2]."""
    half = x.shape[-1] // 2
    c, s = cos[:, :, None, :], sin[:, :, None, :]
    x1, x2 = x[..., :half], x[..., half:]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)


def attention(P, p, cfg, x, cos, sin):
    B, S, d = x.shape
    H, Hkv = cfg["n_attention_heads"], cfg["n_key_value_heads"]
    hd = d // H
    eps = cfg["rms_norm_eps"]
    q = (x @ P[p + "q_proj.weight"].T).view(B, S, H, hd)
    k = (x @ P[p + "k_proj.weight"].T).view(B, S, Hkv, hd)
    v = (x @ P[p + "v_proj.weight"].T).view(B, S, Hkv, hd)
    q = zrms(q, P[p + "q_norm.weight"], eps)
    k = zrms(k, P[p + "k_norm.weight"], eps)
    q, k = rope(q, cos, sin), rope(k, cos, sin)
    rep = H // Hkv
    kq = k.repeat_interleave(rep, dim=2)
    vq = v.repeat_interleave(rep, dim=2)
    o = F.scaled_dot_product_attention(q.transpose(1, 2), kq.transpose(1, 2), vq.transpose(1, 2), is_causal=True)
    o = o.transpose(1, 2)
    gate = torch.sigmoid(x @ P[p + "head_gate_proj.weight"].T)
    o = (o * gate.unsqueeze(-1)).reshape(B, S, H * hd)
    return o @ P[p + "o_proj.weight"].T


def moe(P, p, cfg, x, bias, routing=None, keep=None):
    B, S, d = x.shape
    k = cfg["n_experts_per_token"]
    E = cfg["n_routed_experts"]
    xt = x.reshape(-1, d)
    probs = torch.sigmoid(xt @ P[p + "gate.weight"].T)
    if keep is not None:
        keep["gate_probs"] = probs.detach().clone()
    if routing is None:
        idx = torch.topk(probs + bias, k, dim=-1, sorted=False).indices
    else:
        idx = routing.reshape(-1, k)
    w = F.normalize(probs.gather(-1, idx), p=1, dim=-1)
    g = xt @ P[p + "shared_experts.gate_proj.weight"].T
    u = xt @ P[p + "shared_experts.up_proj.weight"].T
    shared = (F.silu(g) * u) @ P[p + "shared_experts.down_proj.weight"].T
    # one view per expert (unbind: the backward stacks the experts' gradients once)
    W1 = P[p + "routed_experts.experts.weight"].unbind(0)
    W2 = P[p + "routed_experts.output_experts.weight"].unbind(0)
    f = W2[0].shape[-1]
    routed = torch.zeros_like(xt)
    flat = idx.reshape(-1)
    for e in range(E):
        slots = (flat == e).nonzero().squeeze(-1)
        if slots.numel() == 0:
            continue
        tok = slots // k
        h = xt[tok] @ W1[e].T
        a = F.silu(h[:, f:]) * h[:, :f]
        out = (a @ W2[e].T) * w.reshape(-1)[slots].unsqueeze(-1)
        routed = routed.index_add(0, tok, out)
    return (shared + routed).view(B, S, d), idx.view(B, S, k)


def forward_loss(P, cfg, ids, biases, routing=None, keep=None):
    """(mean next-token CE, per-layer top-k ids).  keep (a dict) receives intermediates."""
    B, S = ids.shape
    d = cfg["hidden_size"]
    eps = cfg["rms_norm_eps"]
    hd = d // cfg["n_attention_heads"]
    cos_t, sin_t = rope_tables(cfg, hd)
    pos = torch.arange(S).expand(B, S)
    cos, sin = cos_t[pos], sin_t[pos]
    h = P["embedding.weight"][ids] * (d ** 0.5)
    topks = []
    for i in range(cfg["transformer_depth"]):
        p = f"layers.{i}."
        kp = {} if keep is not None else None
        a = attention(P, p + "self_attn.", cfg, zrms(h, P[p + "input_layernorm.weight"], eps), cos, sin)
        h = h + a
        m, idx = moe(P, p + "mlp.", cfg, zrms(h, P[p + "post_attention_layernorm.weight"], eps), biases[i],
                     None if routing is None else routing[i], kp)
        h = h + m
        topks.append(idx)
        if keep is not None:
            keep[f"layer{i}"] = dict(attn=a.detach().clone(), moe=m.detach().clone(), out=h.detach().clone(),
                                     gate_probs=kp["gate_probs"])
    hn = zrms(h, P["norm.weight"], eps)
    logits = hn[:, :-1].reshape(-1, d) @ P["output_layer.weight"].T
    labels = ids[:, 1:].reshape(-1)
    loss = F.cross_entropy(logits, labels, ignore_index=-100)
    return loss, topks


# ---------------------------------------------------------------- optimizer

def newton_schulz5(G, steps=5):
    a, b, c = NS
    X = G.bfloat16()
    tall = G.size(-2) > G.size(-1)
    if tall:
        X = X.mT
    X = X / (X.norm(dim=(-2, -1), keepdim=True) + 1e-7)
    for _ in range(steps):
        A = X @ X.mT
        Bm = b * A + c * A @ A
        X = a * X + Bm @ X
    return X.mT if tall else X


def _dir_norm(W, axis):
    if axis == "frobenius":
        return W.norm(dim=(-2, -1), keepdim=True)
    return W.norm(dim=-1, keepdim=True) if axis == "row" else W.norm(dim=-2, keepdim=True)


def _adam(g, m1, m2, step, betas, eps):
    m1.lerp_(g, 1 - betas[0])
    m2.lerp_(g.square(), 1 - betas[1])
    return (m1 / (1 - betas[0] ** step)) / ((m2 / (1 - betas[1] ** step)).sqrt() + eps)


def muonmd_step(W, G, st, lr=0.02, momentum=0.95, gain_lr=1e-3, betas=(0.9, 0.95), eps=1e-10, gain_mode="both",
                norm_axis="frobenius", rescale="balanced"):
    """One magnitude/direction-decoupled Muon step on W (in place)."""
    m, n = W.shape[-2:]
    lead = W.shape[:-2]
    if not st:
        st["mom"] = torch.zeros_like(W)
        if gain_mode in ("row", "both"):
            st["row"] = torch.full(lead + (m,), RAW_GAIN_INIT)
        if gain_mode in ("col", "both"):
            st["col"] = torch.full(lead + (n,), RAW_GAIN_INIT)
        for key in ("row", "col"):
            if key in st:
                st[key + "_m1"], st[key + "_m2"] = torch.zeros_like(st[key]), torch.zeros_like(st[key])
        st["t"] = 0
        st["target"] = _dir_norm(W, norm_axis)
    sr = F.softplus(st["row"]).unsqueeze(-1) if "row" in st else None
    sc = F.softplus(st["col"]).unsqueeze(-2) if "col" in st else None
    g = sr if sc is None else (sc if sr is None else sr * sc)
    What = W if g is None else W / g
    Gh = G if g is None else g * G
    st["mom"].lerp_(Gh, 1 - momentum)
    upd = newton_schulz5(Gh.lerp(st["mom"], momentum)).float()
    upd = upd * (max(1.0, m / n) ** 0.5 if rescale == "muon" else (max(m, n) / min(m, n)) ** 0.5)
    Wn = What - lr * upd
    Wn = Wn * (st["target"] / (_dir_norm(Wn, norm_axis) + 1e-12))
    if g is not None:
        st["t"] += 1
        WG = What * G
        grads = {}
        if sr is not None:
            grads["row"] = (WG * sc if sc is not None else WG).sum(-1) * torch.sigmoid(st["row"])
        if sc is not None:
            grads["col"] = (WG * sr if sr is not None else WG).sum(-2) * torch.sigmoid(st["col"])
        for key, gg in grads.items():
            st[key] -= gain_lr * _adam(gg, st[key + "_m1"], st[key + "_m2"], st["t"], betas, eps)
        sr = F.softplus(st["row"]).unsqueeze(-1) if "row" in st else None
        sc = F.softplus(st["col"]).unsqueeze(-2) if "col" in st else None
        g = sr if sc is None else (sc if sr is None else sr * sc)
        Wn = g * Wn
    W.copy_(Wn)


def adamw_step(W, G, st, lr, wd, betas=(0.9, 0.95), eps=1e-16):
    if not st:
        st["m1"], st["m2"], st["t"] = torch.zeros_like(W), torch.zeros_like(W), 0
    st["t"] += 1
    upd = _adam(G, st["m1"], st["m2"], st["t"], betas, eps)
    W.mul_(1 - lr * wd)
    W.sub_(lr * upd)


def sparse_rows_step(W, G, rows, st, lr=3e-3, beta=0.9, eps=1e-10):
    """GramReaperSparse with unit_norm on the touched rows (G dense, rows = the distinct ids)."""
    if rows.numel() == 0:
        return
    if not st:
        st["v"], st["t"] = torch.zeros(W.shape[0]), 0
    st["t"] += 1
    g = G[rows]
    v = st["v"]
    v[rows] = beta * v[rows] + (1 - beta) * (g * g).sum(dim=1)
    step = lr / ((v[rows] / (1 - beta ** st["t"])).sqrt() + eps)
    r = W[rows] - step.unsqueeze(1) * g
    W[rows] = r / r.norm(dim=1, keepdim=True).clamp_min(eps)


def optimizer_step(P, grads, state, ids):
    """The build_muonmd_optimizer step over all parameters (in place)."""
    for name, W in P.items():
        G = grads[name]
        st = state.setdefault(name, {})
        if name == "embedding.weight":
            sparse_rows_step(W, G, torch.unique(ids), st)
        elif name == "output_layer.weight":
            adamw_step(W, G, st, 3e-4, 0.1)
        elif W.dim() == 1:
            adamw_step(W, G, st, 3e-4, 0.0)
        elif "mlp.gate.weight" in name:
            muonmd_step(W, G, st, gain_mode="col", norm_axis="row", rescale="muon")
        else:
            muonmd_step(W, G, st)


def aux_bias_update(biases, topks, E, rate=1e-3):
    for b, idx in zip(biases, topks):
        cnt = torch.bincount(idx.reshape(-1), minlength=E).float()
        b.add_(rate * torch.sign(cnt.mean() - cnt))


def train_step(P, state, biases, cfg, ids, routing=None, keep=None):
    """One full step in place on (P, state, biases); returns (loss, grads, per-layer top-k)."""
    leaves = {k: v.detach().clone().requires_grad_(True) for k, v in P.items()}
    loss, topks = forward_loss(leaves, cfg, ids, biases, routing, keep)
    loss.backward()
    grads = {k: v.grad.detach().clone() for k, v in leaves.items()}
    with torch.no_grad():
        optimizer_step(P, grads, state, ids)
        aux_bias_update(biases, topks, cfg["n_routed_experts"])
    return loss.detach(), grads, topks


# ------------------------------------------------------------- CPU timing

def _threads():
    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    return torch.get_num_threads()


def time_config1_step(reps=2):
    """Tokens/s of the full config-1 step (4 x 256 tokens) on the host cores."""
    cores = _threads()
    cfg = config1()
    P = canonical_params(cfg, 0)
    state, biases = {}, [torch.zeros(cfg["n_routed_experts"]) for _ in range(cfg["transformer_depth"])]
    ids = canonical_ids(cfg, 4, 256, 1)
    train_step(P, state, biases, cfg, ids)
    t0 = time.perf_counter()
    for _ in range(reps):
        train_step(P, state, biases, cfg, ids)
    dt = (time.perf_counter() - t0) / reps
    return {"value": ids.numel() / dt, "unit": "tokens/s", "cores": cores, "ms_per_step": dt * 1e3,
            "sample": "config 1 full step (4 x 256 tokens: forward, CE, backward, MuonMD/AdamW/sparse-row "
                      "optimizer, bias update) through oracle/model_step.py"}


def _sample_cfg(cfg):
    c = dict(cfg)
    c["transformer_depth"] = 1
    return c


def config4_sample_step(cfg, tokens, ns_rows=1, t_opt=None):
    """Seconds of the config-4 step extrapolated from a bounded sample on the CPU:
      * one transformer layer forward + backward on `tokens` tokens (one sequence), times
        L layers and 32768 / tokens (the per-GPU micro-batch);
      * embedding + final norm + classifier CE forward + backward on the same tokens, times
        32768 / tokens;
      * the optimizer: MuonMD on `ns_rows` matrices of every weight shape of one layer plus
        the head's AdamW rows, scaled to all matrices of all layers by count.
    Returns (seconds per config-4 step, breakdown)."""
    c = _sample_cfg(cfg)
    P = canonical_params(c, 3)
    ids = canonical_ids(c, 1, tokens, 4)
    biases = [torch.zeros(c["n_routed_experts"])]
    leaves = {k: v.detach().clone().requires_grad_(True) for k, v in P.items()}
    t0 = time.perf_counter()
    loss, _ = forward_loss(leaves, c, ids, biases)
    loss.backward()
    t_fb = time.perf_counter() - t0
    # the head part alone, to split layer and head costs
    t0 = time.perf_counter()
    hn = zrms(torch.randn(1, tokens, c["hidden_size"], requires_grad=True), leaves["norm.weight"], c["rms_norm_eps"])
    lg = hn[0] @ leaves["output_layer.weight"].T
    F.cross_entropy(lg, ids[0]).backward()
    t_head = time.perf_counter() - t0
    t_layer = max(t_fb - t_head, 0.0)
    L = cfg["transformer_depth"]
    scale = 32768 / tokens
    total = t_layer * L * scale + t_head * scale
    if t_opt is not None:  # the optimizer's cost measured by an earlier sample
        return total + t_opt, {"layer_fwd_bwd_s": t_layer, "head_fwd_bwd_s": t_head,
                               "optimizer_s_extrapolated": t_opt}
    # optimizer sample
    t_opt = 0.0
    shapes = {}
    for name, W in P.items():
        if W.dim() >= 2 and name not in ("embedding.weight", "output_layer.weight"):
            shapes.setdefault(tuple(W.shape[-2:]), []).append((name, W))
    with torch.no_grad():
        for (m, n), ws in shapes.items():
            count = sum(int(W.numel() // (m * n)) for _, W in ws) * L
            W = ws[0][1].reshape(-1, m, n)[:ns_rows].clone()
            G = torch.randn_like(W) * 1e-3
            t0 = time.perf_counter()
            muonmd_step(W, G, {})
            t_opt += (time.perf_counter() - t0) * count / W.shape[0]
        Wh = P["output_layer.weight"][:4096].clone()
        t0 = time.perf_counter()
        adamw_step(Wh, torch.randn_like(Wh), {}, 3e-4, 0.1)
        t_opt += (time.perf_counter() - t0) * P["output_layer.weight"].shape[0] / 4096
    total = t_layer * L * scale + t_head * scale + t_opt
    return total, {"layer_fwd_bwd_s": t_layer, "head_fwd_bwd_s": t_head, "optimizer_s_extrapolated": t_opt}


def time_config4_sample(cfg, budget_s=25.0):
    """cpu_baseline for bench.py: the config-4 step's tokens/s on the host cores, from one
    bounded sample (config4_sample_step), sized to stay near budget_s."""
    cores = _threads()
    tokens = 512
    t0 = time.perf_counter()
    est, parts = config4_sample_step(cfg, 512)
    if time.perf_counter() - t0 < budget_s / 6:        # a fast host: a longer sequence
        tokens = 2048
        est, parts = config4_sample_step(cfg, tokens)
    return {"value": 32768 / est, "unit": "tokens/s", "cores": cores, "kind": "port",
            "ms_per_step_extrapolated": est * 1e3, "parts": parts,
            "sample": f"config 4 widths, one layer + head forward/backward on {tokens} tokens and MuonMD on one "
                      "matrix per weight shape, extrapolated to 16 layers, 8 x 4096 tokens and all matrices "
                      "(oracle/model_step.py, f32 with bf16 Newton-Schulz); attention cost is scaled linearly "
                      "from the sample's sequence length",
            "config1_step": time_config1_step()}


def reference_arm(cfg, steps, warmup, micro_batch=8):
    """--impl reference: per step one bounded config-4 sample on the host cores; value =
    config-4 tokens/s from the mean extrapolated step time."""
    cores = _threads()
    tokens = 256
    _, parts = config4_sample_step(cfg, tokens)          # also measures the optimizer, once
    t_opt = parts["optimizer_s_extrapolated"]
    for _ in range(max(0, warmup)):
        config4_sample_step(cfg, tokens, t_opt=t_opt)
    ests = []
    wall = time.perf_counter()
    for _ in range(max(1, steps)):
        ests.append(config4_sample_step(cfg, tokens, t_opt=t_opt)[0])
    wall = time.perf_counter() - wall
    est = sum(ests) / len(ests)
    value = micro_batch * 4096 / est
    return {"value": value, "steps": steps, "warmup": warmup, "ms_per_step": est * 1e3, "dtype": "f32",
            "config": {"workload": "config4 full training step (CPU restatement, extrapolated from samples)",
                       "sample_tokens_per_step": tokens, "sample_wall_s": wall},
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                             "sample": f"each step: one config-4 layer + head fwd/bwd on {tokens} tokens, "
                                       "extrapolated to 16 layers x 8 x 4096 tokens, plus the optimizer's time "
                                       "extrapolated once from MuonMD on one matrix per weight shape"},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
