"""Muon / MuonMD optimizers with the Newton-Schulz orthogonalisation on the
B200 tensor cores and the magnitude/direction bookkeeping fused into three passes.

Same public functions and classes as the reference module (optimizer/muon.py):
zeropower_via_newtonschulz5 (:6-32), muon_update (:35-42), adam_update
(:131-136), md_decoupled_step (:398-508), SingleDeviceMuonMD (:511-571) and
SingleDeviceMuonMDWithAuxAdam (:574-653), with the same arguments, state
layout and defaults.  zeropower_via_newtonschulz5 runs in libzs.so (three
batched tcgen05 GEMMs per iteration with the linear combinations fused into
their epilogues); the magnitude/direction bookkeeping around it runs as the
fused zs_muonmd_pre / zs_muonmd_post passes (f32), and the optimizers batch
the Newton-Schulz launches of same-shape matrices across parameters.  No step
has host syncs, so a whole step can be captured in a CUDA graph.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist
import torch.nn.functional as F

from zs_b200 import _lib as Z
from zs_b200.shadow import shadow_ptr

NS_COEFFS = (3.4445, -4.7750, 2.0315)
_RAW_GAIN_INIT = 0.5413248546129181  # softplus^-1(1): every gain starts at exactly 1


def newton_schulz_flops(batch, m, n, steps):
    """Tensor FLOPs the kernels execute for `steps` iterations on `batch` m x n matrices
    (m <= n): X X^T and A A on 256-row pair tiles compute only the upper triangle of tiles
    when m is a multiple of 256; B X is a full product."""
    if m % 256 == 0:
        t = m // 256
        sym = t * (t + 1) // 2 * 256 * 256
        per = 2.0 * sym * n + 2.0 * sym * m + 2.0 * m * m * n
    else:
        per = 4.0 * m * m * n + 2.0 * m * m * m
    return per * batch * steps


def zeropower_via_newtonschulz5(G: torch.Tensor, steps: int) -> torch.Tensor:
    """Quintic Newton-Schulz orthogonalisation of the trailing two dims of G
    (batched over leading dims), in bf16; returns a bf16 tensor of G's shape."""
    assert G.ndim >= 2
    Z.require_cuda(G)
    X = G.bfloat16()
    tall = G.size(-2) > G.size(-1)
    if tall:
        X = X.mT
    shape = X.shape
    m, n = shape[-2], shape[-1]
    Xc = X.reshape(-1, m, n)
    # Zero rows and columns stay zero through the iteration and change neither
    # X X^T's live block nor the Frobenius norm, so padding to the kernels'
    # 8-element granularity is exact.
    mp, np_ = -(-m // 8) * 8, -(-n // 8) * 8
    if (mp, np_) != (m, n):
        Xc = torch.nn.functional.pad(Xc, (0, np_ - n, 0, mp - m))
    Xc = Xc.contiguous()
    if Xc.data_ptr() % 16:
        Xc = Xc.clone()
    batch = Xc.size(0)
    out = torch.empty_like(Xc)
    ws = torch.empty(int(Z.lib().zs_newton_schulz5_workspace(batch, mp, np_, Z.ZS_BF16)), dtype=torch.uint8,
                     device=G.device)
    a, b, c = NS_COEFFS
    Z.count(1 + 3 * int(steps))
    with Z.timed("newton_schulz5", newton_schulz_flops(batch, mp, np_, steps)):
        Z.check(Z.lib().zs_newton_schulz5(Xc.data_ptr(), out.data_ptr(), batch, mp, np_, int(steps), a, b, c,
                                          ws.data_ptr(), ws.numel(), Z.ZS_BF16, Z.stream_of(Xc)),
                "zs_newton_schulz5")
    if (mp, np_) != (m, n):
        out = out[:, :m, :n]
    out = out.reshape(shape)
    return out.mT if tall else out


def muon_update(grad, momentum, beta=0.95, ns_steps=5, nesterov=True):
    momentum.lerp_(grad, 1 - beta)
    update = grad.lerp_(momentum, beta) if nesterov else momentum
    if update.ndim == 4:
        update = update.view(len(update), -1)
    update = zeropower_via_newtonschulz5(update, steps=ns_steps)
    update *= max(1, grad.size(-2) / grad.size(-1)) ** 0.5
    return update


def adam_update(grad, buf1, buf2, step, betas, eps):
    buf1.lerp_(grad, 1 - betas[0])
    buf2.lerp_(grad.square(), 1 - betas[1])
    c1 = buf1 / (1 - betas[0] ** step)
    c2 = buf2 / (1 - betas[1] ** step)
    return c1 / (c2.sqrt() + eps)


def _scaled_add_(dst, src, lr):
    """dst -= lr * src for a float or a 0-dim tensor lr."""
    if torch.is_tensor(lr):
        dst.sub_(lr * src)
    else:
        dst.add_(src, alpha=-lr)


def _softplus_gains(state):
    """softplus of each raw gain present, as (scalar, row, col) broadcastable views."""
    sc = F.softplus(state["g_scalar"]) if "g_scalar" in state else None
    rw = F.softplus(state["g_row"]) if "g_row" in state else None
    cl = F.softplus(state["g_col"]) if "g_col" in state else None
    return ((sc.reshape(sc.shape + (1, 1)) if sc is not None else None),
            (rw.unsqueeze(-1) if rw is not None else None),
            (cl.unsqueeze(-2) if cl is not None else None))


def _gain_product(parts):
    g = None
    for t in parts:
        if t is not None:
            g = t if g is None else g * t
    return g


def _effective_gain(state):
    return _gain_product(_softplus_gains(state))


def _direction_norm(W, norm_axis):
    if norm_axis == "frobenius":
        return W.norm(dim=(-2, -1), keepdim=True)
    if norm_axis == "row":
        return W.norm(dim=-1, keepdim=True)
    if norm_axis == "col":
        return W.norm(dim=-2, keepdim=True)
    raise ValueError(f"unknown norm_axis {norm_axis!r}")


def _project_to_sphere(W_hat, target_norm, norm_axis):
    return W_hat * (target_norm / (_direction_norm(W_hat, norm_axis) + 1e-12))


def _init_md_state(state, W, gain_mode, norm_axis, capturable):
    *lead, m, n = W.shape
    lead = tuple(lead)
    if gain_mode not in ("none", "scalar", "row", "col", "both"):
        raise ValueError(f"unknown gain_mode {gain_mode!r}")
    state["momentum_buffer"] = torch.zeros_like(W)
    if gain_mode == "scalar":
        state["g_scalar"] = W.new_full(lead, _RAW_GAIN_INIT)
    if gain_mode in ("row", "both"):
        state["g_row"] = W.new_full(lead + (m,), _RAW_GAIN_INIT)
    if gain_mode in ("col", "both"):
        state["g_col"] = W.new_full(lead + (n,), _RAW_GAIN_INIT)
    for key in ("g_scalar", "g_row", "g_col"):
        if key in state:
            state[key + "_m1"] = torch.zeros_like(state[key])
            state[key + "_m2"] = torch.zeros_like(state[key])
    state["gain_step"] = W.new_zeros(()) if capturable else 0
    state["target_norm"] = _direction_norm(W, norm_axis)


def _flat3(t, m, n):
    return t.reshape(-1, m, n)


def _md_pre(p, grad, state, *, momentum, gain_mode, norm_axis, capturable, x_out=None, x_trans=False):
    """Fused first half of the MD step: returns (W f32, gain reductions, X bf16 [..., m, n]).

    W = p (f32 view or copy); buf.lerp_(g*G, 1-momentum); X = lerp(g*G, buf, momentum) in
    bf16 (the Newton-Schulz input); the gain gradients' reductions of (W/g)*G from the old gains.
    x_out: a contiguous bf16 [L, m, n] destination for X (a slice of a Newton-Schulz stack),
    or [L, n, m] with x_trans (X written transposed, the layout a tall stack runs in)."""
    W = p if p.dtype == torch.float32 else p.float()
    G = grad if grad.dtype == torch.float32 else grad.float()
    W, G = W.contiguous(), G.contiguous()
    m, n = W.shape[-2], W.shape[-1]
    if len(state) == 0:
        _init_md_state(state, W, gain_mode, norm_axis, capturable)
    L = W.numel() // (m * n)
    if x_out is None:
        if x_trans:
            raise ValueError("x_trans needs x_out")
        X = torch.empty(W.shape, dtype=torch.bfloat16, device=W.device)
    else:
        want = (L, n, m) if x_trans else (L, m, n)
        if (tuple(x_out.shape) != want or x_out.dtype != torch.bfloat16 or not x_out.is_contiguous()
                or x_out.device != W.device):
            raise Z.ZsError(f"x_out must be a contiguous bf16 {want} tensor on {W.device}")
        X = x_out
    red = {k: torch.empty_like(state[k]) for k in ("g_scalar", "g_row", "g_col") if k in state}
    buf = state["momentum_buffer"]
    ws = torch.empty(int(Z.lib().zs_muonmd_pre_workspace(L, m, n)) if red else 0, dtype=torch.uint8,
                     device=W.device)
    Z.count(1 + len(red))
    Z.check(Z.lib().zs_muonmd_pre(W.data_ptr(), G.data_ptr(), buf.data_ptr(),
                                  Z.ptr(state.get("g_scalar")), Z.ptr(state.get("g_row")), Z.ptr(state.get("g_col")),
                                  X.data_ptr(), int(bool(x_trans)), Z.ptr(red.get("g_scalar")), Z.ptr(red.get("g_row")),
                                  Z.ptr(red.get("g_col")), L, m, n, float(momentum), ws.data_ptr() if red else None,
                                  ws.numel(), Z.stream_of(W)), "zs_muonmd_pre")
    return W, red, X


_AXIS = {"frobenius": 0, "row": 1, "col": 2}


def _md_post(p, W, red, U, state, *, lr, gain_lr, gain_betas, gain_eps, norm_axis, rescale_mode, u_trans=False):
    """Fused second half: W_hat' = W/g - lr*rescale*U projected onto the sphere, gain Adam
    steps from the old gains, p = g_new * W_hat' in p's dtype.  U is [..., m, n], or the
    transposed [L, n, m] with u_trans."""
    if norm_axis not in _AXIS:
        raise ValueError(f"unknown norm_axis {norm_axis!r}")
    m, n = W.shape[-2], W.shape[-1]
    L = W.numel() // (m * n)
    rescale = (max(1.0, m / n) ** 0.5) if rescale_mode == "muon" else (max(m, n) / min(m, n)) ** 0.5
    if red:
        state["gain_step"] += 1
    step = state["gain_step"]
    step_dev = step if torch.is_tensor(step) else None
    if step_dev is not None and step_dev.dtype != torch.float32:
        raise Z.ZsError("gain_step must be a float32 device scalar")
    lr_dev = lr if torch.is_tensor(lr) else None
    if lr_dev is not None:
        lr_dev = lr_dev.to(device=W.device, dtype=torch.float32)
    if u_trans:
        if tuple(U.shape) != (L, n, m) or not U.is_contiguous() or U.dtype != torch.bfloat16:
            raise Z.ZsError(f"a transposed update must be a contiguous bf16 {(L, n, m)} tensor")
    else:
        U = U.contiguous()
    target = state["target_norm"].contiguous()
    direct = p.is_contiguous() and p.dtype in (torch.float32, torch.bfloat16)
    out = p if direct else W
    ws = torch.empty(int(Z.lib().zs_muonmd_post_workspace(L, m, n)), dtype=torch.uint8, device=W.device)
    # the bf16 copy the forward GEMMs read is written with the new weights (zs_b200.shadow)
    sh_ptr = shadow_ptr(p) if (direct and out.dtype == torch.float32) else None
    g = lambda k: state.get(k)  # noqa: E731
    Z.count(4)
    Z.check(Z.lib().zs_muonmd_post(
        W.data_ptr(), U.data_ptr(), int(bool(u_trans)), out.data_ptr(), Z.dtype_code(out.dtype), sh_ptr,
        Z.ptr(g("g_scalar")), Z.ptr(g("g_row")), Z.ptr(g("g_col")),
        Z.ptr(g("g_scalar_m1")), Z.ptr(g("g_scalar_m2")), Z.ptr(g("g_row_m1")), Z.ptr(g("g_row_m2")),
        Z.ptr(g("g_col_m1")), Z.ptr(g("g_col_m2")),
        Z.ptr(red.get("g_scalar")), Z.ptr(red.get("g_row")), Z.ptr(red.get("g_col")),
        Z.ptr(step_dev), float(step) if step_dev is None else 0.0, float(gain_betas[0]), float(gain_betas[1]),
        float(gain_eps), float(gain_lr), Z.ptr(lr_dev), 0.0 if lr_dev is not None else float(lr), float(rescale),
        _AXIS[norm_axis], target.data_ptr(), L, m, n, ws.data_ptr(), ws.numel(), Z.stream_of(W)), "zs_muonmd_post")
    if not direct:
        p.copy_(W.to(p.dtype))


def _world(process_group):
    """(world size, rank) of process_group; (1, 0) when it is None or torch.distributed is not initialised."""
    if process_group is None or not dist.is_available() or not dist.is_initialized():
        return 1, 0
    return dist.get_world_size(process_group), dist.get_rank(process_group)


def _ns_sharded(stack, steps, process_group, ns, async_op=False):
    """Newton-Schulz of the matrices stack[0..b) split over the ranks of process_group:
    rank r orthogonalises matrices [r*per, (r+1)*per) (per = ceil(b / world)), and one
    all_gather_into_tensor assembles the bf16 results on every rank.  Every rank must
    call this with the same stack shape (data-parallel ranks hold the same reduced
    gradients, so the optimizer state and the Newton-Schulz inputs are identical).
    With async_op, returns (result, work): the gather is in flight and work.wait() makes
    the current stream wait for it (work is None when nothing is gathered)."""
    world, rank = _world(process_group)
    if world == 1:
        y = ns(stack, steps)
        return (y, None) if async_op else y
    b = stack.size(0)
    per = -(-b // world)
    lo, hi = min(rank * per, b), min((rank + 1) * per, b)
    mine = torch.zeros((per,) + tuple(stack.shape[1:]), dtype=torch.bfloat16, device=stack.device)
    if hi > lo:
        mine[:hi - lo].copy_(ns(stack[lo:hi], steps))
    full = torch.empty((per * world,) + tuple(stack.shape[1:]), dtype=torch.bfloat16, device=stack.device)
    work = dist.all_gather_into_tensor(full, mine, group=process_group, async_op=async_op)
    return (full[:b], work) if async_op else full[:b]


def _ns_plan(shapes, steps, world):
    """The batched Newton-Schulz launches for matrices stacks of the given (L, m, n) shapes
    and step counts: [(mm, nn, steps, indices)], mm <= nn the oriented shape.  Stacks of one
    oriented shape and step count share a launch; a stack of 32+ matrices per rank fills
    the GPU on its own; smaller ones are merged up to 64 matrices per rank and about 1 GiB
    of Newton-Schulz workspace per rank."""
    groups = {}
    for i, ((L, m, n), st) in enumerate(zip(shapes, steps)):
        groups.setdefault((min(m, n), max(m, n), int(st)), []).append(i)
    plan = []
    for (mm, nn, st), idx in groups.items():
        chunk, batch = [], 0
        for i in idx:
            b = shapes[i][0]
            if b >= 32 * world:
                plan.append((mm, nn, st, [i]))
                continue
            if chunk and (batch + b > 64 * world or (batch + b) * mm * (2 * mm + nn) * 2 > (1 << 30) * world):
                plan.append((mm, nn, st, chunk))
                chunk, batch = [], 0
            chunk.append(i)
            batch += b
        if chunk:
            plan.append((mm, nn, st, chunk))
    return plan


def _zeropower_many(Xs, steps, process_group=None, ns=None):
    """zeropower_via_newtonschulz5 of every tensor in Xs; matrices of one oriented shape
    (and step count) from different tensors share batched launches (_ns_plan).  With a
    process group of more than one rank, each batch is split over the ranks and the
    orthogonalised matrices are all-gathered (_ns_sharded).  `ns` replaces the
    Newton-Schulz function (default: the libzs kernels)."""
    ns = zeropower_via_newtonschulz5 if ns is None else ns
    world, _ = _world(process_group)
    out = [None] * len(Xs)
    shapes = [(X.numel() // (X.shape[-2] * X.shape[-1]), X.shape[-2], X.shape[-1]) for X in Xs]
    for mm, nn, st, chunk in _ns_plan(shapes, steps, world):
        parts = []
        for i in chunk:
            X = Xs[i]
            Xo = X.mT if X.shape[-2] > X.shape[-1] else X
            parts.append(Xo.reshape(-1, mm, nn))
        stack = parts[0] if len(parts) == 1 else torch.cat(parts, 0)
        Y = _ns_sharded(stack, st, process_group, ns)
        off = 0
        for i, part in zip(chunk, parts):
            X = Xs[i]
            b = part.shape[0]
            tall = X.shape[-2] > X.shape[-1]
            y = Y[off:off + b]
            off += b
            y = y.reshape(X.mT.shape if tall else X.shape)
            out[i] = y.mT if tall else y
    return out


@torch.no_grad()
def md_decoupled_step(p, grad, state, *, lr, momentum, gain_lr, gain_betas, gain_eps, gain_mode, norm_axis,
                      ns_steps, capturable=False, rescale_mode="balanced"):
    """One magnitude/direction-decoupled Muon step on p (a matrix or a stack of
    matrices over leading dims), in place; f32 bookkeeping, p's dtype on write.
    Three fused passes (libzs.so) around the tensor-core Newton-Schulz."""
    Z.require_cuda(p, grad)
    W, red, X = _md_pre(p, grad, state, momentum=momentum, gain_mode=gain_mode, norm_axis=norm_axis,
                        capturable=capturable)
    U = zeropower_via_newtonschulz5(X, steps=ns_steps)
    _md_post(p, W, red, U, state, lr=lr, gain_lr=gain_lr, gain_betas=gain_betas, gain_eps=gain_eps,
             norm_axis=norm_axis, rescale_mode=rescale_mode)


def md_decoupled_steps(jobs, states, process_group=None):
    """md_decoupled_step for many parameters at once: jobs = [(p, hyper-parameter dict)].
    Same result per parameter; the Newton-Schulz launches are shared across parameters
    whose matrices have the same shape (_ns_plan).  zs_muonmd_pre writes each parameter's
    Newton-Schulz input straight into its slice of the batch's stack -- transposed for a
    tall stack -- and zs_muonmd_post reads the orthogonalised update from the same place,
    so no stack is assembled, transposed or split by copies.  With a process group, every
    rank runs the element-wise passes on all parameters (their state stays replicated)
    and the Newton-Schulz batches are split over the ranks and all-gathered."""
    world, _ = _world(process_group)
    shapes = []
    for p, hp in jobs:
        Z.require_cuda(p, p.grad)
        m, n = p.shape[-2], p.shape[-1]
        shapes.append((p.numel() // (m * n), m, n))
    def post(chunk, pre, Us, direct, work):
        if work is not None:
            work.wait()   # the stream waits for this batch's all-gather (no host sync)
        for i, (W, red, _), U in zip(chunk, pre, Us):
            p, hp = jobs[i]
            _md_post(p, W, red, U, states[p], lr=hp["lr"], gain_lr=hp["gain_lr"], gain_betas=hp["gain_betas"],
                     gain_eps=hp["gain_eps"], norm_axis=hp["norm_axis"], rescale_mode=hp["rescale_mode"],
                     u_trans=direct and shapes[i][1] > shapes[i][2])

    # With several ranks a batch's all-gather is left in flight while the next batch's
    # element-wise pass and Newton-Schulz are issued; its post pass runs after them.
    pending = None
    for mm, nn, st, chunk in _ns_plan(shapes, [hp["ns_steps"] for _, hp in jobs], world):
        total = sum(shapes[i][0] for i in chunk)
        # the kernels' 8-element granularity: other shapes are padded by the copying path
        direct = mm % 8 == 0 and nn % 8 == 0
        stack = torch.empty(total, mm, nn, dtype=torch.bfloat16, device=jobs[chunk[0]][0].device) if direct else None
        pre, off = [], 0
        for i in chunk:
            p, hp = jobs[i]
            L, m, n = shapes[i]
            x_out = stack[off:off + L] if direct else None
            off += L
            pre.append(_md_pre(p, p.grad, states[p], momentum=hp["momentum"], gain_mode=hp["gain_mode"],
                               norm_axis=hp["norm_axis"], capturable=hp["capturable"], x_out=x_out,
                               x_trans=direct and m > n))
        work = None
        if direct:
            Y, work = _ns_sharded(stack, st, process_group, zeropower_via_newtonschulz5, async_op=True)
            Us, off = [], 0
            for i in chunk:
                Us.append(Y[off:off + shapes[i][0]])
                off += shapes[i][0]
        else:
            Us = _zeropower_many([x for _, _, x in pre], [st] * len(chunk), process_group)
        if pending is not None:
            post(*pending)
        pending = (chunk, pre, Us, direct, work)
    if pending is not None:
        post(*pending)


def _muon_steps(jobs, states, process_group=None):
    """muon_update + the decoupled-weight-decay apply of the reference's Muon optimizers
    (optimizer/muon.py:35-42, :83-93) for jobs = [(p, group)], with the Newton-Schulz
    launches batched across same-shape matrices and, with a process group, split over
    its ranks.  Parameters without a gradient get a zero one, as the reference does."""
    ups = []
    for p, group in jobs:
        if p.grad is None:
            p.grad = torch.zeros_like(p)
        state = states[p]
        if len(state) == 0:
            state["momentum_buffer"] = torch.zeros_like(p)
        buf = state["momentum_buffer"]
        buf.lerp_(p.grad, 1 - group["momentum"])
        u = p.grad.lerp_(buf, group["momentum"])
        ups.append(u.view(len(u), -1) if u.ndim == 4 else u)
    Us = _zeropower_many(ups, [5] * len(ups), process_group)
    for (p, group), U in zip(jobs, Us):
        U *= max(1, p.grad.size(-2) / p.grad.size(-1)) ** 0.5
        p.mul_(1 - group["lr"] * group["weight_decay"])
        _scaled_add_(p, U.reshape(p.shape), group["lr"])


def _adam_fused_ok(params):
    return all(p.is_cuda and p.dtype == torch.float32 and p.is_contiguous() and p.grad is not None
               and not p.grad.is_sparse and p.grad.dtype == torch.float32 and p.grad.is_contiguous()
               for p in params)


def _adamw_fused(group, params, states):
    """One zs_adamw_step launch for every parameter of an aux-Adam group (CUDA f32): the
    state and its layout are the reference's (exp_avg, exp_avg_sq, step), the step
    counters advance first as `state["step"] += 1` does."""
    b1, b2 = group["betas"]
    lr = group["lr"]
    dev_steps, descs = [], []
    for p in params:
        st = states[p]
        if torch.is_tensor(st["step"]):
            dev_steps.append(st["step"])
        else:
            st["step"] += 1
    if dev_steps:
        torch._foreach_add_(dev_steps, 1.0)
    for p in params:
        st = states[p]
        d = Z.AdamWTensor()
        d.p, d.g, d.m1, d.m2 = p.data_ptr(), p.grad.data_ptr(), st["exp_avg"].data_ptr(), st["exp_avg_sq"].data_ptr()
        if torch.is_tensor(st["step"]):
            d.step_dev = st["step"].data_ptr()
        else:
            # torch divides by a Python scalar as a product with its f32 reciprocal
            d.inv_bc1_host = float(np.float32(1.0) / np.float32(1 - b1 ** st["step"]))
            d.inv_bc2_host = float(np.float32(1.0) / np.float32(1 - b2 ** st["step"]))
        d.shadow_bf16 = shadow_ptr(p)
        d.n = p.numel()
        descs.append(d)
    arr = (Z.AdamWTensor * len(descs))(*descs)
    lr_dev = lr.to(device=params[0].device, dtype=torch.float32) if torch.is_tensor(lr) else None
    Z.count(-(-len(descs) // 96))
    Z.check(Z.lib().zs_adamw_step(arr, len(descs), Z.ptr(lr_dev), 0.0 if lr_dev is not None else float(lr),
                                  1.0 if lr_dev is not None else float(1 - lr * group["weight_decay"]), float(b1),
                                  float(b2), 1 - b1, 1 - b2, float(group["eps"]), float(group["weight_decay"]),
                                  Z.stream_of(params[0])), "zs_adamw_step")


def _adam_steps(group, states, capturable=False):
    """AdamW with decoupled weight decay for an aux-Adam group (optimizer/muon.py:226-240,
    :616-650).  CUDA f32 parameters run as one fused launch (zs_adamw_step); anything else
    (CPU tensors, other dtypes) runs the reference's tensor formulation."""
    params = group["params"]
    for p in params:
        if p.grad is None:
            p.grad = torch.zeros_like(p)
        state = states.setdefault(p, {})
        if len(state) == 0:
            state["exp_avg"] = torch.zeros_like(p)
            state["exp_avg_sq"] = torch.zeros_like(p)
            state["step"] = torch.zeros((), dtype=torch.float32, device=p.device) if capturable else 0
    if params and _adam_fused_ok(params):
        _adamw_fused(group, params, states)
        return
    for p in params:
        state = states[p]
        state["step"] += 1
        update = adam_update(p.grad, state["exp_avg"], state["exp_avg_sq"], state["step"], group["betas"],
                             group["eps"])
        p.mul_(1 - group["lr"] * group["weight_decay"])
        _scaled_add_(p, update, group["lr"])


def _muon_group_defaults(group):
    group.setdefault("lr", 0.02)
    group.setdefault("momentum", 0.95)
    group.setdefault("weight_decay", 0)
    assert set(group.keys()) == {"params", "lr", "momentum", "weight_decay", "use_muon"}


def _adam_group_defaults(group):
    group.setdefault("lr", 3e-4)
    group.setdefault("betas", (0.9, 0.95))
    group.setdefault("eps", 1e-10)
    group.setdefault("weight_decay", 0)
    assert set(group.keys()) == {"params", "lr", "betas", "eps", "weight_decay", "use_muon"}


class SingleDeviceMuon(torch.optim.Optimizer):
    """Muon (optimizer/muon.py:100-128): SGD-momentum with Nesterov, Newton-Schulz
    orthogonalised update scaled by sqrt(max(1, rows/cols)), decoupled weight decay."""

    process_group = None

    def __init__(self, params, lr=0.02, weight_decay=0, momentum=0.95):
        super().__init__(params, dict(lr=lr, weight_decay=weight_decay, momentum=momentum))

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        _muon_steps([(p, g) for g in self.param_groups for p in g["params"]], self.state, self.process_group)
        return loss


class Muon(SingleDeviceMuon):
    """Distributed Muon (optimizer/muon.py:45-97), same arguments and result.  The
    reference gives each rank every world-th parameter and all-gathers the updated
    parameters; here every rank keeps the (replicated) momentum of all parameters,
    the Newton-Schulz matrices are split over the ranks in equal slices, and the
    bf16 orthogonalised updates are all-gathered (half the bytes of f32 weights).
    Uses the default process group unless one is given."""

    def __init__(self, params, lr=0.02, weight_decay=0, momentum=0.95, process_group=None):
        assert isinstance(params, list) and len(params) >= 1 and isinstance(params[0], torch.nn.Parameter)
        params = sorted(params, key=lambda x: x.size(), reverse=True)
        super().__init__(params, lr=lr, weight_decay=weight_decay, momentum=momentum)
        self.process_group = dist.group.WORLD if process_group is None else process_group


class SingleDeviceMuonWithAuxAdam(torch.optim.Optimizer):
    """Muon for groups with use_muon=True, AdamW for the rest (optimizer/muon.py:244-336)."""

    process_group = None

    def __init__(self, param_groups):
        for group in param_groups:
            assert "use_muon" in group
            (_muon_group_defaults if group["use_muon"] else _adam_group_defaults)(group)
        super().__init__(param_groups, dict())

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        _muon_steps([(p, g) for g in self.param_groups if g["use_muon"] for p in g["params"]], self.state,
                    self.process_group)
        for group in self.param_groups:
            if not group["use_muon"]:
                _adam_steps(group, self.state)
        return loss


class MuonWithAuxAdam(SingleDeviceMuonWithAuxAdam):
    """Distributed MuonWithAuxAdam (optimizer/muon.py:154-241): Newton-Schulz split over
    the ranks as in Muon; the Adam groups run replicated on every rank."""

    def __init__(self, param_groups, process_group=None):
        for group in param_groups:
            if group.get("use_muon"):
                group["params"] = sorted(group["params"], key=lambda x: x.size(), reverse=True)
        super().__init__(param_groups)
        self.process_group = dist.group.WORLD if process_group is None else process_group


_MD_KEYS = {"params", "lr", "momentum", "gain_lr", "gain_betas", "gain_eps", "gain_mode", "norm_axis", "ns_steps",
            "capturable", "rescale_mode"}


class SingleDeviceMuonMD(torch.optim.Optimizer):
    def __init__(self, params, lr=0.02, momentum=0.95, gain_lr=1e-3, gain_betas=(0.9, 0.95), gain_eps=1e-10,
                 gain_mode="both", norm_axis="frobenius", ns_steps=5, capturable=False, rescale_mode="balanced"):
        super().__init__(params, dict(lr=lr, momentum=momentum, gain_lr=gain_lr, gain_betas=gain_betas,
                                      gain_eps=gain_eps, gain_mode=gain_mode, norm_axis=norm_axis,
                                      ns_steps=ns_steps, capturable=capturable, rescale_mode=rescale_mode))

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        jobs = []
        for group in self.param_groups:
            for p in group["params"]:
                if p.grad is None:
                    continue
                assert p.ndim >= 2, "MD decoupling needs a matrix or a stack of matrices (>=2D)"
                jobs.append((p, group))
        md_decoupled_steps(jobs, self.state, getattr(self, "process_group", None))
        return loss


class SingleDeviceMuonMDWithAuxAdam(torch.optim.Optimizer):
    """MuonMD for groups with use_muon=True, AdamW (decoupled weight decay) for the rest."""

    def __init__(self, param_groups):
        for group in param_groups:
            assert "use_muon" in group
            if group["use_muon"]:
                for k, v in dict(lr=0.02, momentum=0.95, gain_lr=1e-3, gain_betas=(0.9, 0.95), gain_eps=1e-10,
                                 gain_mode="both", norm_axis="frobenius", ns_steps=5, capturable=False,
                                 rescale_mode="balanced").items():
                    group.setdefault(k, v)
                assert set(group.keys()) == _MD_KEYS | {"use_muon"}
            else:
                for k, v in dict(lr=3e-4, betas=(0.9, 0.95), eps=1e-10, weight_decay=0, capturable=False).items():
                    group.setdefault(k, v)
                assert set(group.keys()) == {"params", "lr", "betas", "eps", "weight_decay", "capturable", "use_muon"}
        super().__init__(param_groups, dict())

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        md_decoupled_steps([(p, group) for group in self.param_groups if group["use_muon"]
                            for p in group["params"] if p.grad is not None], self.state,
                           getattr(self, "process_group", None))
        for group in self.param_groups:
            if group["use_muon"]:
                continue
            # parameters without a gradient are skipped (their state does not advance)
            _adam_steps(dict(group, params=[p for p in group["params"] if p.grad is not None]), self.state,
                        capturable=group["capturable"])
        return loss


class MuonMDWithAuxAdam(SingleDeviceMuonMDWithAuxAdam):
    """Data-parallel SingleDeviceMuonMDWithAuxAdam (no counterpart in the reference,
    which trains on one device): the ranks hold identical all-reduced gradients, so
    each keeps the full MuonMD/Adam state and runs the element-wise passes; the
    Newton-Schulz batches -- most of the step's cost -- are split over the ranks and
    the bf16 orthogonalised matrices all-gathered (the ownership + all-gather pattern
    of the reference's distributed Muon, optimizer/muon.py:82-95).  Parameters end
    bit-identical on every rank and to the single-device optimizer."""

    def __init__(self, param_groups, process_group=None):
        super().__init__(param_groups)
        self.process_group = dist.group.WORLD if process_group is None else process_group
