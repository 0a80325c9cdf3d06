"""bf16 copies of f32 master weights, kept in step by the optimizer.

Under bf16 autocast every GEMM of the step reads its weights in bf16: the
reference re-casts (and, for the fused q/k/v/gate projection, re-concatenates)
each f32 weight on every forward.  Here each weight that a GEMM reads gets one
persistent bf16 copy (a *shadow*), cast once; from then on the optimizer's
weight-writing kernels (zs_muonmd_post's write pass, zs_adamw_step) store the
new bf16 values next to the new f32 ones, so no forward casts again.

Validity: a shadow belongs to one parameter and records the parameter's
in-place version and storage pointer when it was last refreshed.  Any torch
in-place change of the parameter (load_state_dict, a torch-op optimizer, user
code) bumps the version, and the next reader refreshes the shadow in place.
The optimizer kernels write parameter and shadow together without touching the
version, which keeps the shadow valid.  Shadows are refreshed in place and
never reallocated, so a CUDA graph that writes them stays correct; `GEN`
counts allocations, and a recorded optimizer step that predates the newest
shadow is recorded again (optimizer.hybrid).

Shadows of weights that are read concatenated (the q/k/v/head-gate rows of
GatedAttention, the shared expert's up/gate rows) are row slices of one bf16
buffer, so the concatenation is never built per step either.
"""
from __future__ import annotations

import torch

GEN = 0   # bumped whenever a shadow buffer is allocated


def _valid(p: torch.Tensor) -> bool:
    sh = getattr(p, "_zs_sh", None)
    return (sh is not None and p._zs_sh_ver == p._version and p._zs_sh_ptr == p.data_ptr())


def _stamp(p: torch.Tensor):
    p._zs_sh_ver = p._version
    p._zs_sh_ptr = p.data_ptr()


def _eligible(p: torch.Tensor) -> bool:
    return (isinstance(p, torch.nn.Parameter) and p.is_cuda and p.dtype == torch.float32 and p.is_contiguous())


def bf16_shadow(p: torch.Tensor) -> torch.Tensor:
    """p's values in bf16 (a persistent copy refreshed only when p changed outside the optimizer
    kernels); a plain cast for tensors that are not contiguous f32 CUDA parameters."""
    if not _eligible(p):
        return p.to(torch.bfloat16)
    global GEN
    sh = getattr(p, "_zs_sh", None)
    if sh is None:
        sh = torch.empty(p.shape, dtype=torch.bfloat16, device=p.device)
        p._zs_sh = sh
        GEN += 1
    elif _valid(p):
        return sh
    with torch.no_grad():
        sh.copy_(p.detach())
    _stamp(p)
    return sh


def concat_shadow(params, pad: int = 0) -> torch.Tensor:
    """bf16 [sum of rows + pad, K] holding the row-concatenation of 2-D weights (zero rows
    after), each weight's shadow being its row slice; rebuilt only when a weight changed
    outside the optimizer kernels."""
    params = list(params)
    if not all(_eligible(p) and p.dim() == 2 for p in params) or len({p.size(1) for p in params}) != 1:
        ws = [p.to(torch.bfloat16) for p in params]
        if pad:
            ws.append(ws[0].new_zeros(pad, ws[0].size(1)))
        return ws[0].contiguous() if len(ws) == 1 else torch.cat(ws, 0)
    global GEN
    key = tuple(id(p) for p in params) + (int(pad),)
    owner = params[0]
    cache = getattr(owner, "_zs_cat", None)
    if cache is None:
        cache = owner._zs_cat = {}
    buf = cache.get(key)
    rows = sum(p.size(0) for p in params)
    if buf is None or buf.size(0) != rows + pad:
        buf = torch.empty(rows + pad, params[0].size(1), dtype=torch.bfloat16, device=owner.device)
        if pad:
            buf[rows:].zero_()
        cache[key] = buf
        GEN += 1
    off = 0
    with torch.no_grad():
        for p in params:
            view = buf[off:off + p.size(0)]
            sh = getattr(p, "_zs_sh", None)
            if sh is None or sh.data_ptr() != view.data_ptr() or sh.shape != view.shape:
                p._zs_sh = view
                p._zs_sh_ver = -1
            if not _valid(p):
                view.copy_(p.detach())
                _stamp(p)
            off += p.size(0)
    return buf


def shadow_ptr(p: torch.Tensor):
    """Device pointer of p's shadow for an optimizer kernel that writes p in place, which then
    stores the new bf16 values there too (None when p has no shadow).  The shadow is marked
    in step with p: the caller's kernel makes it so, in eager mode and on every replay of a
    recorded step."""
    sh = getattr(p, "_zs_sh", None)
    if sh is None or sh.dtype != torch.bfloat16 or sh.shape != p.shape or not sh.is_contiguous():
        return None
    _stamp(p)
    return sh.data_ptr()
