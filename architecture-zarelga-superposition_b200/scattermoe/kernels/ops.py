"""scattermoe.kernels.ops on the B200 kernels of libzs.so.

Same functions, torch.library op names and schemas as the reference
(scattermoe/kernels/ops.py): rowwise_sum_product (:9-46), scatter2scatter
(:192-255), group_bwd_W / groupXtY (:263-311), group (:449-482).  The Triton
kernels are replaced by the C ABI of include/zs.h; there is no CPU path.

Operand precision: the tensor-core kernels take bf16 or f16.  f32 operands
(the reference's autocast training keeps expert inputs in f32 and runs TF32)
are rounded to bf16 for the contraction; outputs keep the caller's dtype.
"""
from __future__ import annotations

from typing import Optional

import torch

from zs_b200 import _lib as Z

BLOCK_M = 128


def _mma_dtype(*ts):
    dt = ts[0].dtype
    return torch.bfloat16 if dt == torch.float32 else dt


def _as(t, dt):
    return t if t is None or t.dtype == dt else t.to(dt)


# ----------------------------------------------------------- rowwise_sum_product

def rowwise_sum_product(A, B, dtype=None):
    assert A.dim() == 3
    assert B.dim() == 2
    assert A.size(0) == B.size(0)
    assert A.size(2) == B.size(1)
    T, F, H = A.shape
    output = torch.empty((T, F), device=A.device, dtype=dtype or A.dtype)
    rowwise_sum_product_compileable(output, A, B)
    return output


@torch.library.custom_op("scattermoe::rowwise_sum_product", mutates_args={"output"})
def rowwise_sum_product_compileable(output: torch.Tensor, A: torch.Tensor, B: torch.Tensor) -> None:
    Z.require_cuda(output, A, B)
    T, F, H = A.shape
    Z.count(1)
    Z.check(Z.lib().zs_rowwise_sum_product(
        output.data_ptr(), Z.dtype_code(output.dtype), output.stride(0), output.stride(1),
        A.data_ptr(), Z.dtype_code(A.dtype), A.stride(0), A.stride(1), A.stride(2),
        B.data_ptr(), Z.dtype_code(B.dtype), B.stride(0), B.stride(1), T, F, H, Z.stream_of(A)),
        "zs_rowwise_sum_product")


@rowwise_sum_product_compileable.register_fake
def _(output: torch.Tensor, A: torch.Tensor, B: torch.Tensor) -> None:
    return None


# ----------------------------------------------------------------- scatter2scatter

def scatter2scatter(X, W, sorted_expert_idxs, sorted_scattered_idxs, k, b=None, x_grouped=False, y_grouped=False,
                    out=None):
    assert sorted_scattered_idxs.size(0) == sorted_expert_idxs.size(0)
    assert sorted_scattered_idxs.size(0) == X.size(0) * k
    y_dim = W.size(-1)
    L_scattered = sorted_expert_idxs.size(0)
    if out is None:
        output = torch.empty((L_scattered, y_dim), device=X.device, dtype=X.dtype)
    else:
        assert out.size(0) == L_scattered and out.size(1) == y_dim
        output = out
    scatter2scatter_compileable(output, W, X, k, sorted_expert_idxs, sorted_scattered_idxs, b, x_grouped, y_grouped)
    return output


def _launch_scatter2scatter(output, W, X, k, sei, ssi, b, x_grouped, y_grouped, expert_offsets=None,
                            tag="scatter2scatter"):
    Z.require_cuda(output, W, X, sei, ssi, b)
    mdt = _mma_dtype(X)
    Xc = _as(X, mdt)
    if Xc.stride(-1) != 1:
        Xc = Xc.contiguous()
    Wc = _as(W, mdt)
    if not (Wc.stride(1) == 1 or Wc.stride(2) == 1):
        Wc = Wc.contiguous()
    bc = _as(b, mdt)
    out = output if (output.dtype == mdt and output.stride(-1) == 1) else torch.empty(
        output.shape, device=output.device, dtype=mdt)
    sei = sei if sei.dtype == torch.int64 else sei.long()
    ssi = ssi if ssi.dtype == torch.int64 else ssi.long()
    n = sei.numel()
    E, K, N = Wc.shape
    code = Z.dtype_code(mdt)
    ws_bytes = Z.lib().zs_scatter2scatter_workspace(n, K, code, int(bool(x_grouped)))
    ws = torch.empty(max(int(ws_bytes), 1), dtype=torch.uint8, device=X.device)
    Z.count(1 if x_grouped else 2)
    with Z.timed(tag, 2.0 * n * K * N):
      Z.check(Z.lib().zs_scatter2scatter(
        out.data_ptr(), out.stride(0), Wc.data_ptr(), E, K, N, Wc.stride(0), Wc.stride(1), Wc.stride(2),
        Xc.data_ptr(), Xc.size(0), Xc.stride(0),
        Z.ptr(bc), bc.stride(0) if bc is not None else 0, bc.stride(1) if bc is not None else 0,
        int(k), sei.data_ptr(), ssi.data_ptr(), Z.ptr(expert_offsets), n, int(bool(x_grouped)),
        int(bool(y_grouped)), code, ws.data_ptr(), ws.numel(), Z.stream_of(X)), "zs_scatter2scatter")
    if out is not output:
        output.copy_(out)


@torch.library.custom_op("scattermoe::scatter2scatter", mutates_args={"output"})
def scatter2scatter_compileable(output: torch.Tensor, W: torch.Tensor, X: torch.Tensor, k: int,
                                sorted_expert_idxs: torch.Tensor, sorted_scattered_idxs: torch.Tensor,
                                b: Optional[torch.Tensor], x_grouped: bool, y_grouped: bool) -> None:
    _launch_scatter2scatter(output, W, X, k, sorted_expert_idxs, sorted_scattered_idxs, b, x_grouped, y_grouped)


@scatter2scatter_compileable.register_fake
def _(output, W, X, k, sorted_expert_idxs, sorted_scattered_idxs, b, x_grouped, y_grouped) -> None:
    return None


# ------------------------------------------------------------------------ groupXtY

def group_bwd_W(DY, X, expert_offsets, E, has_bias=False, tag="groupXtY"):
    # The kernel writes every element (zeros for experts without rows), so
    # the outputs need no zero fill.
    DWt = torch.empty((E, DY.size(-1), X.size(-1)), device=DY.device, dtype=DY.dtype)
    DW = DWt.permute(0, 2, 1)
    Db = torch.empty((E, DY.size(-1)), device=DY.device, dtype=DY.dtype) if has_bias else None
    with Z.timed(tag, 2.0 * DY.size(0) * DY.size(-1) * X.size(-1)):
        groupXtY_compileable(E, DW, Db, DY, X, expert_offsets)
    return DW, Db


@torch.library.custom_op("scattermoe::groupXtY", mutates_args={"DW"})
def groupXtY_compileable(E: int, DW: torch.Tensor, Db: Optional[torch.Tensor], DY: torch.Tensor, X: torch.Tensor,
                         expert_offsets: torch.Tensor) -> None:
    Z.require_cuda(DW, Db, DY, X, expert_offsets)
    mdt = _mma_dtype(DY)
    DYc = _as(DY, mdt)
    Xc = _as(X, mdt)
    if DYc.stride(-1) != 1:
        DYc = DYc.contiguous()
    if Xc.stride(-1) != 1:
        Xc = Xc.contiguous()
    direct = DW.dtype == mdt and (DW.stride(1) == 1 or DW.stride(2) == 1)
    DWo = DW if direct else torch.empty(DW.shape, device=DW.device, dtype=mdt)
    Dbo = None
    if Db is not None:
        Dbo = Db if Db.dtype == mdt else torch.empty(Db.shape, device=Db.device, dtype=mdt)
    offs = expert_offsets if expert_offsets.dtype == torch.int64 else expert_offsets.long()
    n, K = Xc.shape
    N = DYc.size(1)
    Z.count(1 if Dbo is None else 2)
    Z.check(Z.lib().zs_group_xty(
        int(E), DWo.data_ptr(), DWo.stride(0), DWo.stride(1), DWo.stride(2),
        Z.ptr(Dbo), Dbo.stride(0) if Dbo is not None else 0, Dbo.stride(1) if Dbo is not None else 0,
        DYc.data_ptr(), DYc.stride(0), Xc.data_ptr(), Xc.stride(0), n, K, N, offs.data_ptr(),
        Z.dtype_code(mdt), Z.stream_of(DY)), "zs_group_xty")
    if DWo is not DW:
        DW.copy_(DWo)
    if Db is not None and Dbo is not Db:
        Db.copy_(Dbo)


@groupXtY_compileable.register_fake
def _(E, DW, Db, DY, X, expert_offsets) -> None:
    return None


# --------------------------------------------------------------------------- group

def group(A, sorted_expert_idxs, coeff=None, fan_out=1, out=None):
    N = sorted_expert_idxs.size(0)
    K = A.size(1)
    assert A.size(0) * fan_out == N
    Y = out if out is not None else torch.empty((N, K), dtype=A.dtype, device=A.device)
    group_compileable(A, K, N, Y, coeff, coeff is not None, fan_out, sorted_expert_idxs)
    return Y


@torch.library.custom_op("scattermoe::group", mutates_args={"Y"})
def group_compileable(A: torch.Tensor, K: int, N: int, Y: torch.Tensor, coeff: Optional[torch.Tensor],
                      has_coeff: bool, fan_out: int, sorted_expert_idxs: torch.Tensor) -> None:
    Z.require_cuda(A, Y, coeff, sorted_expert_idxs)
    idx = sorted_expert_idxs if sorted_expert_idxs.dtype == torch.int64 else sorted_expert_idxs.long()
    c = coeff if has_coeff else None
    if c is not None and not c.is_contiguous():
        c = c.contiguous()
    Ac = A if A.dtype == Y.dtype else A.to(Y.dtype)
    if Ac.stride(-1) != 1:
        Ac = Ac.contiguous()
    Z.count(1)
    Z.check(Z.lib().zs_group(
        Ac.data_ptr(), Ac.stride(0), int(K), Y.data_ptr(), Y.stride(0), int(N), Z.ptr(c),
        Z.dtype_code(c.dtype) if c is not None else 0, int(fan_out), idx.data_ptr(), Z.dtype_code(Y.dtype),
        Z.stream_of(A)), "zs_group")


@group_compileable.register_fake
def _(A, K, N, Y, coeff, has_coeff, fan_out, sorted_expert_idxs) -> None:
    return None
