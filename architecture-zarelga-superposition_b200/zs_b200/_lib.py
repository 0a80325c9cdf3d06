"""ctypes binding of libzs.so, the C ABI declared in include/zs.h.

There is no CPU fallback: every op requires CUDA tensors and the compiled
library, and raises when either is missing.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

_LIB = None
_LOCK = threading.Lock()
LIB_PATH = Path(__file__).resolve().parent / "libzs.so"

ZS_F32, ZS_BF16, ZS_F16 = 0, 1, 2
_DTYPE_CODE = {torch.float32: ZS_F32, torch.bfloat16: ZS_BF16, torch.float16: ZS_F16}

_vp, _i64, _i32, _f32, _sz = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.c_size_t

class AdamWTensor(ctypes.Structure):
    """zs_adamw_tensor (include/zs.h)."""
    _fields_ = [("p", _vp), ("g", _vp), ("m1", _vp), ("m2", _vp), ("step_dev", _vp), ("inv_bc1_host", _f32),
                ("inv_bc2_host", _f32), ("shadow_bf16", _vp), ("n", _i64)]


# name -> (restype, argtypes); mirrors include/zs.h
_SIGNATURES = {
    "zs_version": (_i32, []),
    "zs_error_string": (ctypes.c_char_p, [_i32]),
    "zs_device_error_get": (_i32, [ctypes.POINTER(_i32), _vp]),
    "zs_device_error_clear": (_i32, [_vp]),
    "zs_last_cuda_error": (_i32, []),
    "zs_moe_gate_topk": (_i32, [_vp, _i32, _vp, _i64, _i32, _i32, _vp, _vp, _vp]),
    "zs_moe_gate_topk_backward": (_i32, [_vp, _i32, _vp, _vp, _i32, _i64, _i32, _i32, _vp, _vp]),
    "zs_flatten_sort_count_workspace": (_sz, [_i64, _i32]),
    "zs_flatten_sort_count": (_i32, [_vp, _i64, _i32, _vp, _vp, _vp, _vp, _sz, _vp]),
    "zs_flatten_sort_count_noalloc_max_scratch_ints": (_i64, []),
    "zs_flatten_sort_count_noalloc": (_i32, [_vp, _i64, _i32, _vp, _vp, _vp, _vp]),
    "zs_bincount": (_i32, [_vp, _i64, _i32, _vp, _vp]),
    "zs_expert_counts": (_i32, [_vp, _vp, _i64, _i32, _i32, _vp, _vp]),
    "zs_bias_sign_update": (_i32, [_vp, _i32, _f32, _vp, _vp]),
    "zs_scatter2scatter_workspace": (_sz, [_i64, _i64, _i32, _i32]),
    "zs_scatter2scatter": (_i32, [_vp, _i64, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _i64,
                                  _i64, _i32, _vp, _vp, _vp, _i64, _i32, _i32, _i32, _vp, _sz, _vp]),
    "zs_group_xty": (_i32, [_i32, _vp, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _vp, _i64, _i64, _i64, _i64,
                            _vp, _i32, _vp]),
    "zs_set_gemm_cta_limit": (_i32, [_i32]),
    "zs_group_xty_f32": (_i32, [_i32, _vp, _i64, _i64, _i64, _vp, _i64, _vp, _i64, _i64, _i64, _i64, _vp, _i32,
                                _i32, _vp]),
    "zs_group": (_i32, [_vp, _i64, _i64, _vp, _i64, _i64, _vp, _i32, _i32, _vp, _i32, _vp]),
    "zs_rowwise_sum_product": (_i32, [_vp, _i32, _i64, _i64, _vp, _i32, _i64, _i64, _i64, _vp, _i32, _i64, _i64,
                                      _i64, _i64, _i64, _vp]),
    "zs_gathered_row_sum": (_i32, [_vp, _i64, _vp, _i64, _i64, _vp, _i64, _i32, _i64, _i32, _vp]),
    "zs_weighted_row_sum": (_i32, [_vp, _i64, _vp, _i64, _vp, _i32, _i64, _i32, _i64, _i32, _vp]),
    "zs_expert_up_swiglu": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _vp, _i64, _vp, _vp, _i64, _i32, _vp]),
    "zs_swiglu_backward": (_i32, [_vp, _vp, _vp, _i64, _i64, _i32, _vp]),
    "zs_expert_down_dswiglu": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _vp, _i64, _vp, _vp, _i64, _i32, _vp]),
    "zs_zrmsnorm_forward": (_i32, [_vp, _vp, _vp, _vp, _i64, _i32, _f32, _i32, _i32, _vp]),
    "zs_zrmsnorm_backward_workspace": (_sz, [_i64, _i32]),
    "zs_zrmsnorm_backward": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i32, _i32, _i32, _vp, _sz, _vp]),
    "zs_add_zrmsnorm_forward": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i32, _f32, _vp]),
    "zs_add_zrmsnorm_backward": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i32, _vp, _sz, _vp]),
    "zs_rope_partial": (_i32, [_vp, _i64, _vp, _i64, _vp, _vp, _vp, _vp, _i64] + [_i32] * 10 + [_vp]),
    "zs_rope": (_i32, [_vp, _i64, _vp, _i64, _vp, _vp, _vp, _vp, _i64, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32,
                       _i32, _vp]),
    "zs_attention_forward": (_i32, [_vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _i32, _vp, _vp, _i32,
                                    _f32, _vp]),
    "zs_attention_backward": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32,
                                     _i32, _i32, _vp, _vp, _i32, _vp, _f32, _vp]),
    "zs_attention_sink_grad_workspace": (_sz, [_i32, _i32, _i32, _i32]),
    "zs_attention_sink_grad": (_i32, [_vp, _vp, _i64, _i32, _i32, _i32, _i32, _f32, _vp, _vp, _sz, _vp]),
    "zs_muonmd_pre_workspace": (_sz, [_i64, _i64, _i64]),
    "zs_ipc_handle_size": (_i32, []),
    "zs_ipc_export": (_i32, [_vp, _vp, ctypes.POINTER(_i64)]),
    "zs_ipc_open": (_i32, [_vp, _i64, _i32, ctypes.POINTER(_vp), ctypes.POINTER(_vp)]),
    "zs_ipc_close": (_i32, [_vp]),
    "zs_ce_allreduce_chunk": (_i64, [_i64, _i32]),
    "zs_ce_allreduce": (_i32, [_vp, _i64, _i32, _i32, _i32, _vp, _vp, _vp, _i32, _f32, _vp]),
    "zs_muonmd_pre": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _vp, _vp, _vp, _i64, _i64, _i64, _f32, _vp,
                             _sz, _vp]),
    "zs_muonmd_post_workspace": (_sz, [_i64, _i64, _i64]),
    "zs_adamw_step": (_i32, [_vp, _i32, _vp, _f32, _f32, _f32, _f32, ctypes.c_double, ctypes.c_double, _f32, _f32,
                             _vp]),
    "zs_qk_norm_rope_forward": (_i32, [_vp, _i64, _vp, _vp, _vp, _vp, _i32, _i64, _i32, _i32, _vp, _i64, _vp, _i64,
                                       _i32, _i32, _i32, _i32, _f32, _vp]),
    "zs_qk_norm_rope_backward_workspace": (_sz, [_i32]),
    "zs_qk_norm_rope_backward": (_i32, [_vp, _i64, _vp, _i64, _vp, _vp, _vp, _vp, _i32, _i64, _i32, _i32, _vp, _vp,
                                        _i64, _vp, _vp, _i64, _i32, _i32, _i32, _i32, _vp, _sz, _vp]),
    "zs_gated_attention_forward": (_i32, [_vp, _i64, _vp, _i64, _vp, _i64, _vp, _i64, _vp, _vp, _i64, _i32, _i32,
                                          _i32, _i32, _i32, _i32, _vp, _vp, _i32, _f32, _vp]),
    "zs_gated_attention_backward_workspace": (_sz, [_i32, _i32, _i32, _i32, _i32]),
    "zs_gated_attention_backward": (_i32, [_vp, _i64, _vp, _i64, _vp, _i64, _vp, _i64, _vp, _i64, _vp, _vp, _i64,
                                           _vp, _i64, _vp, _i64, _vp, _i64, _vp, _i64, _i32, _vp, _i32, _i32, _i32,
                                           _i32, _i32, _i32, _vp, _vp, _i32, _vp, _f32, _vp, _sz, _vp]),
    "zs_moe_combine": (_i32, [_vp, _i64, _vp, _i64, _vp, _i32, _i64, _i32, _i64, _i32, _vp, _i64, _vp, _i64, _vp]),
    "zs_muonmd_post": (_i32, [_vp, _vp, _i32, _vp, _i32, _vp] + [_vp] * 12 + [_vp, _f32, _f32, _f32, _f32, _f32, _vp, _f32,
                                                                  _f32, _i32, _vp, _i64, _i64, _i64, _vp, _sz, _vp]),
    "zs_newton_schulz5_workspace": (_sz, [_i64, _i64, _i64, _i32]),
    "zs_newton_schulz5": (_i32, [_vp, _vp, _i64, _i64, _i64, _i32, _f32, _f32, _f32, _vp, _sz, _i32, _vp]),
    "zs_xent_forward_workspace": (_sz, [_i64, _i64]),
    "zs_xent_forward": (_i32, [_vp, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _sz,
                               _i32, _vp]),
    "zs_embedding_bag_forward": (_i32, [_vp, _i64, _i64, _vp, _i64, _i32, _f32, _vp, _vp]),
    "zs_embedding_bag_backward": (_i32, [_vp, _i64, _i32, _i64, _f32, _vp, _vp]),
    "zs_sparse_rmsprop_workspace": (_sz, [_i64, _i64]),
    "zs_sparse_rmsprop_step": (_i32, [_vp, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _i64, _i64, _vp, _f32,
                                      ctypes.c_double, _f32, _i32, _vp, _sz, _vp]),
    "zs_xent_backward_workspace": (_sz, [_i64, _i64, _i32]),
    "zs_xent_backward": (_i32, [_vp, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _i32, _vp, _vp, _vp, _vp, _vp, _vp,
                                _i64, _vp, _sz, _i32, _vp]),
}


class ZsError(RuntimeError):
    pass


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is not None:
        return _LIB
    with _LOCK:
        if _LIB is None:
            if not LIB_PATH.exists():
                raise ZsError(f"{LIB_PATH} is missing: build it with __graft_entry__.build() "
                              "(the zs ops have no CPU fallback)")
            h = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in _SIGNATURES.items():
                fn = getattr(h, name)
                fn.restype = res
                fn.argtypes = args
            _LIB = h
    return _LIB


def exported_symbols():
    return list(_SIGNATURES)


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = lib().zs_error_string(rc).decode()
        extra = ""
        if rc == 5:
            extra = f", CUDA error {lib().zs_last_cuda_error()}"
        raise ZsError(f"{what} failed: {msg} (zs code {rc}{extra})")


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DTYPE_CODE[dt]
    except KeyError:
        raise ZsError(f"unsupported dtype {dt}") from None


def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def require_cuda(*tensors) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ZsError("zs ops run only on CUDA tensors (no CPU fallback); got a tensor on " + str(t.device))


def device_error(device=None) -> int:
    out = ctypes.c_int(0)
    check(lib().zs_device_error_get(ctypes.byref(out), torch.cuda.current_stream(device).cuda_stream),
          "zs_device_error_get")
    return out.value


def clear_device_error(device=None) -> None:
    check(lib().zs_device_error_clear(torch.cuda.current_stream(device).cuda_stream), "zs_device_error_clear")


# ------------------------------------------------------------ instrumentation
# Counters and CUDA-event timers used by bench.py; off by default.

class _Instr:
    launches = 0          # kernels of libzs.so launched through these bindings
    timing = False        # record CUDA events around the instrumented launches
    events = {}           # name -> [(start_event, end_event, flops), ...] of eager launches
    graph_events = {}     # the same for launches recorded into a CUDA graph (re-recorded by every replay)


INSTR = _Instr()


def count(n: int = 1) -> None:
    INSTR.launches += n


class timed:
    """Record a CUDA event pair around a launch when INSTR.timing is set.

    `flops` is the launch's algorithmic work (tensor-core FLOPs) for the roofline.  Inside a
    CUDA-graph capture the events are external event-record nodes of the graph, so every
    replay re-records them; they are kept in INSTR.graph_events (the last replay's times)."""

    __slots__ = ("name", "s", "flops", "graph")

    def __init__(self, name, flops=0.0):
        self.name = name
        self.s = None
        self.flops = float(flops)
        self.graph = False

    def __enter__(self):
        if INSTR.timing:
            self.graph = torch.cuda.is_current_stream_capturing()
            self.s = torch.cuda.Event(enable_timing=True, external=self.graph)
            self.s.record()
        return self

    def __exit__(self, *exc):
        if self.s is not None:
            e = torch.cuda.Event(enable_timing=True, external=self.graph)
            e.record()
            (INSTR.graph_events if self.graph else INSTR.events).setdefault(self.name, []).append(
                (self.s, e, self.flops))
        return False
