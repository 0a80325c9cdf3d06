"""All-reduce over NVLink peer memory on the copy engines (zs_ce_allreduce).

The data-parallel gradient reduction of the training step runs while the
backward pass's grouped GEMMs hold every SM; NCCL's all-reduce kernels then
compete with them for the SMs and slow them down.  CopyEngineAllReduce moves
every byte with peer copies (copy engines, no SM time) into buffers that all
ranks of the node map through CUDA IPC, and spends SM time only on one short
reduction kernel: rank r sums chunk r of every rank's data in rank order (f32)
and every rank pulls the reduced chunks, so the result is bit-identical on all
ranks.  One instance serves one buffer size and dtype; every rank must create
it and call it in the same order (it is a collective).
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib as Z

_CODE = {torch.bfloat16: Z.ZS_BF16, torch.float32: Z.ZS_F32}


def _export(t: torch.Tensor):
    L = Z.lib()
    h = ctypes.create_string_buffer(int(L.zs_ipc_handle_size()))
    off = ctypes.c_int64(0)
    Z.check(L.zs_ipc_export(t.data_ptr(), ctypes.cast(h, ctypes.c_void_p), ctypes.byref(off)), "zs_ipc_export")
    return h.raw, int(off.value)


class CopyEngineAllReduce:
    def __init__(self, count: int, dtype: torch.dtype, process_group=None, device=None):
        if dtype not in _CODE:
            raise Z.ZsError(f"copy-engine all-reduce supports bf16 and f32 (got {dtype})")
        self.group = dist.group.WORLD if process_group is None else process_group
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        if self.world > 16:
            raise Z.ZsError("copy-engine all-reduce supports up to 16 ranks")
        self.count, self.dtype = int(count), dtype
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.device = dev
        L = Z.lib()
        c = int(L.zs_ce_allreduce_chunk(self.count, self.world))
        self.recv = torch.empty(self.world * c, dtype=dtype, device=dev)
        self.red = torch.empty(c, dtype=dtype, device=dev)
        self.flags = torch.zeros(3 * self.world, dtype=torch.int32, device=dev)
        mine = [_export(t) for t in (self.recv, self.red, self.flags)]
        allh = [None] * self.world
        dist.all_gather_object(allh, mine, group=self.group)
        self._bases = []
        ptrs = [[0] * self.world for _ in range(3)]
        for p in range(self.world):
            for k, t in enumerate((self.recv, self.red, self.flags)):
                if p == self.rank:
                    ptrs[k][p] = t.data_ptr()
                    continue
                h, off = allh[p][k]
                ptr, base = ctypes.c_void_p(), ctypes.c_void_p()
                hb = ctypes.create_string_buffer(h, len(h))
                Z.check(L.zs_ipc_open(ctypes.cast(hb, ctypes.c_void_p), off, dev.index, ctypes.byref(ptr),
                                      ctypes.byref(base)), "zs_ipc_open")
                ptrs[k][p] = ptr.value
                self._bases.append(base.value)
        arr = ctypes.c_void_p * self.world
        self._recv, self._red, self._flags = (arr(*ptrs[0]), arr(*ptrs[1]), arr(*ptrs[2]))
        self.step = 0
        # every rank's flags are zero before any rank may signal into them
        torch.cuda.synchronize(dev)
        dist.barrier(group=self.group)

    def __call__(self, t: torch.Tensor, scale: float = 1.0, stream=None):
        """t <- scale * sum over ranks of t (in place, on `stream`, default the current one)."""
        Z.require_cuda(t)
        if t.numel() != self.count or t.dtype != self.dtype or not t.is_contiguous() or t.data_ptr() % 16:
            raise Z.ZsError("tensor does not match the all-reduce buffers (count, dtype, contiguous, 16-byte aligned)")
        self.step += 1
        s = stream if stream is not None else torch.cuda.current_stream(t.device)
        Z.count(6)
        v = lambda a: ctypes.cast(a, ctypes.c_void_p)  # noqa: E731
        Z.check(Z.lib().zs_ce_allreduce(t.data_ptr(), self.count, _CODE[self.dtype], self.rank, self.world,
                                        v(self._recv), v(self._red), v(self._flags), self.step, float(scale),
                                        ctypes.c_void_p(s.cuda_stream)), "zs_ce_allreduce")
        return t

    def close(self):
        """Unmap the peers' buffers (after every rank's last call has completed)."""
        for b in self._bases:
            Z.lib().zs_ipc_close(b)
        self._bases = []
