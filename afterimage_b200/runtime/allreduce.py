"""One-shot fp32 all-reduce over NVLink peer memory for the tensor-parallel
decoder's row-parallel projections (csrc/allreduce.cu).

The reference engine runs on one GPU (its layers call nn.Linear on whole
weights, afterimage/runtime/streaming_engine.py:1871-1915), so there is no
reference collective; the alternative here is NCCL's all-reduce. For the
small vectors of a decode step (one token: hidden_size floats) a call is
one kernel: every rank writes each of its partial sums, paired with the
call's number in one 64-bit word, into every peer's receive buffer over
NVLink, then waits in its own buffer for the peers' words of this call and
sums the ranks' values in rank order. Every rank gets bit-identical sums.

Setup is collective: `OneShotAllReduce(group, device, max_floats)` allocates
this rank's buffer, exchanges CUDA IPC handles through the process group
and opens the peers' buffers. All ranks must then make the same calls in
the same order (as for any collective). Waits are bounded; a rank that
gives up sets a status bit that `_device.check_status` raises on.
"""
from __future__ import annotations

import ctypes

import torch

from .. import _lib
from . import _device

# polls before a wait for a peer gives up (~0.5 s with the kernel's backoff):
# far above any healthy step, short enough that a dead peer is reported
DEFAULT_MAX_POLLS = 1 << 22


class OneShotAllReduce:
    def __init__(self, group, device, max_floats: int, max_polls: int = DEFAULT_MAX_POLLS):
        import torch.distributed as dist
        self.device = _device.cuda_device(device)
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if not 1 <= self.world <= _lib.AR_MAX_RANKS:
            raise ValueError(f"one-shot all-reduce supports 1..{_lib.AR_MAX_RANKS} ranks, got {self.world}")
        self.max_floats = int(max_floats)
        self.max_polls = int(max_polls)
        # the ranks' kernels wait on one another: they must run on different GPUs
        uuids = [None] * self.world
        with torch.cuda.device(self.device):
            dist.all_gather_object(uuids, str(torch.cuda.get_device_properties(self.device).uuid), group=group)
        if len(set(uuids)) != self.world:
            raise ValueError("one-shot all-reduce needs one GPU per rank; ranks share a GPU")
        L = _lib.load()
        self._L = L
        self._own = ctypes.c_void_p()
        self._peers: list[int] = []
        with torch.cuda.device(self.device):
            _lib.check(L.aib_ar_alloc(self.max_floats, ctypes.byref(self._own)), "ar_alloc")
            handle = (ctypes.c_uint8 * _lib.AR_HANDLE_BYTES)()
            _lib.check(L.aib_ar_ipc_handle(self._own, handle), "ar_ipc_handle")
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(handle), group=group)
            g = _lib.ArGroup()
            g.rank, g.world, g.max_floats = self.rank, self.world, self.max_floats
            for p, h in enumerate(handles):
                if p == self.rank:
                    g.buffers[p] = self._own.value
                    continue
                ptr = ctypes.c_void_p()
                hb = (ctypes.c_uint8 * _lib.AR_HANDLE_BYTES).from_buffer_copy(h)
                _lib.check(L.aib_ar_ipc_open(hb, ctypes.byref(ptr)), "ar_ipc_open")
                self._peers.append(ptr.value)
                g.buffers[p] = ptr.value
            self._group_desc = g
        # every buffer is zeroed before any rank's first call
        dist.barrier(group=group)

    def __call__(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """Sum of x over the ranks (fp32, contiguous, on this rank's device),
        in place unless `out` is given. Stream-ordered on the current stream."""
        if x.dtype != torch.float32 or not x.is_contiguous() or x.device != self.device:
            raise ValueError("one-shot all-reduce takes a contiguous fp32 tensor on the group's device")
        n = x.numel()
        if n > self.max_floats:
            raise ValueError(f"{n} floats exceed the buffer's {self.max_floats}")
        out = x if out is None else out
        _lib.check(self._L.aib_allreduce_oneshot_f32(
            ctypes.byref(self._group_desc), x.data_ptr(), out.data_ptr(), n, self.max_polls,
            _device.status_word(self.device).data_ptr(), _device.stream_ptr(self.device)), "allreduce_oneshot_f32")
        return out

    def close(self) -> None:
        """Collective: releases the peers' mappings and this rank's buffer
        after every rank has finished its calls."""
        import torch.distributed as dist
        if self._own.value is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for p in self._peers:
                _lib.check(self._L.aib_ar_ipc_close(p), "ar_ipc_close")
            self._peers = []
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            _lib.check(self._L.aib_ar_free(self._own), "ar_free")
        self._own = ctypes.c_void_p()
