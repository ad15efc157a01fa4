"""Symmetric peer-memory heap for the GPUs of one node.

Every rank allocates one device buffer of the same size, exports it with a CUDA IPC
handle and maps every peer's buffer; the handles travel through the process group's
object all-gather.  Buffers carved from the heap in the same order on every rank sit
at the same offset everywhere, so one device table of W pointers per buffer lets a
kernel address any rank's copy.  A slice of the heap holds the flag arrays and the
device-resident epoch of the bounded-wait barrier (``csrc/comm/comm.cu``).

Kernels only read or write peer memory with plain loads and stores; no tensor map
(TMA) is ever built over a peer pointer.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from ..ops import _native as N

DEFAULT_TIMEOUT_NS = 5_000_000_000     # 5 s: a peer that does not arrive by then is reported


class SymBuffer:
    """One symmetric buffer: ``local`` (this rank's tensor view) + ``peers`` (device int64 [W])."""

    def __init__(self, local: torch.Tensor, peers: torch.Tensor, peer_ptrs: list[int]):
        self.local = local
        self.peers = peers
        self.peer_ptrs = peer_ptrs

    def ptr(self) -> int:
        return self.peers.data_ptr()


class PeerGroup:
    def __init__(self, heap_bytes: int, group=None, device=None, timeout_ns: int = DEFAULT_TIMEOUT_NS):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.timeout_ns = timeout_ns
        self.heap = torch.zeros(heap_bytes, dtype=torch.uint8, device=self.device)
        L = N.lib()
        hsz = L.xtu_ipc_handle_size()
        hbuf = ctypes.create_string_buffer(hsz)
        off = ctypes.c_longlong(0)
        rc = L.xtu_ipc_handle(self.heap.data_ptr(), hbuf, ctypes.byref(off))
        if rc != 0:
            raise RuntimeError(f"IPC export of the peer heap failed ({rc})")
        mine = (bytes(hbuf.raw), int(off.value))
        allh = [None] * self.world
        dist.all_gather_object(allh, mine, group=group)
        self._mapped = []
        self.bases = []
        for r, (h, o) in enumerate(allh):
            if r == self.rank:
                self.bases.append(self.heap.data_ptr())
                continue
            p, b = ctypes.c_void_p(), ctypes.c_void_p()
            rc = L.xtu_ipc_open(ctypes.create_string_buffer(h, hsz), o, ctypes.byref(p), ctypes.byref(b))
            if rc != 0:
                self.close()
                raise RuntimeError(f"mapping rank {r}'s peer heap failed ({rc})")
            self._mapped.append(b.value)
            self.bases.append(p.value)
        self._off = 0
        self.flags = self.alloc((self.world,), torch.int32)
        self.epoch = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.status = N.status_buffer(self.device)
        torch.cuda.synchronize(self.device)
        dist.barrier(group=group)

    # ------------------------------------------------------------------ allocation
    def alloc(self, shape, dtype) -> SymBuffer:
        """Carve a buffer from the heap (call in the same order on every rank)."""
        n = 1
        for s in shape:
            n *= s
        nbytes = n * torch.tensor([], dtype=dtype).element_size()
        off = (self._off + 255) & ~255
        if off + nbytes > self.heap.numel():
            raise MemoryError(f"peer heap exhausted: need {off + nbytes} of {self.heap.numel()} bytes")
        self._off = off + nbytes
        local = self.heap[off:off + nbytes].view(dtype).view(*shape)
        ptrs = [b + off for b in self.bases]
        peers = torch.tensor(ptrs, dtype=torch.int64, device=self.device)
        return SymBuffer(local, peers, ptrs)

    @staticmethod
    def heap_bytes_for(*sizes: int) -> int:
        return sum((s + 255) & ~255 for s in sizes) + 4096

    # ------------------------------------------------------------------ collectives
    def barrier(self) -> None:
        """Device-side barrier of all ranks, in stream order (graph-capturable)."""
        N.call("xtu_peer_barrier", self.flags.ptr(), self.epoch.data_ptr(), self.rank, self.world,
               self.status.data_ptr(), self.timeout_ns, N.stream_ptr(self.device))

    def allreduce_(self, buf: SymBuffer, out: torch.Tensor, n: int | None = None) -> torch.Tensor:
        """out = sum over ranks of buf (this rank's input already written to buf.local)."""
        n = buf.local.numel() if n is None else n
        dt = {torch.bfloat16: 0, torch.float32: 1}[buf.local.dtype]
        N.call("xtu_allreduce_oneshot", buf.ptr(), out.data_ptr(), n, dt, self.flags.ptr(), self.epoch.data_ptr(),
               self.rank, self.world, self.status.data_ptr(), self.timeout_ns, N.stream_ptr(self.device))
        return out

    def close(self) -> None:
        L = N.lib()
        for b in self._mapped:
            L.xtu_ipc_close(b)
        self._mapped = []


class P2PAllReduce:
    """All-reduce of tensors up to ``max_numel`` through the peer heap (decode-sized TP
    reductions).  ``__call__`` copies the input into the symmetric buffer and runs the
    one-shot kernel; the copy can be avoided by writing into ``input_buffer`` directly."""

    def __init__(self, pg: PeerGroup, max_numel: int, dtype=torch.bfloat16):
        self.pg = pg
        self.buf = pg.alloc((max_numel,), dtype)

    def input_buffer(self, numel: int) -> torch.Tensor:
        return self.buf.local[:numel]

    def __call__(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        n = x.numel()
        if n > self.buf.local.numel():
            raise ValueError(f"{n} elements exceed the all-reduce buffer ({self.buf.local.numel()})")
        if x.data_ptr() != self.buf.local.data_ptr():
            self.buf.local[:n].copy_(x.reshape(-1))
        y = out if out is not None else torch.empty_like(x)
        self.pg.allreduce_(self.buf, y, n)
        return y
