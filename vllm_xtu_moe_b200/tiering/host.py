"""Host tier of one MoE layer: the CPU engine (single NUMA-sharded weight copy) plus
the DMA plumbing that moves experts from that copy into GPU slots.

The engine stores each node's gate/up rows in the GPU kernels' interleaved order
(per 128-column block: 128 gate rows, then 128 up rows) and its down rows in
checkpoint order, so expert e's slice on node n is one contiguous range for each
matrix.  ``copy_expert`` issues one ``cudaMemcpyAsync`` per (matrix, node) from the
page-locked engine shards straight into a slot -- host DRAM holds one copy that serves
both the CPU compute and the GPU streaming (the reference's
``kmajor_from_engine_shards``, vllm_xiaotu_moe/gpu_prefill.py:1997-2253, without the
on-GPU byte transpose its layout needed).  Block scales, ~1-6% of the bytes, are kept
in GPU layout in a separate pinned tensor.
"""
from __future__ import annotations

import ctypes

import torch

from ..ops import gemm as G
from .cpu_engine import CpuExpertEngine, lib

def _h2d():
    f = lib().xtu_memcpy_h2d_async
    f.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_longlong, ctypes.c_void_p]
    f.restype = ctypes.c_int
    return f


def _row_bytes(fmt: str, K: int) -> int:
    return {"bf16": 2 * K, "fp8": K}.get(fmt, K // 2)


class HostExperts:
    """One layer's routed experts held by a CpuExpertEngine, DMA-able into GPU slots."""

    def __init__(self, engine: CpuExpertEngine, gpu_scales: dict | None, register: bool = True):
        self.engine = engine
        self.fmt = engine.fmt
        self.E, self.H, self.I = engine.E, engine.H, engine.I
        self.shards = []
        L = lib()
        L.xtu_cpu_engine_shard.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_void_p),
                                           ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_longlong)]
        L.xtu_cpu_engine_shard.restype = ctypes.c_int
        L.xtu_host_register.argtypes = [ctypes.c_void_p, ctypes.c_longlong]
        L.xtu_host_register.restype = ctypes.c_int
        L.xtu_host_unregister.argtypes = [ctypes.c_void_p]
        for n in range(engine.info()["numa_nodes"]):
            ptrs = (ctypes.c_void_p * 4)()
            rng = (ctypes.c_int * 4)()
            nb = (ctypes.c_longlong * 4)()
            if L.xtu_cpu_engine_shard(engine._h, n, ptrs, rng, nb) != 0:
                break
            self.shards.append(dict(w13=ptrs[0], w2=ptrs[2], j0=rng[0], j1=rng[1], h0=rng[2], h1=rng[3],
                                    w13_bytes=nb[0], w2_bytes=nb[2]))
        self.registered = []
        if register and torch.cuda.is_available():
            for sh in self.shards:
                for key in ("w13", "w2"):
                    if sh[key] and L.xtu_host_register(sh[key], sh[key + "_bytes"]) == 0:
                        self.registered.append(sh[key])
        # scales in GPU layout (pinned): fp8 [E, 2I/128, H/128] interleaved + [E, H/128, I/128]
        self.s13 = self.s2 = None
        if gpu_scales:
            pin = torch.cuda.is_available()
            self.s13 = gpu_scales["s13"].contiguous()
            self.s2 = gpu_scales["s2"].contiguous()
            if pin:
                self.s13 = self.s13.pin_memory()
                self.s2 = self.s2.pin_memory()

    @staticmethod
    def gpu_scales_from_checkpoint(fmt: str, s13: torch.Tensor | None, s2: torch.Tensor | None) -> dict | None:
        if fmt == "fp8":
            return {"s13": G.interleave_gate_up_scale(s13.float()), "s2": s2.float()}
        return None

    def copy_expert(self, e: int, w13_dst: torch.Tensor, w2_dst: torch.Tensor, s13_dst: torch.Tensor | None,
                    s2_dst: torch.Tensor | None, stream: torch.cuda.Stream) -> None:
        """Expert e -> GPU slot tensors (w13 [2I, H], w2 [H, I], scales), on `stream`."""
        cp = _h2d()
        s = stream.cuda_stream
        rb13, rb2 = _row_bytes(self.fmt, self.H), _row_bytes(self.fmt, self.I)
        for sh in self.shards:
            jn = sh["j1"] - sh["j0"]
            if jn > 0:
                src = sh["w13"] + e * 2 * jn * rb13
                dst = w13_dst.data_ptr() + sh["j0"] * 2 * rb13
                rc = cp(dst, src, 2 * jn * rb13, s)
                if rc:
                    raise RuntimeError(f"cudaMemcpyAsync failed ({rc})")
            hn = sh["h1"] - sh["h0"]
            if hn > 0:
                src = sh["w2"] + e * hn * rb2
                dst = w2_dst.data_ptr() + sh["h0"] * rb2
                rc = cp(dst, src, hn * rb2, s)
                if rc:
                    raise RuntimeError(f"cudaMemcpyAsync failed ({rc})")
        with torch.cuda.stream(stream):
            if s13_dst is not None and self.s13 is not None:
                s13_dst.copy_(self.s13[e], non_blocking=True)
                s2_dst.copy_(self.s2[e], non_blocking=True)

    def expert_bytes(self) -> int:
        return 2 * self.I * _row_bytes(self.fmt, self.H) + self.H * _row_bytes(self.fmt, self.I)

    def close(self):
        """Unregister the engine's shards (must happen before the engine frees them)."""
        if self.registered:
            L = lib()
            for p in self.registered:
                L.xtu_host_unregister(p)
            self.registered = []

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
