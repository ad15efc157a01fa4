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


def _scale_shape(fmt: str, rows: int, K: int) -> tuple[tuple, torch.dtype] | None:
    """Per-expert scale tensor shape/dtype in GPU kernel layout."""
    if fmt == "fp8":
        return ((rows + 127) // 128, (K + 127) // 128), torch.float32
    if fmt == "mxfp4":
        return (rows, K // 32), torch.uint8
    if fmt == "nvfp4":
        return (rows, K // 16), torch.float8_e4m3fn
    return None


def alloc_expert_slots(fmt: str, n: int, H: int, I: int, device):
    """n GPU expert slots of one layer (gate/up rows interleaved) as ExpertWeights."""
    from ..ops import moe as M
    wdt = {"bf16": torch.bfloat16, "fp8": torch.float8_e4m3fn}.get(fmt, torch.uint8)
    kdiv = 2 if fmt in ("mxfp4", "nvfp4") else 1
    w13 = torch.empty(n, 2 * I, H // kdiv, dtype=wdt, device=device)
    w2 = torch.empty(n, H, I // kdiv, dtype=wdt, device=device)
    s13 = s2 = gs13 = gs2 = None
    sh13, sh2 = _scale_shape(fmt, 2 * I, H), _scale_shape(fmt, H, I)
    if sh13 is not None:
        s13 = torch.empty(n, *sh13[0], dtype=sh13[1], device=device)
        s2 = torch.empty(n, *sh2[0], dtype=sh2[1], device=device)
    if fmt == "nvfp4":
        gs13 = torch.ones(n, dtype=torch.float32, device=device)
        gs2 = torch.ones(n, dtype=torch.float32, device=device)
    return M.ExpertWeights(fmt, w13, w2, s13, s2, True, gs13, gs2)


def expert_slot_bytes(fmt: str, H: int, I: int) -> int:
    n = 2 * I * _row_bytes(fmt, H) + H * _row_bytes(fmt, I)
    for sh in (_scale_shape(fmt, 2 * I, H), _scale_shape(fmt, H, I)):
        if sh is not None:
            k = 1
            for d in sh[0]:
                k *= d
            n += k * torch.tensor([], dtype=sh[1]).element_size()
    return n + (8 if fmt == "nvfp4" else 0)


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
        self.s13 = self.s2 = self.gs13 = self.gs2 = None
        if gpu_scales:
            pin = torch.cuda.is_available()
            self.s13 = gpu_scales["s13"].contiguous()
            self.s2 = gpu_scales["s2"].contiguous()
            if pin:
                self.s13 = self.s13.pin_memory()
                self.s2 = self.s2.pin_memory()
            if "gs13" in gpu_scales:
                self.gs13, self.gs2 = gpu_scales["gs13"], gpu_scales["gs2"]

    @staticmethod
    def gpu_scales_from_checkpoint(fmt: str, s13: torch.Tensor | None, s2: torch.Tensor | None, gs13=None,
                                   gs2=None) -> dict | None:
        if fmt == "fp8":
            return {"s13": G.interleave_gate_up_scale(s13.float()), "s2": s2.float()}
        if fmt in ("mxfp4", "nvfp4"):    # per-row scales follow the interleaved gate/up rows
            dt = s13.dtype
            out = {"s13": G.interleave_gate_up(s13.view(torch.uint8)).view(dt), "s2": s2}
            if fmt == "nvfp4":
                out["gs13"], out["gs2"] = gs13.float().reshape(-1), gs2.float().reshape(-1)
            return out
        return None

    def copy_slot(self, e: int, slots, i: int, stream: torch.cuda.Stream) -> None:
        """Expert e -> slot i of an ExpertWeights of slots (weights, scales, global scales)."""
        self.copy_expert(e, slots.w13[i], slots.w2[i], slots.s13[i] if slots.s13 is not None else None,
                         slots.s2[i] if slots.s2 is not None else None, stream)
        if slots.gs13 is not None and self.gs13 is not None:
            with torch.cuda.stream(stream):
                slots.gs13[i].fill_(float(self.gs13[e]))
                slots.gs2[i].fill_(float(self.gs2[e]))

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
        return expert_slot_bytes(self.fmt, self.H, self.I)

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
