"""Python side of the C++ CPU expert engine (``csrc/cpu``).

``CpuExpertEngine`` takes one layer's routed experts in checkpoint layout (host
tensors), copies them into engine-owned NUMA-sharded memory, and can then drop
the caller's copy (single weight copy in host DRAM, like the reference's
``_release_source_weights``, vllm_xiaotu_moe/mixed_experts.py:913-992).

``forward`` runs on host tensors; ``CpuBridge`` enqueues the same computation on a
CUDA stream (D2H of activations/ids/weights -> host function -> H2D of the fp32
partial), which is graph-capturable and overlaps the GPU experts when issued on a
side stream.  ``ShmEpGroup`` is the /dev/shm partial-sum reduction between CPU
ranks (CPU-only expert parallelism).
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

_LIB = Path(__file__).resolve().parent.parent / "_lib" / "libxtu_cpu.so"
_lock = threading.Lock()
_lib = None

FMT = {"bf16": 0, "fp8": 1, "mxfp4": 2, "nvfp4": 3, "int4": 4}
P, I_, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not _LIB.exists():
                    raise RuntimeError(f"{_LIB} is not built; run `python -m vllm_xtu_moe_b200._build`")
                L = ctypes.CDLL(str(_LIB))
                L.xtu_cpu_engine_create.restype = P
                L.xtu_cpu_engine_create.argtypes = [I_, I_, I_, I_, P, P, P, P, P, P, I_, F, F, F, I_, I_, I_]
                L.xtu_cpu_engine_forward.restype = I_
                L.xtu_cpu_engine_forward.argtypes = [P, I_, I_, P, P, P, P, I_, I_]
                L.xtu_cpu_engine_info.restype = I_
                L.xtu_cpu_engine_info.argtypes = [P, ctypes.POINTER(ctypes.c_longlong)]
                L.xtu_cpu_engine_destroy.argtypes = [P]
                L.xtu_cpu_e4m3_to_f32.restype = F
                L.xtu_cpu_e4m3_to_f32.argtypes = [I_]
                L.xtu_cpu_quant_s8.restype = I_
                L.xtu_cpu_quant_s8.argtypes = [P, I_, P, P]
                L.xtu_cpu_bridge_create.restype = P
                L.xtu_cpu_bridge_create.argtypes = [P, I_, I_, I_]
                L.xtu_cpu_bridge_enqueue.restype = I_
                L.xtu_cpu_bridge_enqueue.argtypes = [P, P, I_, P, I_, P, P, P, I_, I_]
                L.xtu_cpu_bridge_stats.restype = I_
                L.xtu_cpu_bridge_stats.argtypes = [P, ctypes.POINTER(ctypes.c_longlong)]
                L.xtu_cpu_bridge_destroy.argtypes = [P]
                L.xtu_async_bridge_create.restype = P
                L.xtu_async_bridge_create.argtypes = [P, I_, I_, I_, I_, I_]
                for name in ("xtu_async_bridge_ptrs", "xtu_async_bridge_stats", "xtu_async_bridge_pause",
                             "xtu_async_bridge_reset", "xtu_async_bridge_add_engine"):
                    getattr(L, name).restype = I_
                L.xtu_async_bridge_ptrs.argtypes = [P, ctypes.POINTER(P)]
                L.xtu_async_bridge_stats.argtypes = [P, ctypes.POINTER(ctypes.c_longlong)]
                L.xtu_async_bridge_pause.argtypes = [P, I_]
                L.xtu_async_bridge_reset.argtypes = [P]
                L.xtu_async_bridge_add_engine.argtypes = [P, P]
                L.xtu_async_bridge_destroy.argtypes = [P]
                L.xtu_shm_ep_open.restype = P
                L.xtu_shm_ep_open.argtypes = [ctypes.c_char_p, I_, I_, I_, I_, I_]
                L.xtu_shm_ep_allreduce.restype = I_
                L.xtu_shm_ep_allreduce.argtypes = [P, P, I_, I_]
                L.xtu_shm_ep_close.argtypes = [P, I_]
                _lib = L
    return _lib


def _p(t: torch.Tensor | None):
    return None if t is None else t.data_ptr()


class CpuExpertEngine:
    """Routed experts of one layer on the CPU (fmt: bf16 | fp8 | mxfp4 | nvfp4).

    w13 [E, 2I, H] (gate rows then up rows) and w2 [E, H, I] in the checkpoint format;
    s13/s2 the matching scales; gs13/gs2 the NVFP4 per-expert global scales.
    int8_mode: 0 off, 1 on, 2 auto (MXFP4 only; on when M >= int8_min_tokens).
    """

    def __init__(self, fmt: str, w13: torch.Tensor, w2: torch.Tensor, s13=None, s2=None, gs13=None, gs2=None, *,
                 threads: int = 0, act_limit: float = 0.0, act_alpha: float = 1.0, act_beta: float = 0.0,
                 int8_mode: int = 2, int8_min_tokens: int = 160, deadline_ms: int = 300000):
        self.fmt = fmt
        self.E, two_i = w13.shape[0], w13.shape[1]
        self.I = two_i // 2
        self.H = w2.shape[1]
        ts = [t.detach().contiguous().cpu() if t is not None else None for t in (w13, w2, s13, s2, gs13, gs2)]
        w13c, w2c, s13c, s2c, gs13c, gs2c = ts
        if fmt in ("fp8", "int4"):
            s13c, s2c = s13c.float().contiguous(), s2c.float().contiguous()
        if fmt == "int4" and (self.H % 128 or self.I % 128):
            raise ValueError("INT4 experts need H and I in multiples of the 128-wide quantization group")
        if gs13c is not None:
            gs13c = gs13c.float().reshape(-1)
            gs2c = gs2c.float().reshape(-1)
        h = lib().xtu_cpu_engine_create(FMT[fmt], self.E, self.H, self.I, _p(w13c), _p(s13c), _p(w2c), _p(s2c),
                                        _p(gs13c), _p(gs2c), threads, act_limit, act_alpha, act_beta, int8_mode,
                                        int8_min_tokens, deadline_ms)
        if not h:
            raise RuntimeError("CPU expert engine creation failed (H and I must be multiples of 16)")
        self._h = h
        self.act = (act_limit, act_alpha, act_beta)

    def info(self) -> dict:
        arr = (ctypes.c_longlong * 5)()
        lib().xtu_cpu_engine_info(self._h, arr)
        return {"bytes": arr[0], "numa_nodes": arr[1], "threads": arr[2], "avx512": bool(arr[3]),
                "deadline_exceeded": bool(arr[4])}

    def forward(self, x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor, lo: int = 0, hi: int | None = None,
                out: torch.Tensor | None = None) -> torch.Tensor:
        """x [M, H] bf16 (host), ids/weights [M, K] -> fp32 [M, H] partial over experts [lo, hi)."""
        M, K = ids.shape
        hi = lo + self.E if hi is None else hi
        x = x.contiguous()
        if x.dtype != torch.bfloat16:
            x = x.to(torch.bfloat16)
        ids = ids.contiguous().to(torch.int32)
        weights = weights.contiguous().float()
        y = out if out is not None else torch.empty(M, self.H, dtype=torch.float32)
        rc = lib().xtu_cpu_engine_forward(self._h, M, K, ids.data_ptr(), weights.data_ptr(), x.data_ptr(),
                                          y.data_ptr(), lo, hi)
        if rc < 0:
            raise RuntimeError(f"CPU engine forward failed ({rc})")
        return y

    def close(self):
        if getattr(self, "_h", None):
            lib().xtu_cpu_engine_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class CpuBridge:
    """Stream-ordered (and CUDA-graph capturable) CPU-expert call for one engine."""

    def __init__(self, engine: CpuExpertEngine, top_k: int, max_tokens: int):
        self.engine = engine
        self.top_k = top_k
        self.max_tokens = max_tokens
        self._h = lib().xtu_cpu_bridge_create(engine._h, engine.H, top_k, max_tokens)
        if not self._h:
            raise RuntimeError("pinned staging allocation for the CPU bridge failed")

    def enqueue(self, x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor, out: torch.Tensor, lo: int, hi: int,
                stream: torch.cuda.Stream | None = None) -> None:
        M = ids.shape[0]
        s = (stream or torch.cuda.current_stream()).cuda_stream
        rc = lib().xtu_cpu_bridge_enqueue(self._h, s, M, x.data_ptr(), x.stride(0), ids.data_ptr(),
                                          weights.data_ptr(), out.data_ptr(), lo, hi)
        if rc < 0:
            raise RuntimeError(f"CPU bridge enqueue failed ({rc})")

    def stats(self) -> dict:
        arr = (ctypes.c_longlong * 2)()
        lib().xtu_cpu_bridge_stats(self._h, arr)
        return {"runs": arr[0], "pairs": arr[1]}

    def close(self):
        if getattr(self, "_h", None):
            lib().xtu_cpu_bridge_destroy(self._h)
            self._h = None


class AsyncCpuBridge:
    """CPU-expert calls through a polling worker thread instead of a host-function node.

    ``post`` launches one kernel that writes the inputs into a pinned, mapped slot and
    publishes the request; ``wait`` launches one kernel that waits (bounded) for the
    worker's result and copies or adds it into a device fp32 buffer.  Requests are read
    back in the order they were posted, at most ``slots`` outstanding; both kernels keep
    their request numbers on the device, so a captured post/wait sequence replays from a
    CUDA graph.  This is the reference's ``XIAOTU_MOE_ASYNC`` path (mapped flags polled by
    one worker thread, xiaotu_moe/csrc/python_binding/binding.cpp:339-430) and the
    mechanism of expert deferral (a layer's request is read back one layer later)."""

    def __init__(self, engine: CpuExpertEngine, top_k: int, max_tokens: int, slots: int = 2,
                 spin_idle_us: int = 50, timeout_ms: int = 20000, device=None):
        self.engine, self.top_k, self.max_tokens, self.slots = engine, top_k, max_tokens, slots
        self.timeout_ns = int(timeout_ms) * 1_000_000
        self.H = engine.H
        self._h = lib().xtu_async_bridge_create(engine._h, engine.H, top_k, max_tokens, slots, spin_idle_us)
        if not self._h:
            raise RuntimeError("mapped pinned allocation for the async CPU bridge failed")
        ptrs = (P * 5)()
        lib().xtu_async_bridge_ptrs(self._h, ptrs)
        self._ctl, self._hx, self._hids, self._hw, self._hout = (ptrs[i] for i in range(5))
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.counters = torch.zeros(4, dtype=torch.int32, device=self.device)   # posted, consumed, 2 arrivals
        self.engines = [engine]

    def add_engine(self, engine: CpuExpertEngine) -> int:
        """Let requests run on another engine (one worker serves every tiered layer)."""
        assert engine.H == self.H
        i = lib().xtu_async_bridge_add_engine(self._h, engine._h)
        if i < 0:
            raise RuntimeError("async CPU bridge: engine table full")
        self.engines.append(engine)
        return i

    def post(self, x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor, engine: int = 0, lo: int = 0,
             hi: int | None = None, stream: torch.cuda.Stream | None = None) -> None:
        from ..ops import _native as N
        M = ids.shape[0]
        hi = self.engines[engine].E if hi is None else hi
        assert x.dtype == torch.bfloat16 and x.stride(1) == 1 and ids.is_contiguous() and weights.is_contiguous()
        assert ids.dtype == torch.int32 and weights.dtype == torch.float32 and ids.shape[1] == self.top_k
        s = (stream or torch.cuda.current_stream(self.device)).cuda_stream
        N.call("xtu_bridge_post", x.data_ptr(), x.stride(0), ids.data_ptr(), weights.data_ptr(), M, self.H,
               self.top_k, lo, hi, engine, self._ctl, self._hx, self._hids, self._hw, self.slots, self.max_tokens,
               self.counters.data_ptr(), N.status_buffer(self.device).data_ptr(), s)

    def wait(self, out: torch.Tensor, accumulate: bool = False, stream: torch.cuda.Stream | None = None) -> None:
        from ..ops import _native as N
        assert out.dtype == torch.float32 and out.stride(1) == 1 and out.shape[1] == self.H
        s = (stream or torch.cuda.current_stream(self.device)).cuda_stream
        N.call("xtu_bridge_wait", self._ctl, self._hout, self.slots, self.max_tokens, self.H, out.data_ptr(),
               out.stride(0), out.shape[0], int(accumulate), self.counters.data_ptr(), self.timeout_ns,
               N.status_buffer(self.device).data_ptr(), s)

    def pending(self) -> int:
        """Requests posted and not read back (synchronises the device)."""
        c = self.counters.tolist()
        return c[0] - c[1]

    def pause(self, paused: bool = True) -> None:
        if lib().xtu_async_bridge_pause(self._h, int(paused)) < 0:
            raise TimeoutError("the async bridge worker did not park")

    def reset(self) -> None:
        """Drop every request on both sides (after a wait ran out of time).  Synchronises."""
        torch.cuda.synchronize(self.device)
        self.pause(True)
        if lib().xtu_async_bridge_reset(self._h) < 0:
            raise RuntimeError("async bridge reset failed")
        self.counters.zero_()
        torch.cuda.synchronize(self.device)
        self.pause(False)

    def stats(self) -> dict:
        arr = (ctypes.c_longlong * 5)()
        lib().xtu_async_bridge_stats(self._h, arr)
        return {"runs": arr[0], "pairs": arr[1], "busy_ms": arr[2] / 1e6, "req": arr[3], "done": arr[4]}

    def close(self):
        if getattr(self, "_h", None):
            lib().xtu_async_bridge_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class ShmEpGroup:
    """Sum of fp32 partials across CPU ranks on one host through /dev/shm, with bounded waits."""

    def __init__(self, name: str, rank: int, world: int, nfloats: int, timeout_ms: int = 10000):
        self.name = name if name.startswith("/") else "/" + name
        self.rank, self.world, self.nfloats, self.timeout_ms = rank, world, nfloats, timeout_ms
        self._h = lib().xtu_shm_ep_open(self.name.encode(), rank, world, nfloats, int(rank == 0), timeout_ms)
        if not self._h:
            raise TimeoutError(f"could not open shared segment {self.name}")

    def allreduce_(self, t: torch.Tensor) -> torch.Tensor:
        assert t.dtype == torch.float32 and t.is_contiguous() and not t.is_cuda
        rc = lib().xtu_shm_ep_allreduce(self._h, t.data_ptr(), t.numel(), self.timeout_ms)
        if rc == -2:
            raise TimeoutError("shm EP reduction timed out (a peer rank is missing)")
        if rc < 0:
            raise RuntimeError(f"shm EP reduction failed ({rc})")
        return t

    def close(self, unlink: bool | None = None):
        if getattr(self, "_h", None):
            lib().xtu_shm_ep_close(self._h, int(self.rank == 0 if unlink is None else unlink))
            self._h = None
