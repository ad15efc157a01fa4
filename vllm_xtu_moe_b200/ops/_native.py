"""ctypes binding of ``_lib/libxtu_cuda.so`` (the sm_100a kernels, C ABI).

Every wrapper in :mod:`vllm_xtu_moe_b200.ops` validates shapes, dtypes and
contiguity on the Python side, then passes raw device pointers and the current
CUDA stream.  Kernels report faults they can detect without trapping (timeouts
of bounded waits, bounds checks) through a per-device status word that
:func:`check_status` reads.

On a machine with a GPU the library is mandatory: a missing or stale build
raises instead of silently falling back to PyTorch.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

_LIB_DIR = Path(__file__).resolve().parent.parent / "_lib"
# XTU_CHECKED=1 loads the bounds-check build (device index checks that record
# XTU_ERR_BOUNDS and skip the access; see csrc/cuda/ptx.cuh XTU_IN_BOUNDS)
_CUDA_LIB = _LIB_DIR / ("libxtu_cuda_checked.so" if os.environ.get("XTU_CHECKED", "0") == "1" else "libxtu_cuda.so")

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None

c_int, c_float, c_void_p = ctypes.c_int, ctypes.c_float, ctypes.c_void_p
P = c_void_p  # device pointer / stream handle

# name -> argtypes (all return int status: 0 ok, <0 error)
_SIGS: dict[str, list] = {
    "xtu_status_size": [],
    "xtu_mtile_bytes": [],
    "xtu_gemm_bf16": [P, P, P, c_int, c_int, c_int, c_int, c_int, P, P, P],
    "xtu_gemm_fp8w": [P, P, P, P, c_int, c_int, c_int, c_int, c_int, P, P],
    "xtu_build_mtiles": [P, c_int, P, P, c_int, P],
    "xtu_grouped_gemm": [P, P, P, c_int, P, c_int, c_int, c_int, c_int, c_int, P, P, c_int, c_int, P, P,
                         c_float, c_float, c_float, P, P],
    "xtu_rmsnorm": [P, P, P, P, P, c_int, c_int, c_float, c_int, c_int, c_int, P, P],
    "xtu_rope_kv": [P, P, P, P, P, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, P, P,
                    c_float, c_int, P, P, P, c_int, ctypes.c_longlong, P, c_int, c_float, c_float, P],
    "xtu_paged_attention_fp8": [P, c_int, P, P, P, c_int, P, P, P, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
                                c_int, c_float, c_float, c_float, c_int, P, P, c_int, P, P, P],
    "xtu_dsa_index_scores": [P, c_int, c_int, P, P, P, c_int, P, P, c_int, c_int, c_int, P, ctypes.c_longlong, P,
                             P],
    "xtu_dsa_topk": [P, ctypes.c_longlong, P, P, P, c_int, c_int, c_int, P, P, P],
    "xtu_dsa_gather": [P, c_int, ctypes.c_longlong, P, P, c_int, c_int, c_int, P, P, P],
    "xtu_gate_mul": [P, c_int, c_int, P, c_int, c_int, c_int, c_int, c_int, P],
    "xtu_shared_gate": [P, c_int, P, c_int, P, c_int, c_int, P],
    "xtu_kv_dequant_gather": [P, P, P, c_int, P, P, c_int, c_int, c_int, c_int, c_int, c_float, c_float, P, P, P,
                              c_int, c_int, P, P],
    "xtu_kv_write": [P, P, c_int, c_int, c_int, c_int, c_int, c_int, P, P, P, c_int, ctypes.c_longlong, P, P],
    "xtu_router_topk": [P, P, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_float, P, P, c_int, P],
    "xtu_moe_permute": [P, P, c_int, c_int, c_int, c_int, P, P, P, P, P, P, c_int, c_int, P, c_int, P],
    "xtu_moe_combine": [P, P, c_int, c_int, c_int, c_int, c_int, P, P, P, P, P],
    "xtu_argmax": [P, c_int, c_int, c_int, c_int, P, P, P, P],
    "xtu_embed": [P, P, c_int, c_int, c_int, P, P, P],
    "xtu_embed_host": [P, P, c_int, c_int, c_int, P, P, P],
    "xtu_route_split": [P, c_int, c_int, c_int, P, P, P, P, P],
    "xtu_spec_verify": [P, P, P, c_int, c_int, P, P, P],
    "xtu_quant_fp8_rows": [P, c_int, c_int, c_int, P, P, P],
    "xtu_gemm_fp8_native": [P, P, P, P, P, c_int, P, c_int, c_int, c_int, c_int, c_int, P, P, c_int, c_int, P, P, P,
                            c_float, c_float, c_float, P, c_int, P, P],
    "xtu_spec_chain_meta": [P, P, P, c_int, c_int, c_int, c_int, c_int, P, P, P, P],
    "xtu_deltanet_fwd": [P, c_int, c_int, c_int, P, P, P, c_int, c_int, c_int, c_int, c_int, P, P, P, P, P,
                         P, P, P, P, c_int, c_int, c_int, P, P, c_int, P, P, P, c_int, c_int, P, c_float, P, P, P,
                         c_int, P],
    "xtu_deltanet_spec_commit": [P, P, c_int, c_int, P, P, ctypes.c_longlong, P, P, ctypes.c_longlong, P],
    "xtu_grouped_gemm_ex": [P, P, P, P, c_int, P, c_int, c_int, c_int, c_int, c_int, P, P, c_int, c_int, P, P,
                            c_float, c_float, c_float, P, c_int, P, P],
    "xtu_ipc_handle_size": [],
    "xtu_ipc_handle": [P, P, ctypes.POINTER(ctypes.c_longlong)],
    "xtu_ipc_open": [P, ctypes.c_longlong, ctypes.POINTER(c_void_p), ctypes.POINTER(c_void_p)],
    "xtu_ipc_close": [P],
    "xtu_peer_barrier": [P, P, c_int, c_int, P, ctypes.c_longlong, P],
    "xtu_allreduce_oneshot": [P, P, ctypes.c_longlong, c_int, P, P, c_int, c_int, P, ctypes.c_longlong, P],
    "xtu_allreduce_twoshot": [P, P, ctypes.c_longlong, c_int, P, P, c_int, c_int, P, ctypes.c_longlong, P],
    "xtu_ep_route": [P, c_int, c_int, c_int, c_int, c_int, P, P, P, P, P, P, P, ctypes.c_longlong, P],
    "xtu_ep_dispatch": [P, P, c_int, c_int, c_int, c_int, c_int, P, c_int, c_int, P, P, P, P, P, c_int, P],
    "xtu_silu_mul": [P, c_int, c_int, c_float, c_float, c_float, P, P],
    "xtu_gemv": [P, P, c_int, c_int, c_int, P, c_int, c_int, P, P, c_int, c_int, P, P, P, P],
    "xtu_moe_gemv": [P, P, P, P, c_int, c_int, c_int, c_int, P, c_int, c_int, P, c_int, P, P, P, P, P, c_int, c_int,
                     c_int, P, c_int, c_float, c_float, c_float, P, P, P, P, c_int, P, P, P],
    "xtu_moe_gemv4": [P, P, P, P, P, P, c_int, c_int, c_int, c_int, P, c_int, P, c_int, P, P, P, P, P, c_int, c_int,
                      c_int, P, c_int, c_float, c_float, c_float, P, P],
    "xtu_gemv_tp": [P, P, c_int, c_int, c_int, P, c_int, c_int, P, P, P, ctypes.c_longlong, c_int, c_int, P, P, P, P,
                    P, P],
    "xtu_tp_sum_rmsnorm": [P, ctypes.c_longlong, c_int, c_int, c_int, P, P, P, P, P, P, P, P, c_float, c_int, P,
                           ctypes.c_longlong, P],
    "xtu_moe_permute_decode": [P, P, c_int, c_int, c_int, c_int, P, P, P, P, P, P],
    "xtu_moe_gather_rows": [P, c_int, c_int, c_int, P, P, c_int, c_int, P, c_int, P],
    "xtu_mla_latent_write_fp8": [P, c_int, c_int, c_int, P, ctypes.c_longlong, P, c_float, P, P],
    "xtu_mla_latent_dequant_gather": [P, c_int, P, c_int, P, c_int, c_int, c_int, c_float, P, P, P],
    "xtu_moe_route_decode": [P, c_int, c_int, P, c_int, c_int, P, c_int, c_int, c_int, c_int, c_int, c_float, P, P,
                             P, P, c_int, c_int, P, P, P, P, P, P],
    "xtu_bridge_post": [P, c_int, P, P, c_int, c_int, c_int, c_int, c_int, c_int, P, P, P, P, c_int, c_int, P, P, P],
    "xtu_bridge_wait": [P, P, c_int, c_int, c_int, P, c_int, c_int, c_int, P, ctypes.c_longlong, P, P],
    "xtu_paged_attention": [P, c_int, P, P, c_int, P, c_int, P, P, P, c_int, c_int, c_int, c_int, c_int, c_int,
                            c_int, c_int, c_int, c_int, c_int, c_float, c_int, P, P, c_int, P, P, P],
}


class NativeLibraryMissing(RuntimeError):
    pass


def lib() -> ctypes.CDLL:
    """Load (once) and return the CUDA kernel library."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not _CUDA_LIB.exists():
                raise NativeLibraryMissing(
                    f"{_CUDA_LIB} is not built; run `python -m vllm_xtu_moe_b200._build`")
            L = ctypes.CDLL(str(_CUDA_LIB), mode=ctypes.RTLD_GLOBAL)
            for name, args in _SIGS.items():
                fn = getattr(L, name, None)
                if fn is None:
                    continue
                fn.argtypes = args
                fn.restype = c_int
            _lib = L
    return _lib


def has_symbol(name: str) -> bool:
    try:
        return hasattr(lib(), name)
    except NativeLibraryMissing:
        return False


# kernels of this library enqueued by this process (entry points return their count)
LAUNCHES = {"total": 0}


_SYNC_CALLS = os.environ.get("XTU_SYNC_CALLS", "0") == "1"


def call(name: str, *args) -> int:
    if _SYNC_CALLS:
        return _call_synced(name, *args)
    rc = getattr(lib(), name)(*args)
    if rc < 0:
        raise RuntimeError(f"{name} failed with code {rc}")
    LAUNCHES["total"] += rc
    return rc


def _call_synced(name: str, *args) -> int:
    """Debug mode (XTU_SYNC_CALLS=1): synchronise after every entry point, log its
    duration and raise at the first kernel that recorded an error."""
    import sys
    import time
    torch.cuda.synchronize()
    t = time.perf_counter()
    print(f"[xtu-call] {name} ...", file=sys.stderr, flush=True)
    rc = getattr(lib(), name)(*args)
    if rc < 0:
        raise RuntimeError(f"{name} failed with code {rc}")
    torch.cuda.synchronize()
    print(f"[xtu-call] {name} {1e3 * (time.perf_counter() - t):.2f} ms", file=sys.stderr, flush=True)
    check_status()
    LAUNCHES["total"] += rc
    return rc


def launches() -> int:
    return LAUNCHES["total"]


def add_launches(n: int) -> None:
    """Account kernels replayed from a CUDA graph (captured launches are counted once at capture)."""
    LAUNCHES["total"] += n


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


# ---------------------------------------------------------------------------
# per-device status word
# ---------------------------------------------------------------------------
_status: dict[int, torch.Tensor] = {}

ERROR_NAMES = {1: "mbarrier wait timed out", 2: "peer flag wait timed out",
               3: "host flag wait timed out", 4: "bounds check failed",
               5: "host bridge protocol misuse"}


def status_buffer(device: torch.device | int | None = None) -> torch.Tensor:
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else
                       (device if isinstance(device, int) else (device.index or 0)))
    t = _status.get(dev.index)
    if t is None:
        with torch.inference_mode(False):      # a process-lifetime buffer, not an inference tensor
            t = torch.zeros(4, dtype=torch.int32, device=dev)
        _status[dev.index] = t
    return t


def check_status(device=None, reset: bool = True) -> None:
    """Raise if any kernel on `device` recorded an error since the last check."""
    st = status_buffer(device)
    vals = st.tolist()
    if vals[0] != 0:
        if reset:
            # the buffers may have been made inside an inference-mode region (an engine
            # step); in-place resets of both kinds of tensor are allowed in inference mode
            with torch.inference_mode():
                st.zero_()
                from . import attention, gemm   # a stopped launch may have left counters set
                gemm.gemv_ws_reset(st.device)
                attention.split_counters_reset(st.device)
        raise RuntimeError(
            f"xtu kernel error: {ERROR_NAMES.get(vals[0], vals[0])} (site {vals[1]}, block {vals[2]}, extra {vals[3]})")


def native_required() -> bool:
    """True when the CUDA path must be used (a GPU is present and not overridden)."""
    return torch.cuda.is_available() and os.environ.get("XTU_ALLOW_TORCH_FALLBACK", "0") != "1"
