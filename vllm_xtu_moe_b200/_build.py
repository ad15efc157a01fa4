"""In-tree build of the native libraries.

* ``_lib/libxtu_cuda.so``: every ``csrc/cuda/*.cu`` and ``csrc/comm/*.cu``, compiled
  for sm_100a only (``-gencode arch=compute_100a,code=sm_100a``), C ABI, no torch
  headers (Python binds through ctypes, so a rebuild takes seconds).
* ``_lib/libxtu_cpu.so``: the C++17 CPU expert engine (``csrc/cpu``), AVX-512
  paths selected at run time from CPUID, plus a scalar fallback.

Objects are rebuilt only when a source or a header it may include is newer.
Run ``python -m vllm_xtu_moe_b200._build`` (or ``__graft_entry__.build()``).
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
CSRC = ROOT / "csrc"
LIBDIR = Path(__file__).resolve().parent / "_lib"
OBJDIR = ROOT / "build" / "obj"

NVCC = os.environ.get("NVCC", shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc")
CXX = os.environ.get("CXX", shutil.which("g++") or "g++")
CUDA_HOME = Path(NVCC).resolve().parent.parent

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC",
    "-DNDEBUG",
]
CXX_FLAGS = ["-O3", "-std=c++17", "-fPIC", "-DNDEBUG", "-pthread",
             "-ffp-contract=fast", "-fno-math-errno"]


def _newest_header(dirs: list[Path]) -> float:
    t = 0.0
    for d in dirs:
        for h in list(d.glob("*.cuh")) + list(d.glob("*.h")) + list(d.glob("*.hpp")) + list(d.glob("*.inc")):
            t = max(t, h.stat().st_mtime)
    return t


def _compile(cmd: list[str]) -> tuple[list[str], int, str]:
    p = subprocess.run(cmd, capture_output=True, text=True)
    return cmd, p.returncode, p.stdout + p.stderr


AVX512_FLAGS = ["-mavx512f", "-mavx512bw", "-mavx512vl", "-mavx512bf16", "-mavx512vnni", "-mavx512vbmi", "-mfma"]


def _build_lib(name: str, sources: list[Path], compiler: str, flags: list[str], link_flags: list[str],
               include: list[Path], jobs: int, verbose: bool, objdir: Path | None = None) -> Path:
    objdir = objdir or OBJDIR
    objdir.mkdir(parents=True, exist_ok=True)
    LIBDIR.mkdir(parents=True, exist_ok=True)
    hdr_time = _newest_header(include)
    objs, todo = [], []
    for src in sources:
        obj = objdir / (src.parent.name + "_" + src.stem + ".o")
        objs.append(obj)
        if not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, hdr_time):
            extra = AVX512_FLAGS if "avx512" in src.name else []   # ISA kernels: picked at run time
            cmd = [compiler, *flags, *extra, *[f"-I{d}" for d in include], "-c", str(src), "-o", str(obj)]
            todo.append(cmd)
    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
            for cmd, rc, out in ex.map(_compile, todo):
                if verbose or rc != 0:
                    print(" ".join(cmd), file=sys.stderr)
                    if out.strip():
                        print(out, file=sys.stderr)
                if rc != 0:
                    raise RuntimeError(f"compile failed: {cmd[-3]}")
    out = LIBDIR / name
    if todo or not out.exists():
        cmd = [compiler, "-shared", "-o", str(out), *map(str, objs), *link_flags]
        p = subprocess.run(cmd, capture_output=True, text=True)
        if p.returncode != 0:
            print(" ".join(cmd), p.stdout, p.stderr, file=sys.stderr)
            raise RuntimeError(f"link failed: {name}")
    return out


def build_cuda(jobs: int = 8, verbose: bool = False, checked: bool = False) -> Path:
    """The kernel library; ``checked``: the bounds-check build (-DXTU_BOUNDS_CHECK), loaded
    instead of the normal one when XTU_CHECKED=1."""
    srcs = sorted((CSRC / "cuda").glob("*.cu")) + sorted((CSRC / "comm").glob("*.cu"))
    name = "libxtu_cuda_checked.so" if checked else "libxtu_cuda.so"
    flags = NVCC_FLAGS + (["-DXTU_BOUNDS_CHECK"] if checked else [])
    return _build_lib(name, srcs, NVCC, flags, ["-Xcompiler", "-fPIC", "-lcudart"],
                      [CSRC / "cuda", CSRC / "comm", CSRC / "cpu"], jobs, verbose,
                      OBJDIR / "checked" if checked else OBJDIR)


def build_cpu(jobs: int = 8, verbose: bool = False) -> Path:
    srcs = sorted((CSRC / "cpu").glob("*.cpp"))
    cuda_inc = CUDA_HOME / "include"
    flags = CXX_FLAGS + [f"-I{cuda_inc}"]
    link = ["-pthread", f"-L{CUDA_HOME / 'lib64'}", "-lcudart", f"-Wl,-rpath,{CUDA_HOME / 'lib64'}"]
    return _build_lib("libxtu_cpu.so", srcs, CXX, flags, link, [CSRC / "cpu"], jobs, verbose)


def build_all(verbose: bool = False) -> list[Path]:
    jobs = max(1, min(16, os.cpu_count() or 1))
    out = [build_cuda(jobs, verbose), build_cuda(jobs, verbose, checked=True)]
    if list((CSRC / "cpu").glob("*.cpp")):
        out.append(build_cpu(jobs, verbose))
    return out


if __name__ == "__main__":
    for p in build_all(verbose="-v" in sys.argv):
        print(p)
