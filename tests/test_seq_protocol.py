"""The asynchronous CPU-bridge handshake (csrc/cpu/seq_protocol.hpp) on the host only: a
three-thread simulator (tests/cpp/seq_protocol_sim.cpp) drives the same slot arithmetic
and the same worker step the library uses, with random stalls, and checks for lost
requests, deadlocks, early slot reuse and out-of-order read-back.  The reference keeps a
model of its handshake the same way (tests/test_seq_protocol.cpp:1-308)."""
from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _build(tmp_path, sanitize: str | None = None) -> Path:
    cxx = shutil.which("g++")
    if cxx is None:
        pytest.skip("no g++")
    exe = tmp_path / ("seq_sim_" + (sanitize or "plain").replace(",", "_"))
    cmd = [cxx, "-std=c++17", "-O1", "-g", "-pthread", f"-I{ROOT / 'csrc' / 'cpu'}",
           str(ROOT / "tests" / "cpp" / "seq_protocol_sim.cpp"), "-o", str(exe)]
    if sanitize:
        cmd.insert(1, f"-fsanitize={sanitize}")
    b = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
    if b.returncode != 0 and sanitize and "cannot find" in b.stderr.lower():
        pytest.skip("sanitizer runtime not installed")
    assert b.returncode == 0, b.stderr[-2000:]
    return exe


def _run(exe: Path, *args, env=None):
    return subprocess.run([str(exe), *args], capture_output=True, text=True, timeout=300, env=env)


def test_protocol_random_stalls(tmp_path):
    r = _run(_build(tmp_path))
    assert r.returncode == 0 and "requests ok" in r.stdout, r.stdout + r.stderr


def test_protocol_refuses_overpost(tmp_path):
    """Posting more requests than slots without reading any back is refused by the slot check."""
    r = _run(_build(tmp_path), "--overpost")
    assert r.returncode == 0 and "over-post refused" in r.stdout, r.stdout + r.stderr


def test_protocol_without_slot_check_is_caught(tmp_path):
    """With the slot check removed, a slot is reused before it is read back; the simulator
    must see the wrong output (so the check above is what keeps results intact)."""
    r = _run(_build(tmp_path), "--unsafe")
    assert r.returncode == 3, r.stdout + r.stderr
    assert "another request's output" in r.stderr


def test_protocol_under_thread_sanitizer(tmp_path):
    import os
    exe = _build(tmp_path, "thread")
    r = _run(exe, env=dict(os.environ, TSAN_OPTIONS="halt_on_error=1"))
    out = r.stdout + r.stderr
    assert r.returncode == 0 and "requests ok" in out, out[-4000:]
    assert "WARNING: ThreadSanitizer" not in out, out[-4000:]
