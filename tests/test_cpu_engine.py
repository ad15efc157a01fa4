"""C++ CPU expert engine vs the PyTorch fp32 MoE reference (runs on the host)."""
import multiprocessing as mp
import os

import pytest
import torch

from vllm_xtu_moe_b200.ops import moe as M
from vllm_xtu_moe_b200.ops.quant import quant_fp8_block, quant_mxfp4, quant_nvfp4
from vllm_xtu_moe_b200.ops.router import router_topk_ref
from vllm_xtu_moe_b200.tiering.cpu_engine import CpuExpertEngine, ShmEpGroup, lib


def _raw(fmt, E, H, I, seed=0):
    g = torch.Generator().manual_seed(seed)
    w13 = torch.randn(E, 2 * I, H, generator=g) / H ** 0.5
    w2 = torch.randn(E, H, I, generator=g) / I ** 0.5
    if fmt == "bf16":
        return dict(w13=w13.to(torch.bfloat16), w2=w2.to(torch.bfloat16))
    if fmt == "fp8":
        q13, s13 = quant_fp8_block(w13)
        q2, s2 = quant_fp8_block(w2)
        return dict(w13=q13, w2=q2, s13=s13, s2=s2)
    if fmt == "mxfp4":
        p13, s13 = quant_mxfp4(w13)
        p2, s2 = quant_mxfp4(w2)
        return dict(w13=p13, w2=p2, s13=s13, s2=s2)
    if fmt == "int4":          # asymmetric 4-bit rows, 128-wide groups: w = (q - zero) * scale
        def q4(w):
            wg = w.view(*w.shape[:-1], -1, 128)
            lo, hi = wg.amin(-1), wg.amax(-1)
            sc = ((hi - lo) / 15).clamp(min=1e-6)
            z = torch.round(-lo / sc).clamp(0, 15)
            q = (torch.round(wg / sc[..., None]) + z[..., None]).clamp(0, 15).to(torch.uint8).flatten(-2)
            return (q[..., 0::2] | (q[..., 1::2] << 4)).contiguous(), torch.stack([sc, z], -1).contiguous()
        p13, s13 = q4(w13)
        p2, s2 = q4(w2)
        return dict(w13=p13, w2=p2, s13=s13, s2=s2)
    p13, s13, g13 = zip(*[quant_nvfp4(w13[e]) for e in range(E)])
    p2, s2, g2 = zip(*[quant_nvfp4(w2[e]) for e in range(E)])
    return dict(w13=torch.stack(p13), w2=torch.stack(p2), s13=torch.stack(s13).view(torch.uint8),
                s2=torch.stack(s2).view(torch.uint8), gs13=torch.stack(g13), gs2=torch.stack(g2))


def _ref(fmt, raw, x, ids, w, lo, hi, limit=0.0):
    if fmt == "int4":
        from vllm_xtu_moe_b200.ops.quant import dequant_int4_rows
        ex = M.ExpertWeights("bf16", dequant_int4_rows(raw["w13"], raw["s13"]).to(torch.bfloat16),
                             dequant_int4_rows(raw["w2"], raw["s2"]).to(torch.bfloat16), None, None, False)
        return M.moe_ref(x, ids, w, ex, lo, hi, act_limit=limit)
    ex = M.ExpertWeights(fmt, raw["w13"], raw["w2"], raw.get("s13"), raw.get("s2"), False, raw.get("gs13"),
                         raw.get("gs2"))
    if fmt == "nvfp4":
        ex.s13 = raw["s13"].view(torch.float8_e4m3fn)
        ex.s2 = raw["s2"].view(torch.float8_e4m3fn)
    return M.moe_ref(x, ids, w, ex, lo, hi, act_limit=limit)


def test_e4m3_decoder_all_codes():
    """All 256 e4m3 codes decode exactly like torch.float8_e4m3fn (NaN codes -> 0)."""
    L = lib()
    codes = torch.arange(256, dtype=torch.uint8)
    ref = codes.view(torch.float8_e4m3fn).float()
    for c in range(256):
        v = L.xtu_cpu_e4m3_to_f32(c)
        r = ref[c].item()
        if r != r:
            assert v == 0.0
        else:
            assert v == r, (c, v, r)


@pytest.mark.parametrize("fmt", ["bf16", "fp8", "mxfp4", "nvfp4", "int4"])
@pytest.mark.parametrize("T", [1, 5, 37])
def test_engine_matches_reference(fmt, T):
    E, H, I, K = 8, 256, 384 if fmt in ("bf16", "mxfp4", "nvfp4", "int4") else 256, 2
    raw = _raw(fmt, E, H, I)
    eng = CpuExpertEngine(fmt, raw["w13"], raw["w2"], raw.get("s13"), raw.get("s2"), raw.get("gs13"),
                          raw.get("gs2"), threads=4, act_limit=7.0, int8_mode=0)
    g = torch.Generator().manual_seed(1)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    ids, w = router_topk_ref(torch.randn(T, E, generator=g), K, "softmax")
    out = eng.forward(x, ids, w)
    ref = _ref(fmt, raw, x, ids, w, 0, E, 7.0)
    err = (out - ref).abs().max().item() / (ref.abs().max().item() + 1e-6)
    assert err < 2e-2, err
    eng.close()


def test_engine_skips_other_tiers_and_zero_weights():
    E, H, I = 8, 256, 256
    raw = _raw("bf16", E, H, I)
    eng = CpuExpertEngine("bf16", raw["w13"], raw["w2"], threads=2)
    g = torch.Generator().manual_seed(2)
    x = torch.randn(6, H, generator=g).to(torch.bfloat16)
    ids, w = router_topk_ref(torch.randn(6, E, generator=g), 2, "softmax")
    w[0, 0] = 0.0
    # this engine holds global experts [8, 16); ids are local here -> shift them
    out = eng.forward(x, ids + 8, w, lo=8, hi=16)
    ref = _ref("bf16", raw, x, ids, w, 0, E)
    assert torch.allclose(out, ref, rtol=2e-2, atol=2e-3)
    out2 = eng.forward(x, ids, w, lo=8, hi=16)    # every pair belongs to another tier
    assert out2.abs().max().item() == 0.0


def test_engine_owns_a_copy():
    """Clobbering the caller's tensors after construction leaves results unchanged."""
    E, H, I = 4, 256, 256
    raw = _raw("fp8", E, H, I)
    eng = CpuExpertEngine("fp8", raw["w13"], raw["w2"], raw["s13"], raw["s2"], threads=2)
    x = torch.randn(3, H).to(torch.bfloat16)
    ids = torch.tensor([[0, 1], [2, 3], [1, 2]], dtype=torch.int32)
    w = torch.full((3, 2), 0.5)
    a = eng.forward(x, ids, w)
    raw["w13"].view(torch.uint8).fill_(0)
    raw["s13"].fill_(0)
    b = eng.forward(x, ids, w)
    assert torch.equal(a, b)


def test_engine_deterministic():
    E, H, I = 8, 256, 256
    raw = _raw("mxfp4", E, H, I)
    eng = CpuExpertEngine("mxfp4", raw["w13"], raw["w2"], raw["s13"], raw["s2"], threads=8)
    x = torch.randn(20, H).to(torch.bfloat16)
    ids, w = router_topk_ref(torch.randn(20, E), 3, "softmax")
    outs = [eng.forward(x, ids, w) for _ in range(4)]
    assert all(torch.equal(outs[0], o) for o in outs[1:])


def test_int8_activation_path_close_to_fp32():
    """MXFP4 x INT8 activations (per-32 power-of-two scales) vs the fp32 path."""
    E, H, I = 8, 256, 256
    raw = _raw("mxfp4", E, H, I)
    g = torch.Generator().manual_seed(3)
    x = torch.randn(200, H, generator=g).to(torch.bfloat16)
    ids, w = router_topk_ref(torch.randn(200, E, generator=g), 2, "softmax")
    e32 = CpuExpertEngine("mxfp4", raw["w13"], raw["w2"], raw["s13"], raw["s2"], int8_mode=0)
    e8 = CpuExpertEngine("mxfp4", raw["w13"], raw["w2"], raw["s13"], raw["s2"], int8_mode=2, int8_min_tokens=160)
    a, b = e32.forward(x, ids, w), e8.forward(x, ids, w)
    rel = ((a - b).pow(2).mean().sqrt() / a.pow(2).mean().sqrt()).item()
    assert 0 < rel < 2e-2, rel     # int8 path is active (not bit-equal) and accurate


def _shm_rank(rank, world, name, q):
    try:
        g = ShmEpGroup(name, rank, world, 1024, timeout_ms=5000)
        t = torch.full((1000,), float(rank + 1))
        g.allreduce_(t)
        q.put((rank, t[0].item()))
        g.close()
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, repr(e)))


def test_shm_ep_allreduce_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    name = f"/xtu_test_{os.getpid()}"
    ps = [ctx.Process(target=_shm_rank, args=(r, 2, name, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=60) for _ in range(2))
    for p in ps:
        p.join(timeout=30)
    assert res == {0: 3.0, 1: 3.0}


def test_shm_ep_missing_peer_times_out():
    """A rank whose peer never joins gets a TimeoutError, not a hang."""
    g = ShmEpGroup(f"/xtu_test_lonely_{os.getpid()}", 0, 2, 64, timeout_ms=300)
    with pytest.raises(TimeoutError):
        g.allreduce_(torch.ones(64))
    g.close()


# ----------------------------------------------------------------------------- sanitizers
@pytest.mark.parametrize("kind", ["thread", "address,undefined"])
def test_engine_under_host_sanitizers(kind, tmp_path):
    """The CPU expert engine and its NUMA work pool built with ThreadSanitizer /
    AddressSanitizer+UBSan into a host-only driver (tests/cpp/engine_sanitize.cpp) that
    checks its forward passes against a scalar MoE; any sanitizer report fails."""
    import shutil
    import subprocess
    from pathlib import Path
    cxx = shutil.which("g++")
    if cxx is None:
        pytest.skip("no g++")
    root = Path(__file__).resolve().parents[1]
    cpu = root / "csrc" / "cpu"
    exe = tmp_path / "engine_sanitize"
    isa = ["-mavx512f", "-mavx512bw", "-mavx512vl", "-mavx512bf16", "-mavx512vnni", "-mavx512vbmi", "-mfma"]
    cmd = [cxx, "-std=c++17", "-O1", "-g", "-fno-omit-frame-pointer", f"-fsanitize={kind}", "-pthread", *isa,
           f"-I{cpu}", str(root / "tests" / "cpp" / "engine_sanitize.cpp"), str(cpu / "moe_engine.cpp"),
           str(cpu / "moe_kernels_avx512.cpp"), str(cpu / "numa_pool.cpp"), "-o", str(exe)]
    b = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
    if b.returncode != 0 and "sanitizer" in b.stderr.lower() and "cannot find" in b.stderr.lower():
        pytest.skip("sanitizer runtime not installed")
    assert b.returncode == 0, b.stderr[-2000:]
    env = dict(os.environ, TSAN_OPTIONS="halt_on_error=1", ASAN_OPTIONS="detect_leaks=1",
               UBSAN_OPTIONS="halt_on_error=1:print_stacktrace=1")
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=600, env=env)
    out = r.stdout + r.stderr
    assert r.returncode == 0 and "engine_sanitize: ok" in out, out[-4000:]
    assert "WARNING: ThreadSanitizer" not in out and "ERROR: AddressSanitizer" not in out, out[-4000:]
    assert "runtime error" not in out, out[-4000:]
