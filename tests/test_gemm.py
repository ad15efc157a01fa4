"""tcgen05 GEMM kernels vs a PyTorch fp32 reference of the same op."""
import pytest
import torch

from vllm_xtu_moe_b200.ops import gemm as G
from vllm_xtu_moe_b200.ops.quant import dequant_fp8_block, quant_fp8_block


def _close(out, ref, tol=2e-2):
    if ref.numel() == 0:
        return
    out = out.float()
    ref = ref.float()
    err = (out - ref).abs().max().item()
    scale = ref.abs().max().item() + 1e-6
    assert err / scale < tol, f"max err {err} vs scale {scale}"


def test_interleave_gate_up_roundtrip():
    w = torch.randn(3, 512, 64)
    wi = G.interleave_gate_up(w)
    # block 0 of the result is gate rows 0..127, block 1 is up rows 0..127
    assert torch.equal(wi[:, :128], w[:, :128])
    assert torch.equal(wi[:, 128:256], w[:, 256:384])
    assert torch.equal(wi[:, 256:384], w[:, 128:256])


def test_grouped_torch_path_swiglu_matches_unfused():
    torch.manual_seed(0)
    E, K, I = 3, 64, 256
    w13 = torch.randn(E, 2 * I, K, dtype=torch.bfloat16) * 0.1
    a = torch.randn(10, K, dtype=torch.bfloat16)
    seg = torch.tensor([0, 4, 4, 10], dtype=torch.int32)
    out = G.grouped_gemm(a, G.interleave_gate_up(w13), seg, epilogue=G.EPI_SWIGLU, act_limit=7.0)
    for e in range(E):
        s0, s1 = seg[e].item(), seg[e + 1].item()
        y = a[s0:s1].float() @ w13[e].float().t()
        ref = G.silu_and_mul_clamped(y[:, :I], y[:, I:], 7.0)
        _close(out[s0:s1], ref)


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (300, 384, 1032), (1, 4096, 4096), (1000, 128, 512),
                                   (4096, 4096, 4096)])
def test_gemm_bf16(M, N, K):
    torch.manual_seed(0)
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) / K ** 0.5
    out = G.gemm_bf16(a, b)
    out32 = G.gemm_bf16(a, b, out_dtype=torch.float32)
    torch.cuda.synchronize()
    G.N.check_status()
    ref = a.float() @ b.float().t()
    _close(out, ref)
    _close(out32, ref, 1e-3)


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", [(200, 512, 1024), (7, 2816, 4096)])
def test_gemm_fp8_weights(M, N, K):
    torch.manual_seed(1)
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda") / K ** 0.5
    q, s = quant_fp8_block(w)
    out = G.gemm_fp8w(a, q, s, out_dtype=torch.float32)
    torch.cuda.synchronize()
    G.N.check_status()
    wd = dequant_fp8_block(q, s).to(torch.bfloat16).float()
    ref = a.float() @ wd.t()
    _close(out, ref, 1e-3)


def _segments(counts):
    seg = [0]
    for c in counts:
        seg.append(seg[-1] + c)
    return torch.tensor(seg, dtype=torch.int32)


@pytest.mark.gpu
@pytest.mark.parametrize("fp8", [False, True])
@pytest.mark.parametrize("counts", [[5, 0, 130, 257, 1], [0, 0, 3, 0]])
def test_grouped_gemm(fp8, counts):
    torch.manual_seed(2)
    E = len(counts)
    K, Nn = 512, 768
    seg = _segments(counts).cuda()
    M = int(seg[-1])
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(E, Nn, K, device="cuda") / K ** 0.5
    if fp8:
        q, s = quant_fp8_block(w)
        out = G.grouped_gemm(a, q, seg, w_scale=s, epilogue=G.EPI_F32)
        wd = dequant_fp8_block(q, s).to(torch.bfloat16)
    else:
        wd = w.to(torch.bfloat16)
        out = G.grouped_gemm(a, wd, seg, epilogue=G.EPI_F32)
    torch.cuda.synchronize()
    G.N.check_status()
    ref = G._grouped_gemm_torch(a.cpu(), wd.cpu(), seg.cpu(), None, G.EPI_F32,
                                torch.zeros(M, Nn), None, None, 0, 1, 0)
    _close(out.cpu(), ref, 1e-3)


@pytest.mark.gpu
@pytest.mark.parametrize("fp8", [False, True])
def test_grouped_swiglu_and_scatter(fp8):
    torch.manual_seed(3)
    counts = [70, 0, 129, 3]
    E, K, I = 4, 256, 256
    seg = _segments(counts).cuda()
    M = int(seg[-1])
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w13 = torch.randn(E, 2 * I, K, device="cuda") / K ** 0.5
    w2 = torch.randn(E, K, I, device="cuda") / I ** 0.5
    scale = torch.rand(M, device="cuda")
    dest = torch.randperm(M, device="cuda").int()
    if fp8:
        q13, s13 = quant_fp8_block(w13)
        q2, s2 = quant_fp8_block(w2)
        h = G.grouped_gemm(a, G.interleave_gate_up(q13.view(torch.uint8)).view(torch.float8_e4m3fn), seg,
                           w_scale=G.interleave_gate_up_scale(s13), epilogue=G.EPI_SWIGLU, act_limit=10.0)
        out = G.grouped_gemm(h, q2, seg, w_scale=s2, row_scale=scale, row_dest=dest, epilogue=G.EPI_F32)
        w13d = dequant_fp8_block(q13, s13).to(torch.bfloat16)
        w2d = dequant_fp8_block(q2, s2).to(torch.bfloat16)
    else:
        w13d, w2d = w13.to(torch.bfloat16), w2.to(torch.bfloat16)
        h = G.grouped_gemm(a, G.interleave_gate_up(w13d), seg, epilogue=G.EPI_SWIGLU, act_limit=10.0)
        out = G.grouped_gemm(h, w2d, seg, row_scale=scale, row_dest=dest, epilogue=G.EPI_F32)
    torch.cuda.synchronize()
    G.N.check_status()
    segc = seg.cpu().tolist()
    ref = torch.zeros(M, K)
    for e in range(E):
        s0, s1 = segc[e], segc[e + 1]
        y = a[s0:s1].float().cpu() @ w13d[e].float().cpu().t()
        hh = G.silu_and_mul_clamped(y[:, :I], y[:, I:], 10.0).to(torch.bfloat16).float()
        _close(h[s0:s1].cpu(), hh) if s1 > s0 else None
        o = h[s0:s1].float().cpu() @ w2d[e].float().cpu().t() * scale[s0:s1].cpu()[:, None]
        ref[dest[s0:s1].long().cpu()] = o
    _close(out.cpu(), ref, 1e-3)


@pytest.mark.gpu
def test_gemm_fp8_many_tiles_per_cta():
    """Persistent CTAs looping over many tiles (the prefill shapes)."""
    torch.manual_seed(5)
    M, N, K = 4096, 4096, 2048
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda") / K ** 0.5
    q, s = quant_fp8_block(w)
    out = G.gemm_fp8w(a, q, s)
    torch.cuda.synchronize()
    G.N.check_status()
    ref = a.float() @ dequant_fp8_block(q, s).to(torch.bfloat16).float().t()
    _close(out, ref)


@pytest.mark.gpu
@pytest.mark.parametrize("fp8", [False, True])
def test_grouped_gemm_prefill_scale(fp8):
    """~16K routed rows over 128 experts with the fused SwiGLU epilogue (GLM-Air shapes, smaller K)."""
    torch.manual_seed(6)
    E, K, I = 128, 1024, 1408 // 11 * 2  # I = 256 keeps the reference cheap
    g = torch.Generator().manual_seed(0)
    counts = torch.multinomial(torch.ones(E), 16000, replacement=True, generator=g).bincount(minlength=E).tolist()
    seg = _segments(counts).cuda()
    M = int(seg[-1])
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w13 = torch.randn(E, 2 * I, K, device="cuda") / K ** 0.5
    if fp8:
        q, s = quant_fp8_block(w13)
        h = G.grouped_gemm(a, G.interleave_gate_up(q.view(torch.uint8)).view(torch.float8_e4m3fn), seg,
                           w_scale=G.interleave_gate_up_scale(s), epilogue=G.EPI_SWIGLU)
        wd = dequant_fp8_block(q, s).to(torch.bfloat16).float()
    else:
        wb = w13.to(torch.bfloat16)
        h = G.grouped_gemm(a, G.interleave_gate_up(wb), seg, epilogue=G.EPI_SWIGLU)
        wd = wb.float()
    torch.cuda.synchronize()
    G.N.check_status()
    segc = seg.tolist()
    for e in range(0, E, 17):
        s0, s1 = segc[e], segc[e + 1]
        if s1 == s0:
            continue
        y = a[s0:s1].float() @ wd[e].t()
        ref = G.silu_and_mul_clamped(y[:, :I], y[:, I:])
        _close(h[s0:s1], ref)


@pytest.mark.gpu
@pytest.mark.parametrize("fp8", [False, True])
@pytest.mark.parametrize("M", [1, 3, 4, 8, 13, 16, 17, 20, 32])
@pytest.mark.parametrize("N_,K", [(14336, 4096), (4096, 10944), (4096, 12288), (300, 512), (40000, 1024)])
def test_gemv_decode(fp8, M, N_, K):
    """Shapes with few 32-row slices, which split K across CTAs, and a many-wave shape; M
    above 16 with fp8 weights runs the tcgen05 form (weights widened to f16 on chip, 128-row
    tiles, tokens as the MMA's N).  Run twice: the split counters must be left zeroed for
    the next call."""
    torch.manual_seed(9)
    w = torch.randn(N_, K, device="cuda") / K ** 0.5
    bias = torch.randn(N_, device="cuda", dtype=torch.bfloat16)
    if fp8:
        q, s = quant_fp8_block(w)
        wd = dequant_fp8_block(q, s)
    else:
        wb = w.to(torch.bfloat16)
        wd = wb.float()
    for it in range(2):
        x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
        y = G.gemv(x, q, s, bias, torch.float32) if fp8 else G.gemv(x, wb, None, bias, torch.float32)
        torch.cuda.synchronize()
        ref = x.float() @ wd.t() + bias.float()
        _close(y, ref, 2e-3)


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["mxfp4", "nvfp4"])
@pytest.mark.parametrize("T,E,H,I,K", [(37, 8, 512, 256, 2), (300, 16, 1024, 512, 4), (5, 4, 256, 128, 2),
                                       # decode sizes: the packed-4-bit grouped GEMV (xtu_moe_gemv4)
                                       (1, 8, 512, 256, 2), (4, 32, 2048, 512, 8), (16, 16, 1024, 512, 4),
                                       (11, 8, 512, 768, 2)])
def test_fused_moe_fp4_matches_reference(fmt, T, E, H, I, K):
    """MXFP4 / NVFP4 experts through the grouped GEMM (on-chip widening) or, at decode sizes, the
    packed-4-bit grouped GEMV, vs the fp32 dequant reference."""
    from vllm_xtu_moe_b200.ops import moe as M
    from vllm_xtu_moe_b200.ops.quant import quant_mxfp4, quant_nvfp4
    g = torch.Generator().manual_seed(T + E)
    w13 = torch.randn(E, 2 * I, H, generator=g) / H ** 0.5
    w2 = torch.randn(E, H, I, generator=g) / I ** 0.5
    if fmt == "mxfp4":
        p13, s13 = quant_mxfp4(w13)
        p2, s2 = quant_mxfp4(w2)
        gs13 = gs2 = None
    else:
        r13 = [quant_nvfp4(w13[e]) for e in range(E)]
        r2 = [quant_nvfp4(w2[e]) for e in range(E)]
        p13, s13, gs13 = (torch.stack([r[i] for r in r13]) for i in range(3))
        p2, s2, gs2 = (torch.stack([r[i] for r in r2]) for i in range(3))
    cpu = M.prepare_experts(fmt, p13, p2, s13, s2, gs13, gs2)
    d = "cuda"
    gpu = M.prepare_experts(fmt, p13.to(d), p2.to(d), s13.to(d), s2.to(d), None if gs13 is None else gs13.to(d),
                            None if gs2 is None else gs2.to(d))
    x = (torch.randn(T, H, generator=g) * 0.5).to(torch.bfloat16)
    ids = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)]).int()
    w = torch.rand(T, K, generator=g)
    w = (w / w.sum(1, keepdim=True)).float()
    ref = M.moe_ref(x, ids, w, cpu).float()
    out = M.fused_moe(x.to(d), ids.to(d), w.to(d), gpu).float().cpu()
    torch.cuda.synchronize()
    err = (out - ref).abs().max().item()
    assert err <= 2e-2 * ref.abs().max().item() + 1e-3, err


def _all_codes_weight(N=256, K=128):
    """e4m3 weight [N, K] holding every finite code: W[n, k] = code (n + k) mod 256, the two
    NaN codes (0x7f, 0xff) replaced by 0."""
    n = torch.arange(N)[:, None]
    k = torch.arange(K)[None, :]
    codes = ((n + k) % 256).to(torch.uint8)
    codes[(codes == 0x7F) | (codes == 0xFF)] = 0
    return codes.view(torch.float8_e4m3fn)


@pytest.mark.gpu
def test_fp8_decode_gemv_widens_every_code_exactly():
    """The decode GEMV's e4m3 widening against torch.float8_e4m3fn for all finite codes:
    one-hot activations pick single weight columns, so every output is one weight value
    (exactly representable on the way: f16 x 2^-8 products, fp32 sums, bf16 output)."""
    w = _all_codes_weight().cuda()
    s = torch.ones(2, 1, device="cuda")
    for k0 in (0, 16, 112):
        x = torch.zeros(16, 128, device="cuda", dtype=torch.bfloat16)
        x[torch.arange(16), k0 + torch.arange(16)] = 1.0
        y = G.gemv(x, w, s)
        torch.cuda.synchronize()
        ref = w.float()[:, k0:k0 + 16].t()
        assert torch.equal(y.float().cpu(), ref.cpu()), k0


@pytest.mark.gpu
def test_fp8_grouped_gemm_widens_every_code_exactly():
    """The same for the prefill grouped GEMM's on-chip e4m3 -> bf16 widening (128 one-hot
    rows cover every column of the 128-column block)."""
    w = _all_codes_weight().cuda()[None]                    # [1, 256, 128]
    s = torch.ones(1, 2, 1, device="cuda")
    a = torch.eye(128, device="cuda", dtype=torch.bfloat16)
    seg = torch.tensor([0, 128], dtype=torch.int32, device="cuda")
    y = G.grouped_gemm(a, w, seg, w_scale=s)
    torch.cuda.synchronize()
    assert torch.equal(y.float().cpu(), w[0].float().t().cpu())
