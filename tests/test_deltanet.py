"""Gated DeltaNet kernels (conv + L2 norm + gated delta rule) against the PyTorch
per-token recurrence, across chunked prefill and decode of several sequences."""
import math

import pytest
import torch

from vllm_xtu_moe_b200.models.config import get_preset, scaled_down
from vllm_xtu_moe_b200.models.deltanet import DeltaNetState, deltanet_ref
from vllm_xtu_moe_b200.ops.attention import AttnMetadata


def _meta(lens, starts, slots, device):
    qs = [0]
    for L in lens:
        qs.append(qs[-1] + L)
    d = device
    return AttnMetadata(num_seqs=len(lens), q_start=torch.tensor(qs, dtype=torch.int32, device=d),
                        kv_len=torch.tensor([s + L for s, L in zip(starts, lens)], dtype=torch.int32, device=d),
                        block_table=torch.zeros(len(lens), 1, dtype=torch.int32, device=d),
                        slot_mapping=torch.zeros(qs[-1], dtype=torch.int32, device=d),
                        positions=torch.zeros(qs[-1], dtype=torch.int32, device=d), max_q_len=max(lens),
                        max_kv_len=max(s + L for s, L in zip(starts, lens)), is_decode=False, q_start_host=qs,
                        seq_slots=torch.tensor(slots, dtype=torch.int32, device=d),
                        seq_fresh=torch.tensor([1 if s == 0 else 0 for s in starts], dtype=torch.int32, device=d))


@pytest.mark.gpu
@pytest.mark.parametrize("chunked", [False, True])
def test_deltanet_kernels_match_reference(chunked):
    """Token-serial kernel (2e-3) and the chunked tensor-core form (tf32 products, 1e-2) of
    the prefill steps; decode steps always run the token-serial kernel."""
    from vllm_xtu_moe_b200.ops.deltanet import deltanet_fwd
    torch.manual_seed(0)
    cfg = scaled_down(get_preset("qwen3-next-80b-a3b"), layers=4, hidden=256, experts=8).replace(
        linear_num_key_heads=2, linear_num_value_heads=4, linear_key_head_dim=128, linear_value_head_dim=128)
    nk, nv, dk, dv, kw = 2, 4, 128, 128, cfg.linear_conv_kernel
    r = nv // nk
    W = 2 * dk + 2 * r * dv
    ch = 2 * nk * dk + nv * dv
    conv_w = (torch.randn(ch, kw) * 0.3).cuda()
    st_gpu = DeltaNetState(cfg, 4, "cuda")
    st_ref = DeltaNetState(cfg, 4, "cuda")
    # step 1: two fresh sequences (prefill chunks); step 2: continue both + decode; step 3: decode only
    plan = [([37, 130], [0, 0], [2, 0]), ([5, 1], [37, 130], [2, 0]), ([1, 1], [42, 131], [2, 0])]
    for lens, starts, slots in plan:
        T = sum(lens)
        qkvz = (torch.randn(T, nk * W) * 0.5).to(torch.bfloat16).cuda()
        g = -torch.rand(T, nv).cuda() * 0.5
        beta = torch.rand(T, nv).cuda()
        meta = _meta(lens, starts, slots, "cuda")
        use_chunks = chunked and max(lens) >= 8
        og = deltanet_fwd(qkvz, conv_w, g, beta, meta, st_gpu, nk, nv, dk, dv, chunked=use_chunks)
        x = qkvz.view(T, nk, W)
        q = x[:, :, :dk].reshape(T, nk * dk)
        k = x[:, :, dk:2 * dk].reshape(T, nk * dk)
        v = x[:, :, 2 * dk:2 * dk + r * dv].reshape(T, nv * dv)
        mixed = torch.cat([q, k, v], -1)
        orf = deltanet_ref(mixed, conv_w, g, beta, meta, st_ref, nk, nv, dk, dv)
        torch.cuda.synchronize()
        err = (og - orf).abs().max().item() / orf.abs().max().item()
        tol = 1e-2 if use_chunks else 2e-3
        assert err < tol, (lens, err)
        for s in slots:
            es = (st_gpu.ssm[s] - st_ref.ssm[s]).abs().max().item() / st_ref.ssm[s].abs().max().item()
            assert es < tol
            assert torch.equal(st_gpu.conv[s], st_ref.conv[s])


@pytest.mark.gpu
@pytest.mark.parametrize("decay", [0.5, 0.01])
def test_chunked_deltanet_long_sequences(decay):
    """Chunked form over many chunks (700 + 64 + 1 tokens, partial last chunks), with strong and
    weak decay (long memory), continued from the state it left, against the recurrence."""
    from vllm_xtu_moe_b200.ops.deltanet import deltanet_fwd
    torch.manual_seed(5)
    cfg = scaled_down(get_preset("qwen3-next-80b-a3b"), layers=4, hidden=256, experts=8).replace(
        linear_num_key_heads=1, linear_num_value_heads=2, linear_key_head_dim=128, linear_value_head_dim=128)
    nk, nv, dk, dv, kw = 1, 2, 128, 128, cfg.linear_conv_kernel
    r = nv // nk
    W = 2 * dk + 2 * r * dv
    ch = 2 * nk * dk + nv * dv
    conv_w = (torch.randn(ch, kw) * 0.3).cuda()
    st_gpu = DeltaNetState(cfg, 3, "cuda")
    st_ref = DeltaNetState(cfg, 3, "cuda")
    for lens, starts, slots in [([700, 64, 1], [0, 0, 0], [0, 1, 2]), ([129, 65], [700, 64], [0, 1])]:
        T = sum(lens)
        qkvz = (torch.randn(T, nk * W) * 0.5).to(torch.bfloat16).cuda()
        g = -torch.rand(T, nv).cuda() * decay
        beta = torch.rand(T, nv).cuda()
        meta = _meta(lens, starts, slots, "cuda")
        og = deltanet_fwd(qkvz, conv_w, g, beta, meta, st_gpu, nk, nv, dk, dv, chunked=True)
        x = qkvz.view(T, nk, W)
        mixed = torch.cat([x[:, :, :dk].reshape(T, nk * dk), x[:, :, dk:2 * dk].reshape(T, nk * dk),
                           x[:, :, 2 * dk:2 * dk + r * dv].reshape(T, nv * dv)], -1)
        orf = deltanet_ref(mixed, conv_w, g, beta, meta, st_ref, nk, nv, dk, dv)
        torch.cuda.synchronize()
        err = (og - orf).abs().max().item() / orf.abs().max().item()
        assert err < 1e-2, (lens, decay, err)
        for s in slots:
            es = (st_gpu.ssm[s] - st_ref.ssm[s]).abs().max().item() / st_ref.ssm[s].abs().max().item()
            assert es < 1e-2, (s, es)


@pytest.mark.gpu
def test_kda_kernels_match_reference():
    """Kimi Delta Attention form of the kernels: blocked [Q | K | V] in-projection rows and a
    decay per key dim, against the per-token recurrence, over prefill chunks and decode."""
    from vllm_xtu_moe_b200.ops.deltanet import deltanet_fwd
    torch.manual_seed(1)
    cfg = scaled_down(get_preset("kimi-linear-48b-a3b"), layers=4, hidden=256, experts=8).replace(
        linear_num_key_heads=2, linear_num_value_heads=2, linear_key_head_dim=128, linear_value_head_dim=128)
    nk, nv, dk, dv, kw = 2, 2, 128, 128, cfg.linear_conv_kernel
    ch = 2 * nk * dk + nv * dv
    conv_w = (torch.randn(ch, kw) * 0.3).cuda()
    st_gpu = DeltaNetState(cfg, 4, "cuda")
    st_ref = DeltaNetState(cfg, 4, "cuda")
    plan = [([37, 130], [0, 0], [1, 3]), ([5, 1], [37, 130], [1, 3]), ([1, 1], [42, 131], [1, 3])]
    for lens, starts, slots in plan:
        T = sum(lens)
        qkv = (torch.randn(T, ch) * 0.5).to(torch.bfloat16).cuda()
        g = -torch.rand(T, nv, dk).cuda() * 0.5
        beta = torch.rand(T, nv).cuda()
        meta = _meta(lens, starts, slots, "cuda")
        og = deltanet_fwd(qkv, conv_w, g, beta, meta, st_gpu, nk, nv, dk, dv, blocked=True)
        orf = deltanet_ref(qkv, conv_w, g, beta, meta, st_ref, nk, nv, dk, dv)
        torch.cuda.synchronize()
        err = (og - orf).abs().max().item() / orf.abs().max().item()
        assert err < 2e-3, (lens, err)
        for s in slots:
            es = (st_gpu.ssm[s] - st_ref.ssm[s]).abs().max().item() / st_ref.ssm[s].abs().max().item()
            assert es < 2e-3
            assert torch.equal(st_gpu.conv[s], st_ref.conv[s])


def test_channel_decay_reduces_to_scalar_decay():
    """A per-key-dim decay that is the same on every key dim is the scalar gated delta rule."""
    from vllm_xtu_moe_b200.models.deltanet import _delta_rule_ref
    torch.manual_seed(3)
    T, H, dk, dv = 9, 3, 8, 5
    q, k = torch.randn(T, H, dk), torch.nn.functional.normalize(torch.randn(T, H, dk), dim=-1)
    v, beta = torch.randn(T, H, dv), torch.rand(T, H)
    g = -torch.rand(T, H)
    s1, s2 = torch.randn(H, dk, dv), None
    s2 = s1.clone()
    a = _delta_rule_ref(q, k, v, g, beta, s1)
    b = _delta_rule_ref(q, k, v, g[:, :, None].expand(T, H, dk).contiguous(), beta, s2)
    assert torch.allclose(a, b, atol=1e-5) and torch.allclose(s1, s2, atol=1e-5)


@pytest.mark.gpu
@pytest.mark.parametrize("chunked", [False, True])
def test_fused_gates_and_gated_norm(chunked):
    """Gates formed by the conv kernel from the in_proj_ba rows (beta = sigmoid(b),
    g = -exp(A_log) softplus(a + dt_bias)) and the silu(z)-gated RMSNorm of the output,
    against the layer's PyTorch math over the same recurrence kernels."""
    import torch.nn.functional as F
    from vllm_xtu_moe_b200.ops.deltanet import deltanet_fwd
    torch.manual_seed(7)
    cfg = scaled_down(get_preset("qwen3-next-80b-a3b"), layers=4, hidden=256, experts=8).replace(
        linear_num_key_heads=2, linear_num_value_heads=4, linear_key_head_dim=128, linear_value_head_dim=128)
    nk, nv, dk, dv, kw = 2, 4, 128, 128, cfg.linear_conv_kernel
    r = nv // nk
    W = 2 * dk + 2 * r * dv
    ch = 2 * nk * dk + nv * dv
    conv_w = (torch.randn(ch, kw) * 0.3).cuda()
    A_log = (torch.rand(nv) * 2 - 1).cuda()
    dt_bias = torch.randn(nv).cuda()
    norm_w = (1 + 0.1 * torch.randn(dv)).cuda()
    st_a = DeltaNetState(cfg, 2, "cuda")
    st_b = DeltaNetState(cfg, 2, "cuda")
    lens, starts, slots = [150, 70], [0, 0], [0, 1]
    T = sum(lens)
    qkvz = (torch.randn(T, nk * W) * 0.5).to(torch.bfloat16).cuda()
    ba = (torch.randn(T, 2 * nv) * 2).to(torch.bfloat16).cuda()
    meta = _meta(lens, starts, slots, "cuda")
    y = deltanet_fwd(qkvz, conv_w, None, None, meta, st_a, nk, nv, dk, dv, chunked=chunked, ba=ba,
                     A_log32=A_log, dt_bias32=dt_bias, norm_w32=norm_w, eps=1e-6)
    bav = ba.view(T, nk, 2 * r)
    b = bav[:, :, :r].reshape(T, nv).float()
    a = bav[:, :, r:].reshape(T, nv).float()
    beta = torch.sigmoid(b)
    g = -torch.exp(A_log) * F.softplus(a + dt_bias)
    o = deltanet_fwd(qkvz, conv_w, g, beta, meta, st_b, nk, nv, dk, dv, chunked=chunked)
    z = qkvz.view(T, nk, W)[:, :, 2 * dk + r * dv:].reshape(T, nv, dv).float()
    ref = (o * torch.rsqrt(o.pow(2).mean(-1, keepdim=True) + 1e-6) * norm_w * F.silu(z)).to(torch.bfloat16)
    torch.cuda.synchronize()
    err = (y.float().view(T, nv, dv) - ref.float()).abs().max().item() / ref.float().abs().max().item()
    assert err < 2e-2, err
    assert torch.allclose(st_a.ssm, st_b.ssm, rtol=1e-3, atol=1e-4)


@pytest.mark.gpu
def test_kda_sigmoid_gated_norm():
    """KDA output path: sigmoid(gate)-gated RMSNorm in the deltanet kernels against PyTorch."""
    from vllm_xtu_moe_b200.ops.deltanet import deltanet_fwd
    torch.manual_seed(8)
    cfg = scaled_down(get_preset("kimi-linear-48b-a3b"), layers=4, hidden=256, experts=8).replace(
        linear_num_key_heads=2, linear_num_value_heads=2, linear_key_head_dim=128, linear_value_head_dim=128)
    nk, nv, dk, dv, kw = 2, 2, 128, 128, cfg.linear_conv_kernel
    ch = 2 * nk * dk + nv * dv
    conv_w = (torch.randn(ch, kw) * 0.3).cuda()
    norm_w = (1 + 0.1 * torch.randn(dv)).cuda()
    st_a = DeltaNetState(cfg, 1, "cuda")
    st_b = DeltaNetState(cfg, 1, "cuda")
    T = 33
    qkv = (torch.randn(T, ch) * 0.5).to(torch.bfloat16).cuda()
    g = -torch.rand(T, nv, dk).cuda() * 0.5
    beta = torch.rand(T, nv).cuda()
    gate = torch.randn(T, nv * dv).to(torch.bfloat16).cuda()
    meta = _meta([T], [0], [0], "cuda")
    y = deltanet_fwd(qkv, conv_w, g, beta, meta, st_a, nk, nv, dk, dv, blocked=True, norm_w32=norm_w, eps=1e-6,
                     gate=gate)
    o = deltanet_fwd(qkv, conv_w, g, beta, meta, st_b, nk, nv, dk, dv, blocked=True)
    ref = (o * torch.rsqrt(o.pow(2).mean(-1, keepdim=True) + 1e-6) * norm_w
           * torch.sigmoid(gate.float().view(T, nv, dv))).to(torch.bfloat16)
    torch.cuda.synchronize()
    err = (y.float().view(T, nv, dv) - ref.float()).abs().max().item() / ref.float().abs().max().item()
    assert err < 2e-2, err


@pytest.mark.gpu
def test_spec_verification_states_and_commit():
    """A speculative verification step (4 rows per sequence, decode metadata): the kernels
    keep the recurrent and conv states after every row, equal to the recurrence's; the
    commit installs the ones of each sequence's accepted row (1 and 3 here)."""
    from vllm_xtu_moe_b200.ops.deltanet import deltanet_fwd
    torch.manual_seed(11)
    cfg = scaled_down(get_preset("qwen3-next-80b-a3b"), layers=4, hidden=256, experts=8).replace(
        linear_num_key_heads=1, linear_num_value_heads=2, linear_key_head_dim=128, linear_value_head_dim=128)
    nk, nv, dk, dv, kw = 1, 2, 128, 128, cfg.linear_conv_kernel
    r = nv // nk
    W = 2 * dk + 2 * r * dv
    ch = 2 * nk * dk + nv * dv
    conv_w = (torch.randn(ch, kw) * 0.3).cuda()
    st_g = DeltaNetState(cfg, 3, "cuda")
    st_r = DeltaNetState(cfg, 3, "cuda")
    st_g.enable_spec(3)
    st_r.enable_spec(3)
    slots = [2, 0]

    def step(lens, starts, spec):
        T = sum(lens)
        qkvz = (torch.randn(T, nk * W) * 0.5).to(torch.bfloat16).cuda()
        g = -torch.rand(T, nv).cuda() * 0.5
        beta = torch.rand(T, nv).cuda()
        meta = _meta(lens, starts, slots, "cuda")
        if spec:
            meta.is_decode = True
            meta.spec_rows = max(lens)
        deltanet_fwd(qkvz, conv_w, g, beta, meta, st_g, nk, nv, dk, dv, chunked=False)
        x = qkvz.view(T, nk, W)
        mixed = torch.cat([x[:, :, :dk].reshape(T, nk * dk), x[:, :, dk:2 * dk].reshape(T, nk * dk),
                           x[:, :, 2 * dk:2 * dk + r * dv].reshape(T, nv * dv)], -1)
        deltanet_ref(mixed, conv_w, g, beta, meta, st_r, nk, nv, dk, dv)

    step([9, 30], [0, 0], False)                 # prompts
    step([4, 4], [9, 30], True)                  # verification: last token + 3 drafts each
    torch.cuda.synchronize()
    for s in slots:
        for j in range(4):
            a, b = st_g.spec_ssm[s, j], st_r.spec_ssm[s, j]
            assert (a - b).abs().max().item() <= 2e-3 * b.abs().max().item(), (s, j)
            assert torch.equal(st_g.spec_conv[s, j], st_r.spec_conv[s, j]), (s, j)
    acc = torch.tensor([1, 3], dtype=torch.int32, device="cuda")
    sl = torch.tensor(slots, dtype=torch.int32, device="cuda")
    st_g.commit_spec(acc, sl)
    torch.cuda.synchronize()
    for s, a in zip(slots, (1, 3)):
        assert torch.equal(st_g.ssm[s], st_g.spec_ssm[s, a])
        assert torch.equal(st_g.conv[s], st_g.spec_conv[s, a])
        assert (st_g.ssm[s] - st_r.spec_ssm[s, a]).abs().max().item() <= 2e-3 * st_r.spec_ssm[s, a].abs().max().item()
