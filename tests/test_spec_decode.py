"""MTP speculative decoding: greedy verification and end-to-end equivalence with
plain greedy decoding (the drafts may only change speed, never the tokens)."""
import pytest
import torch

from vllm_xtu_moe_b200.engine import LLM, SamplingParams
from vllm_xtu_moe_b200.engine.runner import RunnerConfig
from vllm_xtu_moe_b200.engine.spec_decode import SpecDecoder, verify_greedy
from vllm_xtu_moe_b200.models.config import get_preset, scaled_down
from vllm_xtu_moe_b200.models.model import build_model


def _cfg():
    return scaled_down(get_preset("glm-4.5-air"), layers=2, hidden=256, experts=16).replace(
        num_heads=4, num_kv_heads=2, head_dim=64, rotary_dim=32, moe_intermediate=256, shared_intermediate=256,
        dense_intermediate=512, num_mtp_layers=1)


def _run(model, k, prompts, n, device="cpu", oracle=None):
    rc = RunnerConfig(block_size=64, max_seqs=4, max_model_len=512, max_batched_tokens=128, use_cuda_graph=False,
                      num_spec=k)
    llm = LLM(model, device=device, runner_config=rc)
    if oracle is not None:
        def chain(reqs, first, hid, _self=llm.spec):
            out = []
            for r in reqs:
                ref = oracle[tuple(r.prompt)]
                t = r.total_len - len(r.prompt)
                out.append(ref[t:t + k] + [0] * max(0, k - len(ref[t:t + k])))
            return out
        llm.spec._chain = chain
    outs = llm.generate(prompts, SamplingParams(max_tokens=n))
    steps = llm.stats["steps"]
    llm.shutdown()
    return outs, steps


def test_verify_greedy_rules():
    # seq 0: [last, d1, d2, d3] with targets accepting d1, d2 only; seq 1: no drafts
    ids = torch.tensor([5, 7, 8, 9, 4], dtype=torch.int32)
    tgt = torch.tensor([7, 8, 1, 3, 6], dtype=torch.int32)
    q = torch.tensor([0, 4, 5], dtype=torch.int32)
    acc, row = verify_greedy(tgt, ids, q, 2, 3)
    assert acc.tolist() == [2, 0] and row.tolist() == [2, 4]


@pytest.mark.parametrize("k", [1, 3])
def test_spec_decode_matches_greedy_cpu(k):
    m = build_model(_cfg(), device="cpu", seed=1)
    m.act_dtype = torch.float32
    prompts = [list(range(3, 40)), list(range(50, 61))]
    base, steps0 = _run(m, 0, prompts, 12)
    spec, _ = _run(m, k, prompts, 12)
    assert [o.token_ids for o in spec] == [o.token_ids for o in base]
    assert all(o.proposed > 0 for o in spec)


def test_oracle_drafts_are_all_accepted():
    m = build_model(_cfg(), device="cpu", seed=1)
    m.act_dtype = torch.float32
    prompts = [list(range(3, 40)), list(range(50, 61))]
    base, steps0 = _run(m, 0, prompts, 13)
    oracle = {tuple(p): o.token_ids for p, o in zip(prompts, base)}
    spec, steps = _run(m, 3, prompts, 13, oracle=oracle)
    assert [o.token_ids for o in spec] == [o.token_ids for o in base]
    assert all(o.accepted >= 9 for o in spec)
    assert steps < steps0


def _qwen_cfg():
    return scaled_down(get_preset("qwen3-next-80b-a3b"), layers=4, hidden=256, experts=16).replace(
        num_heads=4, num_kv_heads=2, head_dim=64, moe_intermediate=256, shared_intermediate=256,
        linear_num_key_heads=2, linear_num_value_heads=4, linear_key_head_dim=32, linear_value_head_dim=32,
        rotary_dim=32, num_mtp_layers=1)


@pytest.mark.parametrize("oracle", [False, True])
def test_spec_decode_linear_attention_rolls_back_state_cpu(oracle):
    """Qwen3-Next-style hybrid (DeltaNet + gated GQA) with its MTP layer: the recurrent
    state after a verification step is the one after the last accepted token, so tokens
    equal plain greedy decoding, with MTP drafts (mostly rejected) and with oracle drafts
    (all accepted but a wrong tail appended every step, so every step rolls back)."""
    m = build_model(_qwen_cfg(), device="cpu", seed=0)
    m.act_dtype = torch.float32
    prompts = [list(range(3, 30)), list(range(50, 58))]
    base, steps0 = _run(m, 0, prompts, 12)
    if not oracle:
        spec, _ = _run(m, 3, prompts, 12)
    else:
        ref = {tuple(p): o.token_ids for p, o in zip(prompts, base)}
        half = {tuple(p): (o.token_ids[:2] + [1, 2, 3] * 8) for p, o in zip(prompts, base)}
        spec, steps = _run(m, 3, prompts, 12, oracle=ref)
        assert steps < steps0
        spec2, _ = _run(m, 3, prompts, 12, oracle=half)     # right, then wrong drafts
        assert [o.token_ids for o in spec2] == [o.token_ids for o in base]
    assert [o.token_ids for o in spec] == [o.token_ids for o in base]


@pytest.mark.gpu
def test_verify_kernel_matches_host():
    g = torch.Generator().manual_seed(0)
    lens = [1, 4, 4, 2, 3]
    q = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32)
    n = int(q[-1])
    tgt = torch.randint(0, 3, (n,), generator=g, dtype=torch.int32)
    ids = torch.randint(0, 3, (n,), generator=g, dtype=torch.int32)
    a0, r0 = verify_greedy(tgt, ids, q, len(lens), 3)
    a1, r1 = verify_greedy(tgt.cuda(), ids.cuda(), q.cuda(), len(lens), 3)
    assert a0.tolist() == a1.cpu().tolist() and r0.tolist() == r1.cpu().tolist()


@pytest.mark.gpu
def test_oracle_drafts_gpu():
    m = build_model(_cfg(), device="cuda", seed=1)
    prompts = [list(range(3, 40)), list(range(50, 61))]
    base, steps0 = _run(m, 0, prompts, 13, device="cuda")
    oracle = {tuple(p): o.token_ids for p, o in zip(prompts, base)}
    spec, steps = _run(m, 3, prompts, 13, device="cuda", oracle=oracle)
    same = sum(a == b for o, p in zip(spec, base) for a, b in zip(o.token_ids, p.token_ids))
    assert same >= 0.9 * sum(len(o.token_ids) for o in base)
    assert steps < steps0


def test_spec_decode_with_bounded_window_pool_cpu():
    """MiMo-style model (sliding-window layers on their bounded pool, one MTP layer): MTP
    speculative decoding gives the plain greedy tokens."""
    cfg = scaled_down(get_preset("mimo-v2-flash"), layers=4, hidden=256, experts=8).replace(
        num_heads=4, num_kv_heads=2, swa_num_kv_heads=4, head_dim=64, v_head_dim=32, rotary_dim=32,
        sliding_window=16, moe_intermediate=128, dense_intermediate=256, num_mtp_layers=1,
        expert_fmt="bf16", dense_fmt="bf16")
    m = build_model(cfg, device="cpu", seed=2)
    m.act_dtype = torch.float32
    prompts = [list(range(3, 60)), list(range(70, 85))]

    def run(k):
        rc = RunnerConfig(block_size=16, max_seqs=2, max_model_len=256, max_batched_tokens=64,
                          use_cuda_graph=False, num_spec=k)
        llm = LLM(m, device="cpu", runner_config=rc)
        assert rc.swa_blocks > 0
        outs = [o.token_ids for o in llm.generate(prompts, SamplingParams(max_tokens=12))]
        llm.shutdown()
        return outs

    assert run(2) == run(0)


@pytest.mark.gpu
@pytest.mark.parametrize("k", [1, 4])
def test_graph_replayed_spec_step_matches_eager_gpu(k):
    """The CUDA-graph speculative step (verify + MTP + device-side draft chain) gives the
    tokens of the eager step and of plain greedy decoding (up to split-KV rounding)."""
    m = build_model(_cfg(), device="cuda", seed=1)
    prompts = [list(range(3, 40)), list(range(50, 61)), list(range(100, 170))]

    def run(k_, graph):
        rc = RunnerConfig(block_size=64, max_seqs=4, max_model_len=512, max_batched_tokens=128,
                          use_cuda_graph=graph, num_spec=k_)
        llm = LLM(m, device="cuda", runner_config=rc)
        outs = llm.generate(prompts, SamplingParams(max_tokens=24))
        gsteps = llm.spec.graph_steps if llm.spec is not None else 0
        llm.shutdown()
        return outs, gsteps

    eager, g0 = run(k, False)
    graph, g1 = run(k, True)
    plain, _ = run(0, True)
    assert g0 == 0 and g1 > 0
    total = sum(len(o.token_ids) for o in plain)
    assert all(len(o.token_ids) == 24 for o in graph)
    for other in (eager, plain):
        same = sum(a == b for x, y in zip(graph, other) for a, b in zip(x.token_ids, y.token_ids))
        assert same >= 0.9 * total
    assert sum(o.proposed for o in graph) > 0


def test_set_speculation_switches_between_requests_cpu():
    m = build_model(_cfg(), device="cpu", seed=1)
    m.act_dtype = torch.float32
    prompts = [list(range(3, 40)), list(range(50, 61))]
    base, _ = _run(m, 0, prompts, 10)
    rc = RunnerConfig(block_size=64, max_seqs=4, max_model_len=512, max_batched_tokens=128, use_cuda_graph=False,
                      num_spec=3)
    llm = LLM(m, device="cpu", runner_config=rc)
    for k in (0, 2, 3, 0):
        llm.set_speculation(k)
        outs = llm.generate(prompts, SamplingParams(max_tokens=10))
        assert [o.token_ids for o in outs] == [o.token_ids for o in base], k
        assert all((o.proposed > 0) == (k > 0) for o in outs)
    with pytest.raises(ValueError):
        llm.set_speculation(4)
    llm.shutdown()


def test_rejection_sampling_emits_the_target_distribution():
    """verify_sampled with a point-mass draft: the first emitted token is distributed as the
    target's filtered distribution whatever the draft (here a likely one and an unlikely
    one), and a fully accepted chain ends with a draw from the last row."""
    from vllm_xtu_moe_b200.engine.spec_decode import verify_sampled
    from vllm_xtu_moe_b200.engine.sampling import filtered_probs
    torch.manual_seed(0)
    V = 12
    logits = torch.randn(3, V) * 1.5
    sp = SamplingParams(temperature=0.8, top_k=8, max_tokens=1)
    p0 = filtered_probs(logits[0], 0.8, 8)
    for draft0 in (int(p0.argmax()), int(p0.argmin())):
        g = torch.Generator().manual_seed(1)
        N = 6000
        counts = torch.zeros(V)
        lens = []
        for _ in range(N):
            toks = verify_sampled(logits, [draft0, 3], sp, g)
            counts[toks[0]] += 1
            lens.append(len(toks))
        emp = counts / N
        assert (emp - p0).abs().max().item() < 0.025, (draft0, emp, p0)
        assert min(lens) >= 1 and max(lens) <= 3
    # drafts of probability 1 are always kept
    sharp = torch.full((3, V), -30.0)
    sharp[0, 4] = sharp[1, 5] = sharp[2, 6] = 30.0
    toks = verify_sampled(sharp, [4, 5], SamplingParams(temperature=1.0, max_tokens=1), torch.Generator())
    assert toks == [4, 5, 6]


def test_sampled_requests_with_mtp_cpu():
    """Sampled requests run with MTP drafts (rejection sampling); a seeded request repeats
    its tokens, and greedy requests in the same batch still equal plain greedy decoding."""
    m = build_model(_cfg(), device="cpu", seed=1)
    m.act_dtype = torch.float32
    prompts = [list(range(3, 40)), list(range(50, 61))]
    base, _ = _run(m, 0, prompts, 10)
    rc = RunnerConfig(block_size=64, max_seqs=4, max_model_len=512, max_batched_tokens=128, use_cuda_graph=False,
                      num_spec=3)
    outs = []
    for _ in range(2):
        llm = LLM(m, device="cpu", runner_config=rc)
        ra = llm.add_request(prompts[0], SamplingParams(max_tokens=10))
        rb = llm.add_request(prompts[1], SamplingParams(max_tokens=10, temperature=0.9, seed=7))
        while llm.scheduler.has_work():
            llm.step()
        outs.append((list(ra.output), list(rb.output), rb.proposed))
        llm.shutdown()
    assert outs[0][0] == base[0].token_ids            # the greedy request is unchanged
    assert outs[0][1] == outs[1][1] and len(outs[0][1]) == 10
    assert outs[0][2] > 0                              # the sampled request was drafted for


@pytest.mark.gpu
def test_spec_decode_linear_attention_gpu():
    """Hybrid DeltaNet + gated-GQA model with MTP on the GPU.  Oracle drafts (the plain run's
    own tokens, then a wrong tail, so every step rolls the recurrent state back) must be
    accepted and reproduce plain greedy decoding; the graph-replayed step must run.  (MTP
    drafts of a random model are rejected, and bf16 ties between differently shaped kernels
    can flip a random model's argmax, so the drafter's own tokens are not compared.)"""
    cfg = _qwen_cfg().replace(linear_key_head_dim=128, linear_value_head_dim=128, linear_num_key_heads=1,
                              linear_num_value_heads=2)
    m = build_model(cfg, device="cuda", seed=2)
    prompts = [list(range(3, 40)), list(range(50, 61))]
    base, _ = _run(m, 0, prompts, 16, device="cuda")
    half = {tuple(p): (o.token_ids[:2] + [1, 2, 3] * 8) for p, o in zip(prompts, base)}
    exact = {tuple(p): o.token_ids for p, o in zip(prompts, base)}
    for oracle in (exact, half):
        spec, _ = _run(m, 3, prompts, 16, device="cuda", oracle=oracle)
        same = sum(a == b for x, y in zip(base, spec) for a, b in zip(x.token_ids, y.token_ids))
        assert same >= 0.9 * sum(len(o.token_ids) for o in base), ([o.token_ids for o in base],
                                                                    [o.token_ids for o in spec])
    assert sum(o.accepted for o in spec) > 0
    rc = RunnerConfig(block_size=64, max_seqs=4, max_model_len=512, max_batched_tokens=128, use_cuda_graph=True,
                      num_spec=3)
    llm = LLM(m, device="cuda", runner_config=rc)
    outs = llm.generate(prompts, SamplingParams(max_tokens=12))
    assert llm.spec.graph_steps > 0 and all(len(o.token_ids) == 12 for o in outs)
    llm.shutdown()
