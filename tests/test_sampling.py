"""Sampled decoding: the filtered distribution (temperature, top-k, top-p), draws that
follow it, seeded reproducibility through the engine, and greedy limits."""
import pytest
import torch

from vllm_xtu_moe_b200.engine import LLM, SamplingParams
from vllm_xtu_moe_b200.engine.runner import RunnerConfig
from vllm_xtu_moe_b200.engine.sampling import filtered_probs, sample_rows
from vllm_xtu_moe_b200.models.config import get_preset


def test_filtered_probs_top_k_and_top_p():
    logits = torch.tensor([2.0, 1.0, 0.5, -1.0, -3.0])
    p = filtered_probs(logits, 1.0)
    assert torch.allclose(p, torch.softmax(logits, 0))
    pk = filtered_probs(logits, 1.0, top_k=2)
    assert (pk[2:] == 0).all() and torch.allclose(pk[:2], torch.softmax(logits[:2], 0))
    sm = torch.softmax(logits, 0)
    pp = filtered_probs(logits, 1.0, top_p=float(sm[0] + 0.5 * sm[1]))   # needs the top two
    assert (pp[2:] == 0).all() and torch.allclose(pp[:2], sm[:2] / sm[:2].sum())
    cold = filtered_probs(logits, 1e-4)
    assert cold[0] > 0.999


def test_draws_follow_the_distribution():
    class R:
        pass

    logits = torch.log(torch.tensor([0.5, 0.3, 0.15, 0.05]))
    r = R()
    r.params = SamplingParams(temperature=1.0, seed=7)
    counts = torch.zeros(4)
    for _ in range(4000):
        t = sample_rows(logits[None], [r], torch.zeros(1, dtype=torch.int32))
        counts[int(t[0])] += 1
    freq = counts / counts.sum()
    assert (freq - torch.tensor([0.5, 0.3, 0.15, 0.05])).abs().max() < 0.03


def _llm():
    return LLM(get_preset("tiny-mixtral"), device="cpu",
               runner_config=RunnerConfig(block_size=16, max_seqs=4, max_model_len=256, max_batched_tokens=64,
                                          use_cuda_graph=False))


def test_seeded_sampling_is_reproducible_and_top_k_one_is_greedy():
    prompts = [list(range(1, 30)), list(range(40, 55))]
    llm = _llm()
    greedy = [o.token_ids for o in llm.generate(prompts, SamplingParams(max_tokens=8))]
    a = [o.token_ids for o in llm.generate(prompts, SamplingParams(max_tokens=8, temperature=1.5, seed=3))]
    b = [o.token_ids for o in llm.generate(prompts, SamplingParams(max_tokens=8, temperature=1.5, seed=3))]
    c = [o.token_ids for o in llm.generate(prompts, SamplingParams(max_tokens=8, temperature=1.5, seed=4))]
    k1 = [o.token_ids for o in llm.generate(prompts, SamplingParams(max_tokens=8, temperature=1.0, top_k=1, seed=5))]
    assert a == b and a != c
    assert k1 == greedy


def test_mixed_greedy_and_sampled_rows_in_one_batch():
    llm = _llm()
    prompts = [list(range(1, 30)), list(range(40, 55))]
    greedy = [o.token_ids for o in llm.generate(prompts, SamplingParams(max_tokens=6))]
    out = llm.generate(prompts, [SamplingParams(max_tokens=6), SamplingParams(max_tokens=6, temperature=2.0, seed=1)])
    assert out[0].token_ids == greedy[0]
    assert len(out[1].token_ids) == 6


@pytest.mark.gpu
def test_sampling_from_decode_graph_logits():
    """On the GPU decode runs from CUDA graphs; sampled rows are drawn from the graph's
    logits output after each replay: seeded runs reproduce and top_k=1 is greedy."""
    llm = LLM(get_preset("tiny-mixtral"), device="cuda",
              runner_config=RunnerConfig(block_size=64, max_seqs=2, max_model_len=256, max_batched_tokens=128,
                                         use_cuda_graph=True, graph_batch_sizes=(1, 2)))
    prompts = [list(range(1, 30)), list(range(40, 55))]
    greedy = [o.token_ids for o in llm.generate(prompts, SamplingParams(max_tokens=8))]
    a = [o.token_ids for o in llm.generate(prompts, SamplingParams(max_tokens=8, temperature=1.5, seed=3))]
    b = [o.token_ids for o in llm.generate(prompts, SamplingParams(max_tokens=8, temperature=1.5, seed=3))]
    k1 = [o.token_ids for o in llm.generate(prompts, SamplingParams(max_tokens=8, temperature=1.0, top_k=1, seed=5))]
    assert a == b and a != greedy and k1 == greedy
    llm.shutdown()


def test_logprobs_of_greedy_tokens():
    """Greedy tokens come with their log-probability, which is the best of the returned
    alternatives; sampled tokens' log-probabilities are finite and not above 0."""
    llm = _llm()
    out = llm.generate([list(range(1, 30))], SamplingParams(max_tokens=6, logprobs=3))[0]
    assert len(out.logprobs) == 6
    for tok, (lp, alt) in zip(out.token_ids, out.logprobs):
        assert len(alt) == 3 and lp <= 0.0
        assert abs(lp - max(alt.values())) < 1e-5 and tok in alt
    s = llm.generate([list(range(1, 30))], SamplingParams(max_tokens=6, temperature=1.0, seed=2, logprobs=0))[0]
    assert len(s.logprobs) == 6 and all(lp <= 0.0 and alt == {} for lp, alt in s.logprobs)
    assert llm.generate([list(range(1, 30))], SamplingParams(max_tokens=2))[0].logprobs is None
