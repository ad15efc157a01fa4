"""Paged KV block accounting, including the sliding-window pool's release of blocks no
future query can see."""
from vllm_xtu_moe_b200.engine.block_manager import BlockManager, swa_pool_blocks
from vllm_xtu_moe_b200.engine.sequence import Request, SamplingParams


def _req(n_prompt):
    return Request(list(range(n_prompt)), SamplingParams(max_tokens=1000))


def test_full_pool_allocates_and_releases():
    bm = BlockManager(10, 16, 2)
    r = _req(40)
    assert bm.ensure(r, 40) and len(r.blocks) == 3 and bm.num_free == 7
    assert not bm.can_allocate(r, 16 * 11) and bm.can_allocate(r, 16 * 10)
    bm.release(r)
    assert bm.num_free == 10 and r.blocks == []


def test_window_pool_stays_bounded_over_a_long_sequence():
    W, bs = 40, 16
    nb = swa_pool_blocks(1, W, bs, 64)
    bm = BlockManager(200, bs, 1, swa_blocks=nb, window=W)
    r = _req(100)
    # chunked prefill of 100 tokens in chunks of 64, then 300 decode steps
    assert bm.ensure(r, 64)
    r.num_computed = 64
    assert bm.ensure(r, 100)
    r.num_computed = 100
    r.output.append(1)
    most = 0
    for _ in range(300):
        assert bm.ensure(r, r.total_len + 1)
        first_query = r.num_computed
        lo = max(0, first_query - W + 1) // bs
        # every block a query of this step can see is held, nothing older
        need = set(range(lo, (r.total_len + 1 + bs - 1) // bs))
        assert need <= set(r.swa_blocks) and min(r.swa_blocks) >= lo
        most = max(most, len(r.swa_blocks))
        r.num_computed = r.total_len
        r.output.append(1)
    assert most <= (W + bs - 1) // bs + 2
    held = len(r.swa_blocks)
    assert len(bm.swa_free) == nb - held
    bm.release(r)
    assert len(bm.swa_free) == nb and bm.num_free == 200


def test_window_pool_refuses_without_partial_allocation():
    bm = BlockManager(100, 16, 2, swa_blocks=3, window=16)
    a, b = _req(40), _req(40)
    assert bm.ensure(a, 40) and len(a.swa_blocks) == 3
    free_before = bm.num_free
    assert not bm.can_allocate(b, 40)
    assert not bm.ensure(b, 40)
    assert b.swa_blocks == {} and b.blocks == [] and bm.num_free == free_before


def _tiny_llm(prefix, num_blocks=0):
    from vllm_xtu_moe_b200.engine import LLM
    from vllm_xtu_moe_b200.engine.runner import RunnerConfig
    from vllm_xtu_moe_b200.models.config import get_preset
    return LLM(get_preset("tiny-mixtral"), device="cpu",
               runner_config=RunnerConfig(block_size=16, max_seqs=2, max_model_len=256, max_batched_tokens=64,
                                          use_cuda_graph=False, prefix_caching=prefix, num_blocks=num_blocks))


def test_prefix_caching_reuses_blocks_and_keeps_outputs():
    """Requests that share a prompt prefix start from its cached blocks: the same tokens as
    without caching, fewer prompt tokens computed; with a pool too small to keep them,
    cached blocks are evicted and outputs still match."""
    shared = list(range(3, 3 + 50))
    prompts = [shared + [7, 8, 9], shared + [100, 101], shared[:40] + [5], list(range(200, 230))]
    sp = SamplingParams(max_tokens=6)
    base = _tiny_llm(False)
    want = [base.generate([p], sp)[0].token_ids for p in prompts]
    for nb in (0, 12):
        llm = _tiny_llm(True, nb)
        got = [llm.generate([p], sp)[0].token_ids for p in prompts]
        assert got == want, nb
        if nb == 0:
            assert llm.blocks.prefix_hits == 48 + 32        # 3 full blocks, then 2
            assert llm.stats["prefill_tokens"] == sum(len(p) for p in prompts) - 80
        assert llm.blocks.num_free == llm.blocks.num_blocks   # every block back (free or cached)


def test_abort_frees_a_running_request():
    llm = _tiny_llm(False)
    r = llm.add_request(list(range(1, 40)), SamplingParams(max_tokens=50))
    other = llm.add_request(list(range(5, 30)), SamplingParams(max_tokens=3))
    for _ in range(3):
        llm.step()
    assert llm.abort(r.rid) and not llm.abort(r.rid)
    while llm.scheduler.has_work():
        llm.step()
    assert len(other.output) == 3 and r.blocks == [] and r.slot == -1
    assert llm.blocks.num_free == llm.blocks.num_blocks
