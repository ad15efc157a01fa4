"""Bounds-check build (XTU_CHECKED=1 loads libxtu_cuda_checked.so, compiled with
-DXTU_BOUNDS_CHECK): host-supplied indices past their buffers (KV slot mapping, token
ids, KV page ids) are recorded as XTU_ERR_BOUNDS in the status word and the access is
skipped instead of trapping.  Every index used here still falls inside allocated padding
(the kernels get views of padded tensors), so even a missing check could not fault."""
import os
import subprocess
import sys
import textwrap

import pytest
import torch

_SCRIPT = textwrap.dedent('''
    import sys, torch
    sys.path.insert(0, ".")
    from vllm_xtu_moe_b200.ops import _native as N, basic as B
    from vllm_xtu_moe_b200.ops.attention import AttnMetadata, paged_attention
    checked = N._CUDA_LIB.name.endswith("_checked.so")
    d = torch.device("cuda", 0)
    errors = []

    def expect(bad, what):
        torch.cuda.synchronize()
        try:
            N.check_status(d)
            raised = False
        except RuntimeError as e:
            raised = "bounds" in str(e)
        if raised != (bad and checked):
            errors.append((what, raised))

    # KV write: slot one block past a 4-block view of a 6-block cache
    nb, bs, Hk, D = 4, 64, 2, 64
    kc_full = torch.zeros(nb + 2, Hk, bs, D, dtype=torch.bfloat16, device=d)
    vc_full = torch.zeros_like(kc_full)
    k = torch.randn(2, Hk, D, device=d).to(torch.bfloat16)
    for slots, bad in (([3, 70], False), ([3, nb * bs + 5], True)):
        B.write_kv(k, k, torch.tensor(slots, dtype=torch.int32, device=d), kc_full[:nb], vc_full[:nb])
        expect(bad, f"kv_write {slots}")
    assert torch.count_nonzero(kc_full[nb:]) == 0, "a slot past the cache was written"

    # embedding: id == vocab of a padded table
    table = torch.randn(12, 64, device=d).to(torch.bfloat16)
    for ids, bad in (([1, 9], False), ([1, 10], True)):
        B.embed(torch.tensor(ids, dtype=torch.int32, device=d), table[:10])
        expect(bad, f"embed {ids}")

    # decode attention: a page id past the cache (TMA bounds: zero fill, nothing read)
    Hq = 8
    q = torch.randn(1, Hq, D, device=d).to(torch.bfloat16)
    for page, bad in ((2, False), (nb + 1, True)):
        meta = AttnMetadata(num_seqs=1, q_start=torch.tensor([0, 1], dtype=torch.int32, device=d),
                            kv_len=torch.tensor([100], dtype=torch.int32, device=d),
                            block_table=torch.tensor([[1, page]], dtype=torch.int32, device=d),
                            slot_mapping=torch.zeros(1, dtype=torch.int32, device=d),
                            positions=torch.zeros(1, dtype=torch.int32, device=d), max_q_len=1, max_kv_len=100,
                            is_decode=True)
        paged_attention(q, kc_full[:nb], vc_full[:nb], meta)
        expect(bad, f"attention page {page}")
    print("errors:", errors)
    print("OK" if not errors else "FAIL")
''')


@pytest.mark.gpu
@pytest.mark.parametrize("checked", ["1", "0"])
def test_bounds_checks_report_without_faulting(checked):
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    lib = os.path.join(root, "vllm_xtu_moe_b200", "_lib",
                       "libxtu_cuda_checked.so" if checked == "1" else "libxtu_cuda.so")
    if not os.path.exists(lib):
        pytest.fail(f"{lib} is not built")
    env = dict(os.environ, XTU_CHECKED=checked)
    r = subprocess.run([sys.executable, "-c", _SCRIPT], cwd=root, env=env, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0 and "OK" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]


def test_bounds_check_build_exists():
    """__graft_entry__.build() / _build.build_all() produce the bounds-check library too."""
    from vllm_xtu_moe_b200 import _build
    assert "checked" in _build.build_cuda.__doc__
