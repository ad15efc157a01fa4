"""xtu_argmax_static (argmax with its scratch in a fixed device array) against the
allocating xtu_argmax, called through the library's exported C symbol.

Kept in a file of its own, collected last, so that it runs both alone in a fresh
process and after every other test has used the library.
"""
import ctypes

import pytest
import torch

from vllm_xtu_moe_b200.ops import _native as N

MAX_ROWS = 1024
ERR_TOO_MANY_ROWS = -10001


def _fn():
    L = ctypes.CDLL(str(N._CUDA_LIB), mode=ctypes.RTLD_GLOBAL)
    f = L.xtu_argmax_static
    f.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                  ctypes.c_void_p, ctypes.c_void_p]
    f.restype = ctypes.c_int
    return f


def _existing(logits, V):
    T = logits.shape[0]
    out = torch.empty(T, dtype=torch.int32, device=logits.device)
    val = torch.empty(T, dtype=torch.float32, device=logits.device)
    ws = torch.empty(T * 64 * 8, dtype=torch.uint8, device=logits.device)
    rc = N.lib().xtu_argmax(logits.data_ptr(), int(logits.dtype == torch.bfloat16), T, V, logits.stride(0),
                            out.data_ptr(), val.data_ptr(), ws.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc > 0
    return out, val


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,T,V", [(torch.bfloat16, 5, 151552), (torch.float32, 3, 50000),
                                       (torch.bfloat16, 7, 4000), (torch.float32, MAX_ROWS, 20000)])
def test_argmax_static_matches_allocating_entry(dtype, T, V):
    f = _fn()
    s = torch.cuda.current_stream().cuda_stream
    g = torch.Generator(device="cuda").manual_seed(T * 131 + V)
    for call in range(2):                     # two calls in a row, fresh logits each
        full = torch.randn(T, V + 64, device="cuda", generator=g).to(dtype)
        full[:, 17] = full.max() + 1 if call == 0 else full[:, 17]   # a clear winner in the first call
        logits = full[:, :V]                  # padded rows: stride > V
        out = torch.full((T,), -1, dtype=torch.int32, device="cuda")
        val = torch.full((T,), float("nan"), dtype=torch.float32, device="cuda")
        rc = f(logits.data_ptr(), int(dtype == torch.bfloat16), T, V, logits.stride(0), out.data_ptr(),
               val.data_ptr(), s)
        assert rc in (1, 2), rc
        ref_i, ref_v = _existing(logits, V)
        torch.cuda.synchronize()
        assert torch.equal(out, ref_i), call
        assert torch.equal(val, ref_v), call
        exp = logits.float().max(dim=1)
        assert torch.equal(val.cpu(), exp.values.cpu())


@pytest.mark.gpu
def test_argmax_static_rejects_rows_beyond_its_array():
    f = _fn()
    logits = torch.zeros(MAX_ROWS + 1, 16, device="cuda")
    out = torch.zeros(MAX_ROWS + 1, dtype=torch.int32, device="cuda")
    rc = f(logits.data_ptr(), 0, MAX_ROWS + 1, 16, 16, out.data_ptr(), None,
           torch.cuda.current_stream().cuda_stream)
    assert rc == ERR_TOO_MANY_ROWS


@pytest.mark.gpu
@pytest.mark.parametrize("V", [4000, 151552])
def test_argmax_static_rows_without_a_winner_return_index_zero(V):
    """A row of all -inf (or NaN) has no element above the starting value: both entry
    points return index 0, a valid token id, for it."""
    f = _fn()
    s = torch.cuda.current_stream().cuda_stream
    logits = torch.randn(3, V, device="cuda")
    logits[0] = float("-inf")
    logits[2] = float("nan")
    for call in range(2):
        out = torch.full((3,), -1, dtype=torch.int32, device="cuda")
        rc = f(logits.data_ptr(), 0, 3, V, V, out.data_ptr(), None, s)
        assert rc in (1, 2), rc
        ref_i, _ = _existing(logits, V)
        torch.cuda.synchronize()
        assert torch.equal(out, ref_i), call
        assert out[0].item() == 0 and out[2].item() == 0
        assert out[1].item() == int(logits[1].argmax())
