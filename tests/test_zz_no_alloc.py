"""The allocation-free entry point fa2_fwd_sm100_noalloc, called through the C ABI.

It serves callers that cannot allocate device memory at call time (code inside a CUDA graph
being captured, runtimes that own all device allocations, plugins handed only input and
output pointers): the split-KV forward keeps its fp32 partials in a static device array
that belongs to the library instead of a caller workspace. The test compares it with the
regular entry point fa2_fwd_sm100 (given a torch-allocated workspace) on the same split
configuration, on two calls in a row. Between them an unrelated call (other data, other split
layout) leaves its own partials in the shared array, so a slot that a call read before writing
it would show up as a mismatch. It also checks that a call needing more than the array is
refused.
This file sorts last so a run that stops at the first failure has run every other test.
"""

import ctypes
import math

import pytest
import torch

from fa2 import _lib
from oracle.reference import make_qkv

pytestmark = pytest.mark.gpu


def _params(q, k, v, o, num_splits):
    B, Hq, Nq, D = q.shape
    Hkv, Nkv = k.shape[1], k.shape[2]
    return _lib.make_params(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                            q.stride(), k.stride(), v.stride(), o.stride(),
                            B, Hq, Hkv, Nq, Nkv, D, _lib.FA2_DTYPE_BF16, 0, 1,
                            1.4426950408889634 / math.sqrt(D), num_splits=num_splits)


def test_noalloc_matches_regular_entry_point_twice():
    L = _lib.lib()
    stream = torch.cuda.current_stream().cuda_stream
    q, k, v = make_qkv(4, 32, 8, 3, 16384, 128, torch.bfloat16, seed=11, device="cuda")
    splits = 4

    # regular entry point, caller-provided workspace
    ref = torch.empty_like(q)
    p = _params(q, k, v, ref, splits)
    ws = torch.empty(_lib.workspace_bytes(p), dtype=torch.uint8, device="cuda")
    p.workspace, p.workspace_bytes = ws.data_ptr(), ws.numel()
    assert _lib.workspace_bytes(p) <= _lib.NOALLOC_SCRATCH_BYTES
    assert L.fa2_fwd_sm100(ctypes.byref(p), ctypes.c_void_p(stream)) == _lib.FA2_OK

    # an unrelated call: different values, 8 splits over another K/V length, 12 query rows
    q2, k2, v2 = make_qkv(2, 32, 8, 12, 9000, 128, torch.bfloat16, seed=12, device="cuda")
    other = torch.empty_like(q2)

    for i in range(2):  # two calls in a row on the shared static scratch
        out = torch.full_like(q, float("nan"))
        pn = _params(q, k, v, out, splits)
        assert L.fa2_fwd_sm100_noalloc(ctypes.byref(pn), ctypes.c_void_p(stream)) == _lib.FA2_OK
        torch.cuda.synchronize()
        assert torch.isfinite(out).all()
        assert torch.equal(out, ref)
        if i == 0:
            po = _params(q2, k2, v2, other, 8)
            assert L.fa2_fwd_sm100_noalloc(ctypes.byref(po), ctypes.c_void_p(stream)) == _lib.FA2_OK
            torch.cuda.synchronize()
            assert torch.isfinite(other).all()

    # and both agree with the fp64 oracle within the suite's bar
    from oracle.reference import naive_attention
    import torch.nn.functional as F
    truth = naive_attention(q, k, v, causal=False, dtype=torch.float64)
    sdpa = F.scaled_dot_product_attention(q, k, v, is_causal=False, enable_gqa=True)
    e_ours = (out.double() - truth).abs().max().item()
    e_sdpa = (sdpa.double() - truth).abs().max().item()
    assert e_ours <= 2 * e_sdpa + 1e-4


def test_noalloc_rejects_calls_beyond_the_scratch():
    L = _lib.lib()
    q, k, v = make_qkv(64, 32, 8, 256, 2048, 128, torch.bfloat16, seed=1, device="cuda")
    out = torch.zeros_like(q)
    p = _params(q, k, v, out, 8)
    assert _lib.workspace_bytes(p) > _lib.NOALLOC_SCRATCH_BYTES
    rc = L.fa2_fwd_sm100_noalloc(ctypes.byref(p), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == _lib.FA2_ERR_SCRATCH_LIMIT
    torch.cuda.synchronize()
    assert torch.count_nonzero(out) == 0  # nothing was launched
