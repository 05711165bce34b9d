"""GPU parity tests of the variable-length entry point fa2.kernel.attention_varlen (an extension:
the reference's README lists variable-length batches out of scope).

Sequences are packed along one token axis, q [total_q, H_q, D], k/v [total_k, H_kv, D], with
int32 prefix sums cu_seqlens (the layout of flash_attn_varlen_func). The oracle is the
reference's naive_attention applied to each sequence on its own (oracle.naive_attention_varlen,
fp64); the bar is the reference's rule, max|ours - ref| <= 2 * max|SDPA - ref| + 1e-4, with
SDPA also run per sequence at the input dtype.
"""

import itertools

import pytest
import torch
import torch.nn.functional as F

from fa2 import _lib
from fa2.kernel import attention, attention_varlen, check_device_errors
from oracle.reference import naive_attention_varlen

pytestmark = pytest.mark.gpu

ATOL_FLOOR = 1e-4


@pytest.fixture(autouse=True)
def _no_device_errors():
    yield
    check_device_errors()


def packed_inputs(lens_q, lens_k, H_q, H_kv, D, dtype, seed=0):
    g = torch.Generator().manual_seed(seed)
    tq, tk = sum(lens_q), sum(lens_k)
    q = torch.randn(tq, H_q, D, generator=g).to(dtype).cuda()
    k = torch.randn(tk, H_kv, D, generator=g).to(dtype).cuda()
    v = torch.randn(tk, H_kv, D, generator=g).to(dtype).cuda()
    cq = torch.tensor([0, *itertools.accumulate(lens_q)], dtype=torch.int32).cuda()
    ck = torch.tensor([0, *itertools.accumulate(lens_k)], dtype=torch.int32).cuda()
    return q, k, v, cq, ck


def sdpa_varlen(q, k, v, cq, ck, causal, align):
    out = torch.zeros_like(q)
    cq, ck = cq.tolist(), ck.tolist()
    for b in range(len(cq) - 1):
        nq, nk = cq[b + 1] - cq[b], ck[b + 1] - ck[b]
        if nq == 0 or nk == 0:
            continue
        qs = q[cq[b]:cq[b + 1]].transpose(0, 1).unsqueeze(0)
        ks = k[ck[b]:ck[b + 1]].transpose(0, 1).unsqueeze(0)
        vs = v[ck[b]:ck[b + 1]].transpose(0, 1).unsqueeze(0)
        mask = None
        if causal:
            shift = nk - nq if align == "bottom_right" else 0
            mask = torch.ones(nq, nk, dtype=torch.bool, device=q.device).tril(diagonal=shift)
        o = F.scaled_dot_product_attention(qs, ks, vs, attn_mask=mask, enable_gqa=True)
        out[cq[b]:cq[b + 1]] = torch.nan_to_num(o, nan=0.0)[0].transpose(0, 1)
    return out


def check_varlen(lens_q, lens_k, H_q, H_kv, D, dtype, causal, align="top_left", seed=0, **kw):
    q, k, v, cq, ck = packed_inputs(lens_q, lens_k, H_q, H_kv, D, dtype, seed)
    ours = attention_varlen(q, k, v, cq, ck, max(lens_q), max(lens_k), causal=causal, causal_align=align, **kw)
    ref = naive_attention_varlen(q, k, v, cq, ck, causal=causal, dtype=torch.float64, causal_align=align)
    theirs = sdpa_varlen(q, k, v, cq, ck, causal, align)
    torch.cuda.synchronize()
    e_ours = (ours.double() - ref).abs().max().item()
    e_sdpa = (theirs.double() - ref).abs().max().item()
    assert torch.isfinite(ours).all()
    assert e_ours <= 2 * e_sdpa + ATOL_FLOOR, f"max-abs {e_ours:.3e} vs torch {e_sdpa:.3e}"
    return ours


LENS = [1, 130, 257, 1000, 77, 128]


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("H_q,H_kv", [(8, 8), (16, 4), (8, 1)])
@pytest.mark.parametrize("D,dtype", [(128, torch.bfloat16), (64, torch.float16)])
def test_varlen_equal_lengths(causal, H_q, H_kv, D, dtype):
    check_varlen(LENS, LENS, H_q, H_kv, D, dtype, causal)


@pytest.mark.parametrize("pack_gqa", [True, False])
def test_varlen_bottom_right_longer_keys(pack_gqa):
    """Chunked prefill: each sequence's queries are the last n_q of its n_k positions."""
    lens_q = [1, 7, 300, 64, 129]
    lens_k = [1000, 8192, 300, 700, 2000]
    check_varlen(lens_q, lens_k, 16, 4, 128, torch.bfloat16, True, "bottom_right", pack_gqa=pack_gqa)


@pytest.mark.parametrize("align", ["top_left", "bottom_right"])
def test_varlen_unequal_lengths_causal(align):
    """Per-sequence causal masks with n_q != n_k both ways; bottom-right rows before the first key
    (n_q > n_k) and sequences without keys get zeros."""
    lens_q = [200, 5, 300, 0, 40]
    lens_k = [100, 50, 300, 10, 0]
    check_varlen(lens_q, lens_k, 8, 2, 128, torch.bfloat16, True, align)


def test_varlen_noncausal_different_lengths():
    check_varlen([3, 500, 1, 260], [4000, 17, 900, 260], 32, 8, 128, torch.bfloat16, False)


def test_varlen_matches_fixed_length_bit_for_bit():
    """Equal lengths packed along the token axis compute the same tiles in the same order as the
    [B, H, N, D] path: the outputs are identical."""
    B, H, Hkv, N, D = 3, 16, 4, 777, 128
    g = torch.Generator().manual_seed(3)
    q = torch.randn(B, H, N, D, generator=g).to(torch.bfloat16).cuda()
    k = torch.randn(B, Hkv, N, D, generator=g).to(torch.bfloat16).cuda()
    v = torch.randn(B, Hkv, N, D, generator=g).to(torch.bfloat16).cuda()
    cu = torch.arange(0, (B + 1) * N, N, dtype=torch.int32).cuda()
    for causal in (True, False):
        fixed = attention(q, k, v, causal=causal)
        pk = lambda t: t.transpose(1, 2).reshape(B * N, t.shape[1], D)  # noqa: E731
        var = attention_varlen(pk(q), pk(k), pk(v), cu, cu, N, N, causal=causal)
        assert torch.equal(var, pk(fixed))


def test_varlen_every_row_written_and_nothing_else():
    """NaN canary through the C ABI: an output buffer pre-filled with NaN has no NaN left after
    the launch (every row of every sequence is written, including the row-by-row ends of boxes
    that cross a sequence boundary), and a sequence's rows depend only on that sequence (its
    output equals a launch of that sequence alone)."""
    lens = [5, 300, 33, 1000]
    q, k, v, cq, ck = packed_inputs(lens, lens, 16, 2, 128, torch.bfloat16, seed=4)
    out = torch.full_like(q, float("nan"))
    st = lambda t: (0, t.stride(1), t.stride(0), t.stride(2))  # noqa: E731
    p = _lib.make_params(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), st(q), st(k), st(v), st(out),
                         len(lens), 16, 2, max(lens), max(lens), 128, _lib.FA2_DTYPE_BF16, 1, 1,
                         1.4426950408889634 / 128 ** 0.5, cu_seqlens_q=cq.data_ptr(), cu_seqlens_kv=ck.data_ptr(),
                         total_q=sum(lens), total_kv=sum(lens))
    assert _lib.launch(p, torch.cuda.current_stream().cuda_stream) == _lib.FA2_OK
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
    assert torch.equal(out, attention_varlen(q, k, v, cq, ck, max(lens), max(lens), causal=True))
    c = cq.tolist()
    for b in range(len(lens)):
        one = torch.tensor([0, lens[b]], dtype=torch.int32).cuda()
        alone = attention_varlen(q[c[b]:c[b + 1]], k[c[b]:c[b + 1]], v[c[b]:c[b + 1]], one, one,
                                 lens[b], lens[b], causal=True)
        assert torch.equal(alone, out[c[b]:c[b + 1]])


@pytest.mark.parametrize("D", [16, 32])
def test_varlen_small_head_dim(D):
    """The rows of a box that crosses a sequence end are written from registers: only the
    head_dim columns."""
    check_varlen([50, 200, 3, 700], [50, 200, 3, 700], 4, 2, D, torch.float16, True)
    check_varlen([50, 200, 3, 700], [50, 200, 3, 700], 8, 8, D, torch.bfloat16, False)


def test_varlen_longer_than_declared_is_reported():
    """A sequence longer than max_seqlen_q: the kernel reports FA2_ERR_SHAPE in the error word
    (no fault) and leaves that sequence out."""
    q, k, v, cq, ck = packed_inputs([100, 300], [100, 300], 4, 4, 64, torch.float16)
    attention_varlen(q, k, v, cq, ck, 200, 300, causal=False)
    with pytest.raises(RuntimeError, match=f"status {_lib.FA2_ERR_SHAPE}"):
        check_device_errors()
