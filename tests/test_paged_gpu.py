"""GPU parity tests of the paged K/V entry point fa2.kernel.attention_kvcache (an extension: the
reference's README lists paged K/V out of scope).

K and V live in a cache of pages [num_pages, page_size, H_kv, D] (the layout of
flash_attn_with_kvcache); sequence b's key j is in page block_table[b, j // page_size], row
j % page_size, and cache_seqlens[b] says how many keys it has. Pages are handed out in a shuffled
order and the unused table entries hold an out-of-range index, so reading a table entry past a
sequence's last page, or a wrong page, shows up. The oracle gathers each sequence's keys and runs
the reference's naive_attention on it (oracle.naive_attention_paged, fp64); the bar is the
reference's rule, max|ours - ref| <= 2 * max|SDPA - ref| + 1e-4, SDPA run per sequence.
"""

import pytest
import torch
import torch.nn.functional as F

from fa2 import _lib
from fa2.kernel import attention, attention_kvcache, check_device_errors
from oracle.reference import naive_attention_paged

pytestmark = pytest.mark.gpu

ATOL_FLOOR = 1e-4


@pytest.fixture(autouse=True)
def _no_device_errors():
    yield
    check_device_errors()


def paged_inputs(B, H_q, H_kv, N_q, seqlens, page_size, D, dtype, seed=0, shuffle=True):
    g = torch.Generator().manual_seed(seed)
    pages_per_seq = max(1, -(-max(seqlens) // page_size))
    num_pages = B * pages_per_seq + 3
    q = torch.randn(B, H_q, N_q, D, generator=g).to(dtype).cuda()
    k = torch.randn(num_pages, page_size, H_kv, D, generator=g).to(dtype).cuda()
    v = torch.randn(num_pages, page_size, H_kv, D, generator=g).to(dtype).cuda()
    order = torch.randperm(num_pages, generator=g) if shuffle else torch.arange(num_pages)
    bt = torch.full((B, pages_per_seq), num_pages + 1000, dtype=torch.int32)  # out of range on purpose
    used = 0
    for b, n in enumerate(seqlens):
        need = -(-n // page_size)
        bt[b, :need] = order[used:used + need].to(torch.int32)
        used += need
    return q, k, v, bt.cuda(), torch.tensor(seqlens, dtype=torch.int32).cuda()


def sdpa_paged(q, k, v, bt, sl, causal, align):
    out = torch.zeros_like(q)
    ps = k.shape[1]
    for b, n in enumerate(sl.tolist()):
        if n == 0:
            continue
        pages = bt[b, :-(-n // ps)].long()
        ks = k[pages].reshape(-1, *k.shape[2:])[:n].transpose(0, 1).unsqueeze(0)
        vs = v[pages].reshape(-1, *v.shape[2:])[:n].transpose(0, 1).unsqueeze(0)
        mask = None
        if causal:
            nq = q.shape[2]
            shift = n - nq if align == "bottom_right" else 0
            mask = torch.ones(nq, n, dtype=torch.bool, device=q.device).tril(diagonal=shift)
        o = F.scaled_dot_product_attention(q[b:b + 1], ks, vs, attn_mask=mask, enable_gqa=True)
        out[b] = torch.nan_to_num(o, nan=0.0)[0]
    return out


def check_paged(q, k, v, bt, sl, causal=True, align="bottom_right", **kw):
    ours = attention_kvcache(q, k, v, bt, sl, causal=causal, causal_align=align, **kw)
    ref = naive_attention_paged(q, k, v, bt, sl, causal=causal, dtype=torch.float64, causal_align=align)
    theirs = sdpa_paged(q, k, v, bt, sl, causal, align)
    torch.cuda.synchronize()
    e_ours = (ours.double() - ref).abs().max().item()
    e_sdpa = (theirs.double() - ref).abs().max().item()
    assert torch.isfinite(ours).all()
    assert e_ours <= 2 * e_sdpa + ATOL_FLOOR, f"max-abs {e_ours:.3e} vs torch {e_sdpa:.3e}"
    return ours


@pytest.mark.parametrize("page_size", [16, 64, 128, 256])
@pytest.mark.parametrize("N_q", [1, 7, 130])
@pytest.mark.parametrize("causal", [True, False])
def test_paged_parity(page_size, N_q, causal):
    seqlens = [1000, 4097, 300, 2048]
    seqlens = [max(n, N_q) for n in seqlens]  # bottom-right: every query sees at least one key
    check_paged(*paged_inputs(4, 32, 8, N_q, seqlens, page_size, 128, torch.bfloat16, seed=page_size + N_q),
                causal=causal)


@pytest.mark.parametrize("num_splits", [1, 3, 8])
def test_paged_split_kv_fp16_d64(num_splits):
    q, k, v, bt, sl = paged_inputs(3, 16, 2, 4, [5000, 129, 8192], 32, 64, torch.float16, seed=2)
    check_paged(q, k, v, bt, sl, causal=True, num_splits=num_splits)


@pytest.mark.parametrize("D", [16, 32])
def test_paged_small_head_dims(D):
    """head_dim 16 / 32 pages read in place by the D = 64 build (zero-filled box columns)."""
    q, k, v, bt, sl = paged_inputs(3, 8, 2, 5, [3000, 77, 1024], 64, D, torch.bfloat16, seed=7)
    check_paged(q, k, v, bt, sl, causal=True, num_splits=1)
    check_paged(q, k, v, bt, sl, causal=True, num_splits=4)


def test_paged_unequal_lengths_top_left_and_empty():
    """Per-sequence top-left masks, a sequence without keys (zeros), a one-key sequence."""
    q, k, v, bt, sl = paged_inputs(4, 8, 8, 64, [0, 1, 700, 64], 64, 128, torch.bfloat16, seed=3)
    check_paged(q, k, v, bt, sl, causal=True, align="top_left", num_splits=1)
    check_paged(q, k, v, bt, sl, causal=False)


@pytest.mark.parametrize("num_splits", [1, 4])
def test_paged_matches_contiguous_bit_for_bit(num_splits):
    """Pages of 128 keys laid out in order hold exactly the contiguous K/V: the paged launch and the
    fixed-length launch with the same split count compute the same tiles in the same order."""
    B, Hq, Hkv, N_q, N_kv, D = 2, 16, 4, 5, 1024, 128
    q, k, v, bt, sl = paged_inputs(B, Hq, Hkv, N_q, [N_kv] * B, 128, D, torch.bfloat16, seed=4, shuffle=False)
    paged = attention_kvcache(q, k, v, bt, sl, causal=True, num_splits=num_splits)
    pages = N_kv // 128
    kc = k[: B * pages].reshape(B, N_kv, Hkv, D).transpose(1, 2)
    vc = v[: B * pages].reshape(B, N_kv, Hkv, D).transpose(1, 2)
    contiguous = attention(q, kc, vc, causal=True, causal_align="bottom_right", num_splits=num_splits)
    assert torch.equal(paged, contiguous)


def test_paged_decode_long_cache():
    """One new token per sequence against long caches (the decode case split-KV is for)."""
    q, k, v, bt, sl = paged_inputs(4, 32, 8, 1, [65536, 30000, 17, 8192], 256, 128, torch.bfloat16, seed=5)
    check_paged(q, k, v, bt, sl, causal=True)


def test_paged_longer_than_declared_is_reported():
    q, k, v, bt, sl = paged_inputs(2, 4, 4, 1, [300, 200], 64, 64, torch.float16, seed=6)
    attention_kvcache(q, k, v, bt, sl, max_seqlen_k=256, causal=True, num_splits=1)
    with pytest.raises(RuntimeError, match=f"status {_lib.FA2_ERR_SHAPE}"):
        check_device_errors()
