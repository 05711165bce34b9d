"""CPU tests of the oracle, pinned to the reference.

1. The tiled mirror matches the full-matrix formula (the reference's own algorithm test,
   tests/test_correctness.py:51-66 of roy6n23/triton-fa2-forward, same grid).
2. The oracle reproduces the golden fixtures that tests/golden/make_golden.py produced by
   running the reference's fa2.reference.naive_attention / blocked_attention.
3. The reference's own Triton kernel output stored in the fixtures meets the reference's
   acceptance rule against that ground truth (it is the bar our kernel is held to).
4. The extensions' oracles (bottom-right mask, variable-length batches, paged K/V cache) against
   independent masked-softmax formulations in fp64.
"""

import glob
import os

import pytest
import torch
import torch.nn.functional as F

from oracle.reference import (attn_flops, blocked_attention, make_qkv, naive_attention, naive_attention_paged,
                              naive_attention_varlen)

GOLDEN = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "*.pt")))
ATOL_FLOOR = 1e-4  # reference tests/test_correctness.py:31


def load(path):
    return torch.load(path, weights_only=False)


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("H_q,H_kv", [(4, 4), (4, 2), (4, 1)])
@pytest.mark.parametrize("N", [1, 16, 37, 100])
def test_blocked_matches_naive(causal, H_q, H_kv, N):
    q, k, v = make_qkv(2, H_q, H_kv, N, N, 32, torch.float64)
    ref = naive_attention(q, k, v, causal=causal)
    out = blocked_attention(q, k, v, causal=causal, block_m=32, block_n=16)
    torch.testing.assert_close(out, ref, atol=1e-5, rtol=1e-5)


def test_blocked_noncausal_different_lengths():
    q, k, v = make_qkv(1, 4, 2, 23, 70, 32, torch.float64)
    torch.testing.assert_close(blocked_attention(q, k, v, causal=False),
                               naive_attention(q, k, v, causal=False), atol=1e-5, rtol=1e-5)


def test_golden_fixtures_present():
    names = {os.path.basename(p) for p in GOLDEN}
    assert "plumbing_fp16_causal_d64.pt" in names
    assert len(GOLDEN) >= 6


@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(p)[:-3] for p in GOLDEN])
def test_oracle_reproduces_reference_naive(path):
    g = load(path)
    ours = naive_attention(g["q"].double(), g["k"].double(), g["v"].double(), causal=g["causal"])
    # fixtures store the fp64 reference result rounded to fp32
    torch.testing.assert_close(ours.float(), g["ref_naive"], atol=2e-6, rtol=2e-6)


@pytest.mark.parametrize("path", [p for p in GOLDEN if "ref_blocked" in load(p)],
                         ids=lambda p: os.path.basename(p)[:-3])
def test_oracle_reproduces_reference_blocked(path):
    g = load(path)
    ours = blocked_attention(g["q"].double(), g["k"].double(), g["v"].double(), causal=g["causal"])
    torch.testing.assert_close(ours.float(), g["ref_blocked"], atol=2e-6, rtol=2e-6)


@pytest.mark.parametrize("path", [p for p in GOLDEN if "ref_triton" in load(p)],
                         ids=lambda p: os.path.basename(p)[:-3])
def test_reference_kernel_meets_its_bar(path):
    g = load(path)
    q, k, v, causal = g["q"], g["k"], g["v"], g["causal"]
    ref = g["ref_naive"].double()
    sdpa = F.scaled_dot_product_attention(q.float(), k.float().repeat_interleave(q.shape[1] // k.shape[1], 1),
                                          v.float().repeat_interleave(q.shape[1] // k.shape[1], 1),
                                          is_causal=causal).to(q.dtype)
    e_ref_kernel = (g["ref_triton"].double() - ref).abs().max().item()
    e_sdpa = (sdpa.double() - ref).abs().max().item()
    assert e_ref_kernel <= 2 * e_sdpa + ATOL_FLOOR


def test_flops_formula():
    # bench/bench.py:83-87 of the reference: 4 * B * H * pairs * D, pairs = N(N+1)/2 causal
    assert attn_flops(2, 32, 8192, 8192, 128, True) == pytest.approx(1.0996e12, rel=1e-4)
    assert attn_flops(2, 32, 16384, 16384, 64, False) == pytest.approx(4.398e12, rel=1e-4)
    assert attn_flops(1, 2, 256, 256, 64, True) == pytest.approx(1.684e7, rel=1e-3)


def test_make_qkv_spikes():
    _, k, _ = make_qkv(1, 2, 1, 200, 200, 128, torch.float32, spike_frac=0.01)
    n = int((k.abs() == 8.0).sum())
    assert n == int(k.numel() * 0.01)


@pytest.mark.parametrize("N_q,N_kv", [(1, 9), (5, 13), (13, 13)])
def test_naive_bottom_right_mask(N_q, N_kv):
    """The bottom-right extension: query i sees keys j <= i + N_kv - N_q (checked against an
    explicit softmax over the visible keys of each row); equal to top-left when N_q == N_kv."""
    q, k, v = make_qkv(1, 4, 2, N_q, N_kv, 16, torch.float64, seed=3)
    out = naive_attention(q, k, v, causal=True, causal_align="bottom_right")
    ke, ve = k.repeat_interleave(2, dim=1), v.repeat_interleave(2, dim=1)
    for i in range(N_q):
        vis = i + N_kv - N_q + 1
        s = (q[:, :, i:i + 1] @ ke[:, :, :vis].transpose(-1, -2)) / 4.0
        want = torch.softmax(s, dim=-1) @ ve[:, :, :vis]
        torch.testing.assert_close(out[:, :, i:i + 1], want, rtol=1e-12, atol=1e-12)
    if N_q == N_kv:
        assert torch.equal(out, naive_attention(q, k, v, causal=True))


def _masked_sdpa64(q, k, v, align):
    """Independent fp64 reference for one sequence ([1, H, n, D]): explicit boolean mask, rows with
    no visible key set to zero."""
    nq, nk = q.shape[2], k.shape[2]
    shift = nk - nq if align == "bottom_right" else 0
    mask = torch.ones(nq, nk, dtype=torch.bool).tril(diagonal=shift)
    h = q.shape[1] // k.shape[1]
    ke, ve = k.repeat_interleave(h, dim=1), v.repeat_interleave(h, dim=1)
    s = (q @ ke.transpose(-1, -2)) / q.shape[-1] ** 0.5
    s = s.masked_fill(~mask, float("-inf"))
    p = torch.softmax(s, dim=-1).nan_to_num(0.0)
    return p @ ve


@pytest.mark.parametrize("align", ["top_left", "bottom_right"])
def test_naive_varlen_matches_per_sequence_masked_softmax(align):
    """The variable-length oracle (an extension) against an explicit per-sequence masked softmax,
    with a sequence without queries, one without keys and bottom-right rows before the first key."""
    lens_q, lens_k = [7, 0, 12, 5, 9], [10, 4, 12, 0, 3]
    g = torch.Generator().manual_seed(11)
    q = torch.randn(sum(lens_q), 4, 16, generator=g, dtype=torch.float64)
    k = torch.randn(sum(lens_k), 2, 16, generator=g, dtype=torch.float64)
    v = torch.randn(sum(lens_k), 2, 16, generator=g, dtype=torch.float64)
    cq = torch.tensor([0] + list(torch.tensor(lens_q).cumsum(0)), dtype=torch.int32)
    ck = torch.tensor([0] + list(torch.tensor(lens_k).cumsum(0)), dtype=torch.int32)
    out = naive_attention_varlen(q, k, v, cq, ck, causal=True, causal_align=align)
    for b in range(len(lens_q)):
        qs = q[cq[b]:cq[b + 1]].transpose(0, 1).unsqueeze(0)
        rows = out[cq[b]:cq[b + 1]]
        if lens_q[b] == 0:
            continue
        if lens_k[b] == 0:
            assert torch.equal(rows, torch.zeros_like(rows))
            continue
        ks = k[ck[b]:ck[b + 1]].transpose(0, 1).unsqueeze(0)
        vs = v[ck[b]:ck[b + 1]].transpose(0, 1).unsqueeze(0)
        want = _masked_sdpa64(qs, ks, vs, align)[0].transpose(0, 1)
        torch.testing.assert_close(rows, want, rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("page_size", [4, 16])
def test_naive_paged_matches_contiguous_cache(page_size):
    """The paged-cache oracle (an extension) gathers each sequence's keys through a shuffled block
    table: equal to the masked softmax over the contiguous keys; unused table entries (out of
    range on purpose) are never read; a sequence without keys gives zeros."""
    B, H, Hkv, N_q, D = 3, 4, 2, 3, 16
    lens = [10, 0, 7]
    g = torch.Generator().manual_seed(12)
    q = torch.randn(B, H, N_q, D, generator=g, dtype=torch.float64)
    kc = [torch.randn(1, Hkv, max(n, 1), D, generator=g, dtype=torch.float64) for n in lens]
    vc = [torch.randn(1, Hkv, max(n, 1), D, generator=g, dtype=torch.float64) for n in lens]
    per = -(-max(lens) // page_size)
    num_pages = B * per + 2
    k_cache = torch.randn(num_pages, page_size, Hkv, D, generator=g, dtype=torch.float64)
    v_cache = torch.randn(num_pages, page_size, Hkv, D, generator=g, dtype=torch.float64)
    order = torch.randperm(num_pages, generator=g).tolist()
    bt = torch.full((B, per), num_pages + 100, dtype=torch.int32)
    used = 0
    for b, n in enumerate(lens):
        for j in range(-(-n // page_size)):
            pg = order[used]
            used += 1
            bt[b, j] = pg
            rows = min(page_size, n - j * page_size)
            k_cache[pg, :rows] = kc[b][0, :, j * page_size:j * page_size + rows].transpose(0, 1)
            v_cache[pg, :rows] = vc[b][0, :, j * page_size:j * page_size + rows].transpose(0, 1)
    out = naive_attention_paged(q, k_cache, v_cache, bt, torch.tensor(lens, dtype=torch.int32), causal=True)
    for b, n in enumerate(lens):
        if n == 0:
            assert torch.equal(out[b], torch.zeros_like(out[b]))
            continue
        want = _masked_sdpa64(q[b:b + 1], kc[b][:, :, :n], vc[b][:, :, :n], "bottom_right")
        torch.testing.assert_close(out[b:b + 1], want, rtol=1e-12, atol=1e-12)
