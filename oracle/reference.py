"""Oracle for the FA2 forward -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs may import this
module, and only as the checker / the timed CPU baseline. The product path
(fa2.kernel.attention) never calls it; it has no CPU fallback.

Restates the reference's own pure-torch references (roy6n23/triton-fa2-forward,
fa2/reference.py):

  naive_attention    fa2/reference.py:22-32  softmax(QK^T * scale [+ tril mask]) V with the
                     full score matrix, computed in the input dtype (the tests pass fp64).
                     GQA by repeating each KV head for its query heads
                     (fa2/reference.py:16-19). Here it is evaluated one (batch, kv-head
                     group) unit at a time so the [N, N] scores of the headline shape
                     (N = 8192) fit in memory; the arithmetic per element is unchanged.
  blocked_attention  fa2/reference.py:35-82  the kernel's tiled online-softmax recurrence
                     (fa2/kernel.py:60-107) with fp32 state and Python loops: stage 1
                     unmasked tiles [0, start_m), stage 2 the diagonal band, nothing to
                     the right. Small shapes only.

Pinned against fixtures produced by importing the reference itself
(tests/golden/make_golden.py); see tests/test_oracle.py.
"""

import math

import torch

LOG2E = 1.4426950408889634


def _expand_kv(k, v, h_q):
    """GQA -> MHA: repeat each KV head for the query heads that share it (fa2/reference.py:16-19)."""
    group = h_q // k.shape[1]
    return k.repeat_interleave(group, dim=1), v.repeat_interleave(group, dim=1)


def naive_attention(q, k, v, causal=True, sm_scale=None, dtype=None, causal_align="top_left"):
    """softmax(Q K^T * sm_scale [+ causal]) V (fa2/reference.py:22-32), per (b, kv-head) unit.

    dtype: compute dtype (default: q's dtype, as the reference). Returns that dtype.
    causal_align: "top_left" is the reference's mask (tril of the [N_q, N_kv] scores).
    "bottom_right" is an extension the reference does not have (its README lists it out of
    scope): query i sees keys j <= i + (N_kv - N_q), i.e. tril shifted by N_kv - N_q, the mask
    FlashAttention uses for N_q != N_kv. Identical to top-left when N_q == N_kv.
    """
    dtype = dtype or q.dtype
    B, H_q, N_q, D = q.shape
    H_kv = k.shape[1]
    group = H_q // H_kv
    sm_scale = sm_scale if sm_scale is not None else 1.0 / math.sqrt(D)
    out = torch.empty(B, H_q, N_q, D, dtype=dtype, device=q.device)
    mask = None
    for b in range(B):
        for h in range(H_kv):
            qs = q[b, h * group:(h + 1) * group].to(dtype)          # [G, N_q, D]
            ks = k[b, h].to(dtype)                                 # [N_kv, D]
            vs = v[b, h].to(dtype)
            s = (qs @ ks.transpose(-1, -2)) * sm_scale             # [G, N_q, N_kv]
            if causal:
                if mask is None:
                    n_q, n_kv = s.shape[-2:]
                    shift = n_kv - n_q if causal_align == "bottom_right" else 0
                    mask = torch.ones(n_q, n_kv, dtype=torch.bool, device=q.device).tril(diagonal=shift)
                s = s.masked_fill(~mask, float("-inf"))
            out[b, h * group:(h + 1) * group] = torch.softmax(s, dim=-1) @ vs
    return out


def naive_attention_varlen(q, k, v, cu_seqlens_q, cu_seqlens_k, causal=True, sm_scale=None, dtype=None,
                           causal_align="top_left"):
    """Variable-length batch (an extension; the reference has no such mode): sequences packed
    along one token axis, q [total_q, H_q, D], k/v [total_k, H_kv, D], sequence b owning rows
    cu_seqlens[b]:cu_seqlens[b + 1]. Each sequence is naive_attention on its own ([1, H, n, D]),
    with the causal mask per sequence; a query that sees no key (no keys, or bottom-right rows
    before the first key) is defined as zeros, as the kernel writes them."""
    dtype = dtype or q.dtype
    out = torch.zeros(q.shape, dtype=dtype, device=q.device)
    cq = [int(x) for x in cu_seqlens_q.tolist()]
    ck = [int(x) for x in cu_seqlens_k.tolist()]
    for b in range(len(cq) - 1):
        nq, nk = cq[b + 1] - cq[b], ck[b + 1] - ck[b]
        if nq == 0 or nk == 0:
            continue
        qs = q[cq[b]:cq[b + 1]].transpose(0, 1).unsqueeze(0)   # [1, H_q, nq, D]
        ks = k[ck[b]:ck[b + 1]].transpose(0, 1).unsqueeze(0)
        vs = v[ck[b]:ck[b + 1]].transpose(0, 1).unsqueeze(0)
        o = naive_attention(qs, ks, vs, causal=causal, sm_scale=sm_scale, dtype=dtype, causal_align=causal_align)
        o = torch.nan_to_num(o, nan=0.0)                        # rows with no visible key
        out[cq[b]:cq[b + 1]] = o[0].transpose(0, 1)
    return out


def naive_attention_paged(q, k_cache, v_cache, block_table, cache_seqlens, causal=True, sm_scale=None,
                          dtype=None, causal_align="bottom_right"):
    """Paged K/V cache (an extension; the reference has no such mode): q [B, H_q, N_q, D] against
    k/v caches [num_pages, page_size, H_kv, D], sequence b's key j in page block_table[b, j //
    page_size], row j % page_size, cache_seqlens[b] keys. Each sequence's keys are gathered and
    naive_attention runs on that sequence alone; a query that sees no key is zeros."""
    dtype = dtype or q.dtype
    B, H_q, N_q, D = q.shape
    page_size = k_cache.shape[1]
    out = torch.zeros(q.shape, dtype=dtype, device=q.device)
    bt, sl = block_table.tolist(), [int(x) for x in cache_seqlens.tolist()]
    for b in range(B):
        n = sl[b]
        if n == 0:
            continue
        pages = bt[b][:-(-n // page_size)]
        ks = k_cache[pages].reshape(-1, *k_cache.shape[2:])[:n].transpose(0, 1).unsqueeze(0)  # [1, H_kv, n, D]
        vs = v_cache[pages].reshape(-1, *v_cache.shape[2:])[:n].transpose(0, 1).unsqueeze(0)
        o = naive_attention(q[b:b + 1], ks, vs, causal=causal, sm_scale=sm_scale, dtype=dtype, causal_align=causal_align)
        out[b] = torch.nan_to_num(o, nan=0.0)[0]
    return out


def _tile_walk(n_kv, row_lo, row_hi, causal, block_n):
    """K/V column ranges a Q tile of rows [row_lo, row_hi) visits, with a mask flag:
    stage 1 = whole block_n tiles left of row_lo (no mask), stage 2 = the diagonal band up
    to min(row_hi, n_kv) (masked); nothing to the right (fa2/kernel.py:150-175)."""
    if not causal:
        return [(c, min(c + block_n, n_kv), False) for c in range(0, n_kv, block_n)]
    walk = [(c, min(c + block_n, n_kv), False) for c in range(0, row_lo, block_n)]
    band_end = min(row_hi, n_kv)
    walk += [(c, min(c + block_n, band_end), True) for c in range(row_lo, band_end, block_n)]
    return walk


def blocked_attention(q, k, v, causal=True, sm_scale=None, block_m=32, block_n=16):
    """Tiled online softmax in fp32 state, as the kernel computes it (fa2/kernel.py:60-183,
    mirrored by fa2/reference.py:35-82): per Q tile, running max m, running sum l and the
    unnormalised accumulator, rescaled by exp2(m_old - m_new) at every K/V tile; base-2
    exponentials with log2(e) folded into the scale; one normalisation at the end."""
    B, H_q, N_q, D = q.shape
    H_kv, N_kv = k.shape[1], k.shape[2]
    group = H_q // H_kv
    sm_scale = sm_scale if sm_scale is not None else 1.0 / math.sqrt(D)
    c = sm_scale * LOG2E
    out = torch.empty_like(q)
    for b in range(B):
        for hq in range(H_q):
            keys = k[b, hq // group].float()
            vals = v[b, hq // group].float()
            for lo in range(0, N_q, block_m):
                hi = min(lo + block_m, N_q)
                rows = torch.arange(lo, hi, device=q.device)
                qt = q[b, hq, lo:hi].float()
                run_max = torch.full((hi - lo,), float("-inf"), device=q.device)
                run_sum = torch.zeros(hi - lo, device=q.device)
                acc = torch.zeros(hi - lo, D, device=q.device)
                for c0, c1, use_mask in _tile_walk(N_kv, lo, lo + block_m, causal, block_n):
                    scores = (qt @ keys[c0:c1].T) * c
                    if use_mask:
                        cols = torch.arange(c0, c1, device=q.device)
                        scores = torch.where(rows[:, None] >= cols[None, :], scores,
                                             torch.full_like(scores, float("-inf")))
                    new_max = torch.maximum(run_max, scores.amax(dim=1))
                    probs = torch.exp2(scores - new_max[:, None])
                    corr = torch.exp2(run_max - new_max)
                    run_sum = run_sum * corr + probs.sum(dim=1)
                    acc = acc * corr[:, None] + probs @ vals[c0:c1]
                    run_max = new_max
                out[b, hq, lo:hi] = (acc / run_sum[:, None]).to(q.dtype)
    return out


def attn_flops(B, H_q, N_q, N_kv, D, causal):
    """Causal-adjusted FLOPs of the forward, the reference's own count (bench/bench.py:83-87)."""
    pairs = N_q * (N_q + 1) / 2 if causal else N_q * N_kv
    return 4 * B * H_q * pairs * D


def make_qkv(B, H_q, H_kv, N_q, N_kv, D, dtype, seed=0, scale=1.0, spike_frac=0.0, device="cpu"):
    """Seeded N(0,1) inputs generated on the CPU (so every box sees the same values), then
    moved to `device`. `scale` multiplies all three; `spike_frac` sets that fraction of k's
    entries to +-8 (chosen by a second seeded generator) to stress the running max."""
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H_q, N_q, D, generator=g, dtype=torch.float32)
    k = torch.randn(B, H_kv, N_kv, D, generator=g, dtype=torch.float32)
    v = torch.randn(B, H_kv, N_kv, D, generator=g, dtype=torch.float32)
    if scale != 1.0:
        q, k, v = q * scale, k * scale, v * scale
    if spike_frac > 0:
        g2 = torch.Generator().manual_seed(seed + 1)
        n = k.numel()
        idx = torch.randperm(n, generator=g2)[: int(n * spike_frac)]
        sign = torch.randint(0, 2, (idx.numel(),), generator=g2).float() * 2 - 1
        k.view(-1)[idx] = 8.0 * sign
    return tuple(t.to(dtype).to(device) for t in (q, k, v))
