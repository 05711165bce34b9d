"""FlashAttention-2 forward on Blackwell (sm_100a): the drop-in for the reference's
`fa2.kernel` module (roy6n23/triton-fa2-forward, fa2/kernel.py).

Same public surface as the reference:
    attention(q, k, v, causal=True, sm_scale=None, block_m=None, block_n=None,
              num_warps=None, num_stages=None, pack_gqa=None)        fa2/kernel.py:210-260
    should_pack_gqa(n_q, group, block_m)                             fa2/kernel.py:202-207
    _default_config(head_dim, on_cuda)                               fa2/kernel.py:186-195

q: [B, H_q, N_q, D]; k, v: [B, H_kv, N_kv, D] (any strides); H_q % H_kv == 0; fp16/bf16;
returns out = softmax(q k^T * sm_scale [+ causal mask]) v with q's strides.
The computation is the hand-written sm_100a CUDA kernel in csrc/fa2_fwd_sm100.cu, reached
through the C ABI of include/fa2_sm100.h. There is no Triton and no CPU path: tensors not
on an sm_100 CUDA device raise RuntimeError.

Differences from the reference that do not change results:
  * The compiled tile is 128 x 128 (two 128-row Q tiles per CTA). block_m / block_n /
    num_warps / num_stages are accepted as hints: block_m feeds the GQA-packing decision and
    its ValueError exactly as in the reference; the others do not change the kernel.
  * Packed and unpacked runs are bit-identical (same tiles, same order, per-row decisions),
    so a group that divides the hinted block_m but not 128 simply runs unpacked.
  * head_dim 16 and 32 run on the 64 kernel in place: its tensor maps are head_dim wide, so
    TMA fills the rest of each 64-column box with zeros (adding nothing to QK^T) and clips the
    stores of the zero output columns. No copies, no extra HBM traffic.

Also (no counterpart in the reference, whose README lists variable-length batches and paged K/V
out of scope):
    attention_varlen(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, causal=True, ...)
with q [total_q, H_q, D], k/v [total_k, H_kv, D] packed along one token axis, and
    attention_kvcache(q, k_cache, v_cache, block_table, cache_seqlens, causal=True, ...)
with q [B, H_q, N_q, D] against a paged K/V cache [num_pages, page_size, H_kv, D].

Extensions (keyword arguments the reference does not have; their defaults keep its behaviour):
  * causal_align="bottom_right": the causal mask lines the last query up with the last key
    (query i sees keys j <= i + N_kv - N_q), for chunked prefill and decode with N_q <= N_kv.
    The default "top_left" is the reference's mask and keeps its N_q == N_kv assertion.
  * num_splits: split-KV for short queries against long K/V (auto_num_splits by default).
  * FA2_SYNC_CHECK=1 in the environment: every call synchronises and raises RuntimeError if
    the kernel reported a timed-out wait (a debugging aid; calls are asynchronous otherwise).
"""

import math
import os

import torch

from . import _lib

LOG2E = 1.4426950408889634
KERNEL_BLOCK_M = 128
KERNEL_BLOCK_N = 128
CTA_ROWS = 256          # two 128-row Q tiles per CTA
NUM_SMS_B200 = 148
MAX_SPLITS = 16

_err_words = {}
CAUSAL_ALIGNS = {"top_left": _lib.FA2_CAUSAL_TOP_LEFT, "bottom_right": _lib.FA2_CAUSAL_BOTTOM_RIGHT}


def _sync_check_enabled():
    return os.environ.get("FA2_SYNC_CHECK", "0") not in ("", "0")


def _default_config(head_dim, on_cuda):
    """(BLOCK_M, BLOCK_N, num_warps, num_stages) of the compiled sm_100a kernel for head_dim.

    Mirrors fa2/kernel.py:186-195. `on_cuda` is accepted for signature compatibility; there
    is only one (CUDA) implementation, so it does not change the answer.
    """
    del on_cuda
    d = 64 if head_dim <= 64 else 128
    bm, bn, threads, stages, _ = _lib.config(d)
    return bm, bn, threads // 32, stages


def _tile_efficiency(rows, block_m):
    return rows / (-(-rows // block_m) * block_m)


def should_pack_gqa(n_q, group, block_m):
    """FlashAttention-3's rule, as in fa2/kernel.py:202-207: pack when the unpacked tiles are
    less than 90% as full as the packed ones; packing needs block_m % group == 0."""
    if group == 1 or block_m % group:
        return False
    return _tile_efficiency(n_q, block_m) < 0.9 * _tile_efficiency(n_q * group, block_m)


def _err_word(device):
    """Per-device int32 that the kernel ORs FA2_ERR_TIMEOUT into when a bounded wait expires."""
    key = device.index
    w = _err_words.get(key)
    if w is None:
        w = torch.zeros(1, dtype=torch.int32, device=device)
        _err_words[key] = w
    return w


def check_device_errors(device=None):
    """Synchronise `device` and raise RuntimeError if a kernel reported a timed-out wait
    since the last check (the word is cleared). Launches never synchronise on their own."""
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    w = _err_words.get(device.index)
    if w is None:
        return
    val = int(w.item())
    if val:
        w.zero_()
        raise RuntimeError(f"fa2 sm100 kernel reported status {val}: {_lib.strerror(val)}")


def _strides(t):
    return tuple(int(s) for s in t.stride())


def auto_num_splits(batch, heads_q, n_q, n_kv, group, pack, causal, num_sms=NUM_SMS_B200,
                    causal_align="top_left"):
    """Split-KV count for a launch (an extension; the reference has no split-KV). Splitting
    pays when the (batch, head block, 256-row block) CTAs cannot fill the GPU and each has a
    long K/V range, i.e. short queries against long K/V. One CTA fits per SM, so the split
    CTAs are kept within one wave (measured: a second partial wave costs more than the split
    gains), with at least 4 K/V tiles per split. Top-left causal attention has N_q == N_kv and
    is not split; bottom-right causal with N_q < N_kv is split like the unmasked case (every
    query sees nearly all of the K/V)."""
    if causal and (causal_align != "bottom_right" or n_q >= n_kv):
        return 1
    P = pack if pack else 1
    ctas = batch * (heads_q // P) * (-(-(n_q * P) // CTA_ROWS))
    tiles = -(-n_kv // KERNEL_BLOCK_N)
    if tiles < 8:
        return 1
    if n_q * P <= KERNEL_BLOCK_M:
        # All rows fit the first Q tile: splits run in pairs inside one CTA (the second Q-tile
        # slot streams the other split of the same rows), so 2 splits add no CTAs.
        z = max(1, min(MAX_SPLITS // 2, num_sms // ctas, tiles // 8))
        return 2 * z
    if 2 * ctas > num_sms:
        return 1
    return max(1, min(MAX_SPLITS, num_sms // ctas, tiles // 4))


def _launch(q, k, v, out, causal, pack, qk_scale, num_splits=1, timeout_cycles=0, align=0):
    B, H_q, N_q, D = q.shape
    H_kv, N_kv = k.shape[1], k.shape[2]
    err = _err_word(q.device)
    p = _lib.make_params(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
        _strides(q), _strides(k), _strides(v), _strides(out),
        B, H_q, H_kv, N_q, N_kv, D,
        _lib.FA2_DTYPE_BF16 if q.dtype == torch.bfloat16 else _lib.FA2_DTYPE_FP16,
        causal, pack, qk_scale, err.data_ptr(), timeout_cycles, num_splits=num_splits,
        causal_align=align,
    )
    ws = None
    if num_splits > 1:
        nbytes = _lib.workspace_bytes(p)
        ws = torch.empty(nbytes, dtype=torch.uint8, device=q.device)  # caching allocator
        p.workspace, p.workspace_bytes = ws.data_ptr(), nbytes
    stream = torch.cuda.current_stream(q.device).cuda_stream
    rc = _lib.launch(p, stream)
    if ws is not None:
        ws.record_stream(torch.cuda.current_stream(q.device))
    return rc


def _run(q, k, v, out, causal, pack, qk_scale, num_splits=1, align=0):
    with torch.cuda.device(q.device):
        rc = _launch(q, k, v, out, causal, pack, qk_scale, num_splits, align=align)
        if rc == _lib.FA2_ERR_TMA_ENCODE and pack:
            pack = False  # bit-identical result; some stride orders only encode unpacked
            rc = _launch(q, k, v, out, causal, pack, qk_scale, num_splits, align=align)
        if rc in (_lib.FA2_ERR_LAYOUT, _lib.FA2_ERR_TMA_ENCODE):
            # Layout copy (not a compute fallback): TMA needs 16-byte strides/alignment.
            qc, kc, vc = q.contiguous(), k.contiguous(), v.contiguous()
            oc = torch.empty_like(qc)
            rc = _launch(qc, kc, vc, oc, causal, pack, qk_scale, num_splits, align=align)
            if rc == _lib.FA2_OK:
                out.copy_(oc)
        if rc != _lib.FA2_OK:
            raise _lib.Fa2Error(rc, _lib.strerror(rc))
        if _sync_check_enabled():
            check_device_errors(q.device)
    return out


def attention(q, k, v, causal=True, sm_scale=None, block_m=None, block_n=None,
              num_warps=None, num_stages=None, pack_gqa=None, num_splits=None,
              causal_align="top_left"):
    """softmax(Q K^T * sm_scale [+ causal mask]) V, fused (fa2/kernel.py:210-260).

    q: [B, H_q, N_q, D]; k, v: [B, H_kv, N_kv, D]; returns [B, H_q, N_q, D].
    pack_gqa: put each GQA group's query heads into one tile; None packs whenever the group
    divides the 128-row tile (results are bit-identical either way; see the body). Asynchronous
    on torch's current stream, like the reference.
    num_splits (extension, not in the reference): split-KV count; None picks one with
    auto_num_splits (short queries against long K/V), 1 disables it.
    causal_align (extension): "top_left" (the reference's mask, N_q == N_kv) or
    "bottom_right" (query i sees keys j <= i + N_kv - N_q; needs N_q <= N_kv).
    """
    assert q.dim() == k.dim() == v.dim() == 4
    B, H_q, N_q, D = q.shape
    Bk, H_kv, N_kv, Dk = k.shape
    assert v.shape == k.shape and Bk == B and Dk == D
    assert q.dtype == k.dtype == v.dtype and q.dtype in (torch.float16, torch.bfloat16)
    assert H_q % H_kv == 0, "GQA needs H_q divisible by H_kv"
    assert D in (16, 32, 64, 128), "head_dim must be a power of two in [16, 128]"
    assert causal_align in CAUSAL_ALIGNS, f"causal_align must be one of {sorted(CAUSAL_ALIGNS)}"
    if causal and causal_align == "top_left":
        # Top-left aligned causal mask (prefill), as in the reference.
        assert N_q == N_kv, "causal attention here assumes N_q == N_kv"
    if causal and causal_align == "bottom_right":
        assert N_q <= N_kv, "bottom-right causal attention needs N_q <= N_kv"

    bm, bn, nw, ns = _default_config(D, q.is_cuda)
    bm, bn = block_m or bm, block_n or bn
    nw, ns = num_warps or nw, num_stages or ns
    group = H_q // H_kv
    if pack_gqa is None:
        # The reference decides with should_pack_gqa(N_q, group, bm). Here packed and unpacked
        # runs are bit-identical, and packing is never slower on this kernel (one K/V tile load
        # serves `group` heads): measured +14% on B=16 Hq=64 Hkv=8 N=1000, where the
        # reference's rule leaves it off, and +1% at the headline shape. So pack whenever the
        # compiled 128-row tile allows it; should_pack_gqa() itself is unchanged.
        pack_gqa = group > 1 and KERNEL_BLOCK_M % group == 0
    elif pack_gqa and bm % group:
        raise ValueError(f"pack_gqa needs BLOCK_M ({bm}) to be a multiple of the GQA group ({group})")
    pack = bool(pack_gqa) and group > 1 and KERNEL_BLOCK_M % group == 0

    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    if not sm_scale > 0:
        raise ValueError(f"sm_scale must be positive (the row max is scaled after it is taken), got {sm_scale}")
    qk_scale = sm_scale * LOG2E

    if not (q.is_cuda and k.is_cuda and v.is_cuda):
        raise RuntimeError("fa2.kernel.attention runs only on an sm_100 CUDA device (no CPU path)")
    if not (q.device == k.device == v.device):
        raise RuntimeError("q, k and v must be on the same CUDA device")

    if num_splits is None:
        num_splits = auto_num_splits(B, H_q, N_q, N_kv, group, group if pack else 1, causal,
                                     causal_align=causal_align)
    num_splits = max(1, int(num_splits))
    align = CAUSAL_ALIGNS[causal_align]

    out = torch.empty_like(q)
    if out.numel() == 0:
        return out
    return _run(q, k, v, out, causal, pack, qk_scale, num_splits, align=align)


def attention_varlen(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, causal=True,
                     sm_scale=None, pack_gqa=None, causal_align="top_left"):
    """Attention over a batch of sequences of different lengths packed along one token axis
    (the layout of flash_attn_varlen_func). An extension: the reference has no such entry point.

    q: [total_q, H_q, D]; k, v: [total_k, H_kv, D]; cu_seqlens_q / cu_seqlens_k: int32 CUDA
    tensors [B + 1] of prefix sums (sequence b owns q rows cu_seqlens_q[b]:cu_seqlens_q[b+1]);
    max_seqlen_q / max_seqlen_k: upper bounds of the lengths (a longer sequence is reported as a
    device error, see check_device_errors). Each sequence is attended on its own, with the causal
    mask per sequence ("top_left": query i sees keys j <= i; "bottom_right": j <= i + n_k - n_q).
    A query that sees no key gets zeros. Returns [total_q, H_q, D]; asynchronous like attention().
    """
    assert q.dim() == k.dim() == v.dim() == 3
    total_q, H_q, D = q.shape
    total_k, H_kv, Dk = k.shape
    assert v.shape == k.shape and Dk == D
    assert q.dtype == k.dtype == v.dtype and q.dtype in (torch.float16, torch.bfloat16)
    assert H_q % H_kv == 0, "GQA needs H_q divisible by H_kv"
    assert D in (16, 32, 64, 128), "head_dim must be a power of two in [16, 128]"
    assert causal_align in CAUSAL_ALIGNS, f"causal_align must be one of {sorted(CAUSAL_ALIGNS)}"
    assert cu_seqlens_q.dtype == torch.int32 and cu_seqlens_k.dtype == torch.int32
    assert cu_seqlens_q.dim() == 1 and cu_seqlens_q.shape == cu_seqlens_k.shape and cu_seqlens_q.numel() >= 2
    if not (q.is_cuda and k.is_cuda and v.is_cuda and cu_seqlens_q.is_cuda and cu_seqlens_k.is_cuda):
        raise RuntimeError("fa2.kernel.attention_varlen runs only on an sm_100 CUDA device (no CPU path)")
    B = cu_seqlens_q.numel() - 1
    group = H_q // H_kv
    if pack_gqa is None:
        pack_gqa = group > 1 and KERNEL_BLOCK_M % group == 0
    elif pack_gqa and KERNEL_BLOCK_M % group:
        raise ValueError(f"pack_gqa needs BLOCK_M ({KERNEL_BLOCK_M}) to be a multiple of the GQA group ({group})")
    pack = bool(pack_gqa) and group > 1
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    if not sm_scale > 0:
        raise ValueError(f"sm_scale must be positive (the row max is scaled after it is taken), got {sm_scale}")
    out = torch.empty_like(q)
    if total_q == 0 or max_seqlen_q == 0:
        return out
    if total_k == 0 or max_seqlen_k == 0:
        return out.zero_()  # no sequence has a key: every query sees none
    cq, ck = cu_seqlens_q.contiguous(), cu_seqlens_k.contiguous()

    def launch(qq, kk, vv, oo, pk):
        err = _err_word(qq.device)
        st = lambda t: (0, int(t.stride(1)), int(t.stride(0)), int(t.stride(2)))  # noqa: E731
        p = _lib.make_params(
            qq.data_ptr(), kk.data_ptr(), vv.data_ptr(), oo.data_ptr(), st(qq), st(kk), st(vv), st(oo),
            B, H_q, H_kv, int(max_seqlen_q), int(max_seqlen_k), D,
            _lib.FA2_DTYPE_BF16 if qq.dtype == torch.bfloat16 else _lib.FA2_DTYPE_FP16,
            causal, pk, sm_scale * LOG2E, err.data_ptr(), 0, causal_align=CAUSAL_ALIGNS[causal_align],
            cu_seqlens_q=cq.data_ptr(), cu_seqlens_kv=ck.data_ptr(), total_q=total_q, total_kv=total_k)
        return _lib.launch(p, torch.cuda.current_stream(qq.device).cuda_stream)

    with torch.cuda.device(q.device):
        rc = launch(q, k, v, out, pack)
        if rc == _lib.FA2_ERR_TMA_ENCODE and pack:
            pack = False
            rc = launch(q, k, v, out, pack)
        if rc in (_lib.FA2_ERR_LAYOUT, _lib.FA2_ERR_TMA_ENCODE):
            qc, kc, vc = q.contiguous(), k.contiguous(), v.contiguous()
            oc = torch.empty_like(qc)
            rc = launch(qc, kc, vc, oc, pack)
            if rc == _lib.FA2_OK:
                out.copy_(oc)
        if rc != _lib.FA2_OK:
            raise _lib.Fa2Error(rc, _lib.strerror(rc))
        if _sync_check_enabled():
            check_device_errors(q.device)
    return out


def attention_kvcache(q, k_cache, v_cache, block_table, cache_seqlens, max_seqlen_k=None, causal=True,
                      sm_scale=None, pack_gqa=None, causal_align="bottom_right", num_splits=None):
    """Attention of new queries against a paged K/V cache (the layout of flash_attn_with_kvcache).
    An extension: the reference has no such entry point.

    q: [B, H_q, N_q, D]; k_cache, v_cache: [num_pages, page_size, H_kv, D] (page_size 16, 32, 64 or a
    multiple of 128); block_table: int32 CUDA [B, pages_per_seq], sequence b's key j living in page
    block_table[b, j // page_size], row j % page_size; cache_seqlens: int32 CUDA [B], keys per
    sequence. max_seqlen_k bounds them (default: pages_per_seq * page_size; a longer sequence is
    reported as a device error). The causal mask is per sequence, bottom-right by default (the new
    queries are the sequence's last N_q positions). Split-KV as in attention(). Returns
    [B, H_q, N_q, D], asynchronously.
    """
    assert q.dim() == 4 and k_cache.dim() == 4 and v_cache.shape == k_cache.shape
    B, H_q, N_q, D = q.shape
    num_pages, page_size, H_kv, Dk = k_cache.shape
    assert Dk == D and D in (16, 32, 64, 128), "head_dim must be a power of two in [16, 128]"
    assert q.dtype == k_cache.dtype == v_cache.dtype and q.dtype in (torch.float16, torch.bfloat16)
    assert H_q % H_kv == 0, "GQA needs H_q divisible by H_kv"
    assert causal_align in CAUSAL_ALIGNS, f"causal_align must be one of {sorted(CAUSAL_ALIGNS)}"
    assert page_size in (16, 32, 64) or (page_size >= 128 and page_size % 128 == 0), "page_size"
    assert block_table.dtype == torch.int32 and block_table.dim() == 2 and block_table.shape[0] == B
    assert cache_seqlens.dtype == torch.int32 and cache_seqlens.shape == (B,)
    if not (q.is_cuda and k_cache.is_cuda and v_cache.is_cuda and block_table.is_cuda and cache_seqlens.is_cuda):
        raise RuntimeError("fa2.kernel.attention_kvcache runs only on an sm_100 CUDA device (no CPU path)")
    if max_seqlen_k is None:
        max_seqlen_k = block_table.shape[1] * page_size
    group = H_q // H_kv
    if pack_gqa is None:
        pack_gqa = group > 1 and KERNEL_BLOCK_M % group == 0
    elif pack_gqa and KERNEL_BLOCK_M % group:
        raise ValueError(f"pack_gqa needs BLOCK_M ({KERNEL_BLOCK_M}) to be a multiple of the GQA group ({group})")
    pack = bool(pack_gqa) and group > 1
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    if not sm_scale > 0:
        raise ValueError(f"sm_scale must be positive (the row max is scaled after it is taken), got {sm_scale}")
    out = torch.empty_like(q)
    if out.numel() == 0:
        return out
    if max_seqlen_k == 0:
        return out.zero_()
    if num_splits is None:
        num_splits = auto_num_splits(B, H_q, N_q, max_seqlen_k, group, group if pack else 1, causal,
                                     causal_align=causal_align)
    num_splits = max(1, int(num_splits))
    bt, sl = block_table.contiguous(), cache_seqlens.contiguous()
    kst = lambda t: (int(t.stride(0)), int(t.stride(2)), int(t.stride(1)), int(t.stride(3)))  # noqa: E731

    def launch(qq, kk, vv, oo, pk):
        err = _err_word(qq.device)
        p = _lib.make_params(
            qq.data_ptr(), kk.data_ptr(), vv.data_ptr(), oo.data_ptr(), _strides(qq), kst(kk), kst(vv), _strides(oo),
            B, H_q, H_kv, N_q, int(max_seqlen_k), D,
            _lib.FA2_DTYPE_BF16 if qq.dtype == torch.bfloat16 else _lib.FA2_DTYPE_FP16,
            causal, pk, sm_scale * LOG2E, err.data_ptr(), 0, num_splits=num_splits,
            causal_align=CAUSAL_ALIGNS[causal_align], block_table=bt.data_ptr(), seqlens_kv=sl.data_ptr(),
            block_table_stride=bt.shape[1], page_size=page_size, num_pages=num_pages)
        ws = None
        if num_splits > 1:
            nbytes = _lib.workspace_bytes(p)
            ws = torch.empty(nbytes, dtype=torch.uint8, device=qq.device)
            p.workspace, p.workspace_bytes = ws.data_ptr(), nbytes
        rc = _lib.launch(p, torch.cuda.current_stream(qq.device).cuda_stream)
        if ws is not None:
            ws.record_stream(torch.cuda.current_stream(qq.device))
        return rc

    with torch.cuda.device(q.device):
        rc = launch(q, k_cache, v_cache, out, pack)
        if rc == _lib.FA2_ERR_TMA_ENCODE and pack:
            pack = False
            rc = launch(q, k_cache, v_cache, out, pack)
        if rc in (_lib.FA2_ERR_LAYOUT, _lib.FA2_ERR_TMA_ENCODE):
            qc, kc, vc = q.contiguous(), k_cache.contiguous(), v_cache.contiguous()
            oc = torch.empty_like(qc)
            rc = launch(qc, kc, vc, oc, pack)
            if rc == _lib.FA2_OK:
                out.copy_(oc)
        if rc != _lib.FA2_OK:
            raise _lib.Fa2Error(rc, _lib.strerror(rc))
        if _sync_check_enabled():
            check_device_errors(q.device)
    return out
