"""GPU parity tests of the sm_100a kernel, called through fa2.kernel.attention -> C ABI.

Acceptance rule (the reference's, tests/test_correctness.py:90-103 of
roy6n23/triton-fa2-forward): against the fp64 naive oracle,
    max|ours - ref| <= 2 * max|SDPA(same dtype) - ref| + 1e-4     and all(isfinite(ours)).
The grids below port the reference's GPU sweep; on top of it: the five BASELINE configs at
full size, the golden fixtures made by the reference itself, bit-exact properties that hold
at any size (packed == unpacked, shard == slice, V-linearity, determinism, batch
permutation), edge cases (N = 1, ragged tails, non-contiguous, MQA, D = 16/32) and the
bounded-wait failure report.
"""

import ctypes
import glob
import math
import os

import pytest
import torch
import torch.nn.functional as F

from fa2 import _lib
from fa2.kernel import attention, check_device_errors
from fa2.shard import shard_qkv
from oracle.reference import make_qkv, naive_attention

pytestmark = pytest.mark.gpu

ATOL_FLOOR = 1e-4  # reference tests/test_correctness.py:31
GOLDEN = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "*.pt")))


@pytest.fixture(autouse=True)
def _no_device_errors():
    yield
    check_device_errors()


def make_cuda_qkv(B, H_q, H_kv, N_q, N_kv, D, dtype, seed=0, **kw):
    return make_qkv(B, H_q, H_kv, N_q, N_kv, D, dtype, seed=seed, device="cuda", **kw)


def errors(out, ref):
    diff = (out.double() - ref).abs()
    return diff.max().item()


def sdpa(q, k, v, causal, causal_align="top_left", **kw):
    """torch SDPA at the input dtype: the tolerance yardstick of the reference's rule. Its
    is_causal mask is top-left; the bottom-right mask is passed explicitly."""
    if causal and causal_align == "bottom_right":
        n_q, n_kv = q.shape[2], k.shape[2]
        mask = torch.ones(n_q, n_kv, dtype=torch.bool, device=q.device).tril(diagonal=n_kv - n_q)
        return F.scaled_dot_product_attention(q, k, v, attn_mask=mask, enable_gqa=True, **kw)
    return F.scaled_dot_product_attention(q, k, v, is_causal=causal, enable_gqa=True, **kw)


def check_against_oracle(q, k, v, causal, **kw):
    align = kw.get("causal_align", "top_left")
    ref = naive_attention(q, k, v, causal=causal, dtype=torch.float64, causal_align=align)
    ours = attention(q, k, v, causal=causal, **kw)
    theirs = sdpa(q, k, v, causal, align)
    torch.cuda.synchronize()
    e_ours, e_sdpa = errors(ours, ref), errors(theirs, ref)
    assert torch.isfinite(ours).all()
    assert e_ours <= 2 * e_sdpa + ATOL_FLOOR, f"max-abs {e_ours:.3e} vs torch {e_sdpa:.3e}"
    return ours


# ----------------------------------------------------------------- reference GPU sweep
SEQ_LENS = [128, 1000, 2048, 4096]      # 1000: not a multiple of any block size
HEAD_DIMS = [64, 128]
HEADS = [(32, 32), (32, 8), (32, 1)]    # MHA, GQA (Llama-3-8B ratio), MQA


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("H_q,H_kv", HEADS)
@pytest.mark.parametrize("D", HEAD_DIMS)
@pytest.mark.parametrize("N", SEQ_LENS)
def test_kernel_fp16(causal, H_q, H_kv, D, N):
    check_against_oracle(*make_cuda_qkv(2, H_q, H_kv, N, N, D, torch.float16), causal)


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("D", [64, 128])
def test_kernel_bf16(causal, D):
    check_against_oracle(*make_cuda_qkv(2, 4, 2, 100, 100, D, torch.bfloat16), causal)


def test_kernel_noncausal_different_lengths():
    check_against_oracle(*make_cuda_qkv(2, 4, 2, 23, 70, 64, torch.float16), causal=False)


# ------------------------------------------------------- persistent unit walk
# One CTA per SM walks the work units (a 256-row block of one (batch, head block)). These
# shapes give every CTA several units of one K/V tile each, unit counts just above one and
# exactly two waves of 148, and causal units of every length on the same CTA.
@pytest.mark.parametrize("B,H,H_kv,N,causal,D,dtype", [
    (8, 40, 40, 96, False, 64, torch.float16),      # 320 units, J = 1 each
    (8, 40, 40, 96, True, 128, torch.bfloat16),
    (1, 149, 149, 256, True, 128, torch.bfloat16),  # 149 units: one CTA takes two
    (1, 149, 149, 300, False, 64, torch.float16),   # 298 units, ragged last block
    (2, 37, 37, 1000, True, 128, torch.float16),    # 296 units = 2 x 148
    (3, 99, 99, 513, True, 64, torch.bfloat16),     # 891 units, J from 1 to 5
    (3, 45, 9, 700, True, 128, torch.bfloat16),     # GQA group 5 (unpacked), 405 units
    (5, 21, 7, 333, False, 128, torch.float16),     # GQA group 3, 210 units
])
def test_persistent_unit_walk(B, H, H_kv, N, causal, D, dtype):
    check_against_oracle(*make_cuda_qkv(B, H, H_kv, N, N, D, dtype, seed=B + H), causal)


@pytest.mark.parametrize("N_q,N_kv", [(1, 1), (1, 300), (5, 129), (129, 5), (300, 128)])
def test_kernel_noncausal_ragged(N_q, N_kv):
    check_against_oracle(*make_cuda_qkv(2, 8, 2, N_q, N_kv, 128, torch.bfloat16), causal=False)


@pytest.mark.parametrize("N", [1, 2, 127, 129, 255, 257])
def test_kernel_causal_tile_edges(N):
    check_against_oracle(*make_cuda_qkv(1, 4, 4, N, N, 128, torch.float16), causal=True)


def test_kernel_noncontiguous_input():
    """[B, N, H, D] storage viewed as [B, H, N, D], as it comes out of a QKV projection."""
    q, k, v = (t.transpose(1, 2).contiguous().transpose(1, 2)
               for t in make_cuda_qkv(2, 4, 2, 64, 64, 64, torch.float16))
    assert not q.is_contiguous()
    out = check_against_oracle(q, k, v, causal=True)
    assert out.stride() == q.stride()  # empty_like(q) keeps q's strides, like the reference


def test_kernel_unaligned_strides_take_a_layout_copy():
    """Rows of 72 elements (144 bytes) are not TMA-legal; the wrapper copies, results hold."""
    base = make_cuda_qkv(1, 4, 2, 100, 100, 72, torch.float16)
    q, k, v = (t[..., :64] for t in base)
    check_against_oracle(q, k, v, causal=True)


# head_dim 16 and 32 run on the D = 64 build in place: the tensor maps are head_dim wide, TMA
# fills the rest of each 64-column box with zeros and clips the output stores.
@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("D", [16, 32])
def test_kernel_small_head_dims(D, dtype, causal):
    check_against_oracle(*make_cuda_qkv(2, 4, 2, 300, 300, D, dtype), causal=causal)


@pytest.mark.parametrize("D", [16, 32])
def test_small_head_dims_full_tiles_and_packing(D):
    """Long enough that unmasked tiles (the FMA-pipe exp2 pairs) run; packed == unpacked."""
    q, k, v = make_cuda_qkv(2, 32, 8, 1000, 1000, D, torch.bfloat16, seed=1)
    assert torch.equal(attention(q, k, v, pack_gqa=True), attention(q, k, v, pack_gqa=False))
    check_against_oracle(q, k, v, causal=True)
    check_against_oracle(*make_cuda_qkv(1, 8, 8, 2048, 2048, D, torch.float16, seed=2), causal=False)


@pytest.mark.parametrize("D", [16, 32])
@pytest.mark.parametrize("num_splits", [2, 5])
def test_small_head_dims_split_kv(D, num_splits):
    """Split-KV: the fp32 partials keep 64 columns, the merge writes head_dim of them."""
    check_against_oracle(*make_cuda_qkv(2, 16, 4, 3, 5000, D, torch.bfloat16, seed=3), causal=False,
                         num_splits=num_splits)
    check_against_oracle(*make_cuda_qkv(2, 4, 4, 100, 3000, D, torch.float16, seed=4), causal=False,
                         num_splits=num_splits)


@pytest.mark.parametrize("D", [16, 32])
@pytest.mark.parametrize("num_splits", [1, 4])
def test_small_head_dim_writes_only_its_columns(D, num_splits):
    """Through the C ABI, with q/k/v/o as the first D columns of 64-column rows: the output
    columns past D (pre-filled with NaN) are never written, by the clipped TMA stores or by the
    merge kernel, and every column below D is."""
    B, H, N = 2, 8, 333 if num_splits == 1 else 5
    base = [t for t in make_cuda_qkv(B, H, H, N, 2000 if num_splits > 1 else N, 64, torch.bfloat16, seed=5)]
    q, k, v = (t[..., :D] for t in base)
    wide = torch.full_like(base[0], float("nan"))
    out = wide[..., :D]
    p = _lib.make_params(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                         q.stride(), k.stride(), v.stride(), out.stride(),
                         B, H, H, N, k.shape[2], D, _lib.FA2_DTYPE_BF16, 0, 0,
                         1.0 / math.sqrt(D) * 1.4426950408889634, num_splits=num_splits)
    ws = None
    if num_splits > 1:
        nbytes = _lib.workspace_bytes(p)
        ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
        p.workspace, p.workspace_bytes = ws.data_ptr(), nbytes
    assert _lib.launch(p, torch.cuda.current_stream().cuda_stream) == _lib.FA2_OK
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
    assert torch.isnan(wide[..., D:]).all()
    assert torch.equal(out, attention(q.contiguous(), k.contiguous(), v.contiguous(), causal=False,
                                      num_splits=num_splits))


# ------------------------------------------------------------------- GQA head packing
PACK_HEADS = [(32, 8), (32, 1), (64, 8)]   # group 4, MQA (group 32), group 8
PACK_LENS = [1, 64, 1000, 2048]


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("H_q,H_kv", PACK_HEADS)
@pytest.mark.parametrize("N", PACK_LENS)
def test_kernel_pack_gqa(causal, H_q, H_kv, N):
    """Packed and unpacked runs compute every row with the same tiles in the same order:
    bit-identical outputs, and the packed output meets the bar on its own."""
    q, k, v = make_cuda_qkv(2, H_q, H_kv, N, N, 64, torch.float16)
    packed = attention(q, k, v, causal=causal, pack_gqa=True)
    unpacked = attention(q, k, v, causal=causal, pack_gqa=False)
    assert torch.equal(packed, unpacked)
    check_against_oracle(q, k, v, causal, pack_gqa=True)


@pytest.mark.parametrize("N_q", [1, 3, 16])
def test_kernel_pack_gqa_short_queries_long_kv(N_q):
    check_against_oracle(*make_cuda_qkv(2, 8, 2, N_q, 200, 64, torch.float16), causal=False, pack_gqa=True)


def test_pack_gqa_needs_block_m_divisible_by_group():
    q, k, v = make_cuda_qkv(2, 6, 2, 16, 16, 64, torch.float16)
    with pytest.raises(ValueError, match="BLOCK_M"):
        attention(q, k, v, causal=True, pack_gqa=True)
    check_against_oracle(q, k, v, causal=True)


def test_sm_scale_must_be_positive():
    q, k, v = make_cuda_qkv(2, 4, 2, 16, 16, 64, torch.float16)
    with pytest.raises(ValueError, match="sm_scale"):
        attention(q, k, v, sm_scale=-0.125)


@pytest.mark.parametrize("sm_scale", [0.03, 0.5])
def test_custom_sm_scale(sm_scale):
    q, k, v = make_cuda_qkv(1, 4, 2, 200, 200, 128, torch.bfloat16)
    ref = naive_attention(q, k, v, causal=True, sm_scale=sm_scale, dtype=torch.float64)
    ours = attention(q, k, v, causal=True, sm_scale=sm_scale)
    theirs = F.scaled_dot_product_attention(q, k, v, is_causal=True, scale=sm_scale, enable_gqa=True)
    assert errors(ours, ref) <= 2 * errors(theirs, ref) + ATOL_FLOOR


@pytest.mark.parametrize("block_m,block_n", [(32, 32), (32, 16), (64, 32), (16, 16)])
@pytest.mark.parametrize("causal", [True, False])
def test_kernel_other_tile_sizes(block_m, block_n, causal):
    """Tile-size hints the reference sweeps (tests/test_correctness.py:211-218)."""
    check_against_oracle(*make_cuda_qkv(2, 4, 2, 100, 100, 64, torch.float16), causal,
                         block_m=block_m, block_n=block_n)


# ------------------------------------------------------------- BASELINE configs, full size
CONFIGS = {
    "plumbing": dict(B=1, Hq=2, Hkv=2, N=256, D=64, dtype=torch.float16, causal=True),
    "mha_causal": dict(B=4, Hq=16, Hkv=16, N=4096, D=128, dtype=torch.bfloat16, causal=True),
    "headline": dict(B=2, Hq=32, Hkv=8, N=8192, D=128, dtype=torch.bfloat16, causal=True),
    "full_long": dict(B=2, Hq=32, Hkv=32, N=16384, D=64, dtype=torch.float16, causal=False, scale=0.5),
    "pack_tail": dict(B=16, Hq=64, Hkv=8, N=1000, D=128, dtype=torch.bfloat16, causal=True, spike_frac=0.01),
}


def config_inputs(c):
    return make_cuda_qkv(c["B"], c["Hq"], c["Hkv"], c["N"], c["N"], c["D"], c["dtype"],
                         scale=c.get("scale", 1.0), spike_frac=c.get("spike_frac", 0.0))


@pytest.mark.parametrize("name", list(CONFIGS))
def test_baseline_config_parity(name):
    c = CONFIGS[name]
    check_against_oracle(*config_inputs(c), c["causal"])


# Full-size shapes of the other dtype at each head dim. They run every compiled exp2 path on
# unmasked tiles: D=64 bf16 puts pairs 7 and 15 of each chunk on the FMA-pipe polynomial
# (degree 3), D=128 fp16 pairs 3, 7, 11 and 15 (degree 4); masked tiles use the MUFU only.
@pytest.mark.parametrize("name,shape", [
    ("full_long_bf16", dict(B=2, Hq=32, Hkv=32, N=16384, D=64, dtype=torch.bfloat16, causal=False, scale=0.5)),
    ("headline_fp16", dict(B=2, Hq=32, Hkv=8, N=8192, D=128, dtype=torch.float16, causal=True)),
    ("mha_causal_d64_bf16", dict(B=4, Hq=16, Hkv=16, N=4096, D=64, dtype=torch.bfloat16, causal=True)),
])
def test_full_size_other_dtype_parity(name, shape):
    check_against_oracle(*config_inputs(shape), shape["causal"])


def test_pack_tail_config_both_modes_bit_equal():
    c = CONFIGS["pack_tail"]
    q, k, v = config_inputs(c)
    packed = attention(q, k, v, causal=True, pack_gqa=True)
    unpacked = attention(q, k, v, causal=True, pack_gqa=False)
    assert torch.equal(packed, unpacked)
    check_against_oracle(q, k, v, True, pack_gqa=True)


# ------------------------------------------------------------ size-independent properties
def test_headline_linearity_in_v():
    """Scaling V by 2 is exact in bf16 and in every fp32 step: the output doubles exactly."""
    q, k, v = config_inputs(CONFIGS["headline"])
    a = attention(q, k, v)
    b = attention(q, k, v * 2)
    assert torch.equal(b, a * 2)


def test_headline_deterministic():
    q, k, v = config_inputs(CONFIGS["headline"])
    assert torch.equal(attention(q, k, v), attention(q, k, v))


@pytest.mark.parametrize("world", [2, 8])
def test_headline_shard_equals_slice(world):
    """Each (batch, kv-head) shard computed alone is bit-identical to its slice of the full
    run: sharding across GPUs cannot change results."""
    q, k, v = config_inputs(CONFIGS["headline"])
    full = attention(q, k, v).reshape(-1, q.shape[2], q.shape[3])
    G = q.shape[1] // k.shape[1]
    for r in (0, world - 1):
        qs, ks, vs = shard_qkv(q, k, v, r, world)
        lo = r * (q.shape[0] * k.shape[1]) // world
        part = attention(qs, ks, vs)
        assert torch.equal(part[0], full[lo * G: lo * G + part.shape[1]])


def test_batch_permutation():
    q, k, v = make_cuda_qkv(4, 8, 2, 700, 700, 128, torch.bfloat16)
    perm = torch.tensor([2, 0, 3, 1], device="cuda")
    a = attention(q, k, v)[perm]
    b = attention(q[perm], k[perm], v[perm])
    assert torch.equal(a, b)


def test_output_fully_written():
    """Canary: an output buffer pre-filled with NaN has no NaN left after a launch through
    the C ABI (every row of every tile, including ragged tails, is written)."""
    q, k, v = make_cuda_qkv(3, 8, 2, 333, 333, 128, torch.bfloat16)
    out = torch.full_like(q, float("nan"))
    p = _lib.make_params(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                         q.stride(), k.stride(), v.stride(), out.stride(),
                         3, 8, 2, 333, 333, 128, _lib.FA2_DTYPE_BF16, 1, 0, 1.0 / math.sqrt(128) * 1.4426950408889634)
    assert _lib.launch(p, torch.cuda.current_stream().cuda_stream) == _lib.FA2_OK
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
    assert torch.equal(out, attention(q, k, v))


# ------------------------------------------------------------- golden fixtures (reference)
@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(p)[:-3] for p in GOLDEN])
def test_golden_fixture(path):
    g = torch.load(path, weights_only=False)
    q, k, v = (g[n].cuda() for n in ("q", "k", "v"))
    kw = {"pack_gqa": g["pack_gqa"]} if g.get("pack_gqa") is not None else {}
    ours = attention(q, k, v, causal=g["causal"], **kw)
    ref = g["ref_naive"].cuda().double()
    theirs = F.scaled_dot_product_attention(q, k, v, is_causal=g["causal"], enable_gqa=True)
    e_ours, e_sdpa = errors(ours, ref), errors(theirs, ref)
    assert torch.isfinite(ours).all()
    assert e_ours <= 2 * e_sdpa + ATOL_FLOOR
    if "ref_triton" in g:
        # the reference kernel's own output (Triton interpreter) is within the same bar of ours
        e_cross = errors(ours, g["ref_triton"].cuda().double())
        assert e_cross <= 2 * (2 * e_sdpa + ATOL_FLOOR)


# ------------------------------------------------------------------ failure detection
@pytest.mark.parametrize("D", [64, 128])
def test_start_gate_timeout_is_reported(D):
    """A start gate that nothing opens: the kernel's bounded wait expires, it writes
    FA2_ERR_TIMEOUT to the error word, returns without a fault, and the context stays
    usable (a normal launch right after is correct). D = 128 runs the softmax warps'
    warp-voted waits, D = 64 the per-lane ones."""
    q, k, v = make_cuda_qkv(1, 2, 2, 256, 256, D, torch.float16)
    out = torch.zeros_like(q)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    gate = torch.zeros(1, dtype=torch.int32, device="cuda")  # never set
    p = _lib.make_params(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                         q.stride(), k.stride(), v.stride(), out.stride(),
                         1, 2, 2, 256, 256, D, _lib.FA2_DTYPE_FP16, 1, 0, 1.4426950408889634 / D ** 0.5,
                         err_flag=err.data_ptr(), timeout_cycles=20_000_000, gate=gate.data_ptr())
    assert _lib.launch(p, torch.cuda.current_stream().cuda_stream) == _lib.FA2_OK
    torch.cuda.synchronize()
    assert int(err.item()) == _lib.FA2_ERR_TIMEOUT
    assert torch.count_nonzero(out) == 0  # nothing was written
    # gate opened: same launch completes and is correct
    gate.fill_(1)
    err.zero_()
    assert _lib.launch(p, torch.cuda.current_stream().cuda_stream) == _lib.FA2_OK
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(out, attention(q, k, v))


# ------------------------------------------------------------------------ split-KV
# Extension beyond the reference (its README lists split-KV out of scope): short queries
# against long K/V split each CTA's K/V range over several CTAs and merge the fp32 partials.
@pytest.mark.parametrize("num_splits", [2, 3, 4, 7])
@pytest.mark.parametrize("causal", [False, True])
def test_split_kv_parity(num_splits, causal):
    N = 1000
    check_against_oracle(*make_cuda_qkv(2, 8, 2, N, N, 128, torch.bfloat16), causal, num_splits=num_splits)


@pytest.mark.parametrize("N_q,N_kv", [(1, 4096), (4, 4096), (16, 8192), (1, 1000), (33, 2048)])
@pytest.mark.parametrize("D", [64, 128])
def test_split_kv_short_queries(N_q, N_kv, D):
    q, k, v = make_cuda_qkv(4, 32, 8, N_q, N_kv, D, torch.bfloat16)
    from fa2.kernel import auto_num_splits
    assert auto_num_splits(4, 32, N_q, N_kv, 4, 4 if N_q * 4 <= 256 else 1, False) >= 1
    check_against_oracle(q, k, v, causal=False)                 # auto splits
    check_against_oracle(q, k, v, causal=False, num_splits=5)   # forced


def test_split_kv_more_splits_than_tiles():
    """Splits past a row block's K/V range are skipped by the kernel and by the merge."""
    check_against_oracle(*make_cuda_qkv(1, 4, 1, 300, 300, 64, torch.float16), True, num_splits=16)


@pytest.mark.parametrize("causal", [False, True])
def test_split_kv_pack_bit_equal(causal):
    q, k, v = make_cuda_qkv(2, 32, 4, 700, 700, 128, torch.bfloat16)
    a = attention(q, k, v, causal=causal, pack_gqa=True, num_splits=3)
    b = attention(q, k, v, causal=causal, pack_gqa=False, num_splits=3)
    assert torch.equal(a, b)


def test_split_kv_noncontiguous_output_strides():
    q, k, v = (t.transpose(1, 2).contiguous().transpose(1, 2)
               for t in make_cuda_qkv(2, 8, 2, 9, 3000, 128, torch.float16))
    out = check_against_oracle(q, k, v, causal=False, num_splits=4)
    assert out.stride() == q.stride()


@pytest.mark.parametrize("num_splits", [2, 3, 5, 8])
@pytest.mark.parametrize("N_kv", [1000, 4096])
def test_split_kv_dual_pairs(num_splits, N_kv):
    """All query rows in one Q tile: the CTA's two Q-tile slots stream two splits of the same
    rows. Odd counts round up to pairs, and a slot whose split lies past N_kv contributes
    nothing."""
    q, k, v = make_cuda_qkv(3, 16, 4, 7, N_kv, 128, torch.bfloat16)
    out = check_against_oracle(q, k, v, causal=False, pack_gqa=True, num_splits=num_splits)
    ref1 = attention(q, k, v, causal=False, pack_gqa=True, num_splits=1)
    assert (out.float() - ref1.float()).abs().max().item() < 2e-2


@pytest.mark.parametrize("D", [64, 128])
def test_split_kv_dual_fp16_unpacked(D):
    check_against_oracle(*make_cuda_qkv(2, 4, 4, 100, 3000, D, torch.float16), causal=False, num_splits=4)


def test_split_kv_combine_more_slices_than_grid_y():
    """More (batch, head block) slices than a grid's y extent allows (65535): the merge kernel
    strides over them. 1100 x 64 unpacked query heads = 70400 slices."""
    q, k, v = make_cuda_qkv(1100, 64, 1, 1, 1024, 128, torch.bfloat16, seed=5)
    check_against_oracle(q, k, v, causal=False, pack_gqa=False, num_splits=2)


# ------------------------------------------------------------- bottom-right causal mask
# Extension beyond the reference (whose wrapper asserts N_q == N_kv under causal and whose
# README lists bottom-right alignment out of scope): query i sees keys j <= i + N_kv - N_q,
# the decode / chunked-prefill mask. The oracle applies the same shifted tril.
@pytest.mark.parametrize("N_q", [1, 7, 300])
@pytest.mark.parametrize("N_kv", [1000, 8192])
@pytest.mark.parametrize("D,dtype", [(128, torch.bfloat16), (64, torch.float16)])
def test_bottom_right_causal(N_q, N_kv, D, dtype):
    q, k, v = make_cuda_qkv(2, 32, 8, N_q, N_kv, D, dtype, seed=N_q + N_kv)
    check_against_oracle(q, k, v, True, causal_align="bottom_right")                  # auto split-KV
    check_against_oracle(q, k, v, True, causal_align="bottom_right", num_splits=1)
    check_against_oracle(q, k, v, True, causal_align="bottom_right", pack_gqa=False, num_splits=3)


def test_bottom_right_equals_top_left_when_lengths_match():
    q, k, v = make_cuda_qkv(2, 8, 2, 777, 777, 128, torch.bfloat16)
    assert torch.equal(attention(q, k, v, causal=True, causal_align="bottom_right"), attention(q, k, v, causal=True))


def test_bottom_right_chunked_prefill_matches_full_causal_rows():
    """A chunk of queries at the end of a sequence, attended with the bottom-right mask against
    the whole K/V, gives the last rows of the full causal run (same values within the bar;
    the tile boundaries differ, so not bit for bit)."""
    q, k, v = make_cuda_qkv(1, 16, 4, 2048, 2048, 128, torch.bfloat16, seed=9)
    full = attention(q, k, v, causal=True)
    tail = attention(q[:, :, -300:], k, v, causal=True, causal_align="bottom_right")
    assert (tail.float() - full[:, :, -300:].float()).abs().max().item() < 2e-2
