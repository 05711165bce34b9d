"""CPU tests of the host side: the C-ABI library loads and exports what include/fa2_sm100.h
declares, its host-only validation mirrors the reference's asserts/ValueErrors
(fa2/kernel.py:218-244 of roy6n23/triton-fa2-forward), and the Python wrapper keeps the
reference's API (should_pack_gqa, _default_config, error messages, no CPU path)."""

import ctypes
import os
import re

import pytest
import torch

from fa2 import _lib
from fa2.kernel import _default_config, attention, should_pack_gqa

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "fa2_sm100.h")


def header_functions():
    txt = open(HEADER).read()
    return set(re.findall(r"FA2_API\s+[\w\s\*]+?\b(fa2_\w+)\s*\(", txt))


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    declared = header_functions()
    assert declared == set(_lib.EXPORTED)
    for name in declared:
        assert hasattr(L, name), name


def test_abi_version_and_struct_size():
    L = _lib.lib()
    assert L.fa2_sm100_abi_version() == _lib.ABI_VERSION
    assert L.fa2_sm100_params_size() == ctypes.sizeof(_lib.Fa2FwdParams) == 304


def test_config_entry_point():
    assert _lib.config(128)[:2] == (128, 128)
    assert _lib.config(64)[:2] == (128, 128)
    assert _lib.config(16) == _lib.config(32) == _lib.config(64)  # served by the 64 build
    with pytest.raises(_lib.Fa2Error):
        _lib.config(96)
    bm, bn, warps, stages = _default_config(128, True)
    assert (bm, bn) == (128, 128) and warps in (12, 20) and stages >= 2  # 8 or 16 softmax warps
    assert _default_config(64, False)[0] == 128


def test_strerror_covers_all_codes():
    for code in range(0, 15):
        assert _lib.strerror(code) != "unknown fa2_sm100 status"
    assert _lib.strerror(999) == "unknown fa2_sm100 status"


def contiguous_strides(B, H, N, D):
    return (H * N * D, N * D, D, 1)


def params(**kw):
    B, Hq, Hkv, Nq, Nkv, D = (kw.pop(n, d) for n, d in
                              (("B", 2), ("Hq", 8), ("Hkv", 2), ("Nq", 100), ("Nkv", 100), ("D", 128)))
    base = dict(q_ptr=0x1000, k_ptr=0x2000, v_ptr=0x3000, o_ptr=0x4000,
                q_stride=contiguous_strides(B, Hq, Nq, D), k_stride=contiguous_strides(B, Hkv, Nkv, D),
                v_stride=contiguous_strides(B, Hkv, Nkv, D), o_stride=contiguous_strides(B, Hq, Nq, D),
                batch=B, heads_q=Hq, heads_kv=Hkv, seqlen_q=Nq, seqlen_kv=Nkv, head_dim=D,
                dtype=_lib.FA2_DTYPE_BF16, causal=1, pack_gqa=0, qk_scale=0.1275)
    base.update(kw)
    return _lib.make_params(**base)


def test_check_accepts_valid():
    assert _lib.check(params()) == _lib.FA2_OK
    assert _lib.check(params(pack_gqa=1)) == _lib.FA2_OK
    assert _lib.check(params(causal=0, Nq=23, Nkv=70, D=64)) == _lib.FA2_OK
    assert _lib.check(params(Nq=0, Nkv=0, causal=0)) == _lib.FA2_ERR_SHAPE  # N_kv must be >= 1
    assert _lib.check(params(Nq=0, Nkv=5, causal=0)) == _lib.FA2_OK          # empty query is a no-op
    assert _lib.check(params(D=16)) == _lib.FA2_OK                            # 16 / 32 in place
    assert _lib.check(params(D=32, pack_gqa=1)) == _lib.FA2_OK


@pytest.mark.parametrize("kw,status", [
    (dict(q_ptr=0), _lib.FA2_ERR_NULL),
    (dict(o_ptr=0), _lib.FA2_ERR_NULL),
    (dict(batch=0), _lib.FA2_ERR_SHAPE),
    (dict(Nq=64, Nkv=100), _lib.FA2_ERR_SHAPE),          # causal needs N_q == N_kv (fa2/kernel.py:225-228)
    (dict(dtype=7), _lib.FA2_ERR_DTYPE),
    (dict(D=96), _lib.FA2_ERR_HEAD_DIM),
    (dict(D=8), _lib.FA2_ERR_HEAD_DIM),
    (dict(Hq=6, Hkv=4), _lib.FA2_ERR_GQA),                # fa2/kernel.py:223
    (dict(Hq=6, Hkv=2, pack_gqa=1), _lib.FA2_ERR_PACK),   # group 3 does not divide 128
    (dict(qk_scale=-0.1), _lib.FA2_ERR_SCALE),            # fa2/kernel.py:242-243
    (dict(qk_scale=float("nan")), _lib.FA2_ERR_SCALE),
    (dict(q_stride=(8 * 100 * 128, 100 * 128, 128, 2)), _lib.FA2_ERR_LAYOUT),  # d stride != 1
    (dict(k_stride=(2 * 100 * 130, 100 * 130, 130, 1)), _lib.FA2_ERR_LAYOUT),  # 260-byte rows
    (dict(v_ptr=0x3002), _lib.FA2_ERR_LAYOUT),            # misaligned base
    (dict(Nq=200, Nkv=100, causal_align=1), _lib.FA2_ERR_SHAPE),  # bottom-right needs N_q <= N_kv
    (dict(causal_align=2), _lib.FA2_ERR_SHAPE),           # unknown alignment
    (dict(num_splits=300), _lib.FA2_ERR_SHAPE),           # more than 256 splits
])
def test_check_rejects(kw, status):
    assert _lib.check(params(**kw)) == status


def test_bottom_right_causal_accepts_shorter_queries():
    assert _lib.check(params(Nq=7, Nkv=1000, causal_align=_lib.FA2_CAUSAL_BOTTOM_RIGHT)) == _lib.FA2_OK
    assert _lib.check(params(Nq=7, Nkv=1000, causal_align=_lib.FA2_CAUSAL_TOP_LEFT)) == _lib.FA2_ERR_SHAPE
    # non-causal calls ignore the alignment
    assert _lib.check(params(causal=0, Nq=300, Nkv=100, causal_align=_lib.FA2_CAUSAL_BOTTOM_RIGHT)) == _lib.FA2_OK


@pytest.mark.parametrize("kw", [dict(Hkv=0), dict(Hq=-(2 ** 31), Hkv=-1), dict(Hq=6, Hkv=4), dict(batch=0)])
def test_split_entry_points_reject_bad_heads_without_dividing(kw):
    """Shapes that the split-KV planner would divide by (H_kv = 0, INT_MIN / -1) come back as
    error codes from every entry point; no host arithmetic fault. Host only: the noalloc entry
    point validates before it touches the device."""
    L = _lib.lib()
    p = params(causal=0, Nq=4, Nkv=4096, num_splits=4, **kw)
    assert _lib.workspace_bytes(p) == 0
    assert _lib.check(p) in (_lib.FA2_ERR_SHAPE, _lib.FA2_ERR_GQA)
    assert L.fa2_fwd_sm100_noalloc(ctypes.byref(p), None) in (_lib.FA2_ERR_SHAPE, _lib.FA2_ERR_GQA)
    assert L.fa2_fwd_sm100(ctypes.byref(p), None) in (_lib.FA2_ERR_SHAPE, _lib.FA2_ERR_GQA)


def test_should_pack_gqa_follows_tile_efficiency():
    # the reference's truth table (tests/test_correctness.py:189-198)
    assert should_pack_gqa(1, 4, 128)
    assert should_pack_gqa(64, 4, 128)
    assert not should_pack_gqa(4096, 4, 128)
    assert not should_pack_gqa(1000, 4, 128)
    assert not should_pack_gqa(64, 1, 128)
    assert not should_pack_gqa(64, 3, 128)
    # config 5 (N=1000, group 8) is not auto-packed; its tests force both modes
    assert not should_pack_gqa(1000, 8, 128)


def cpu_qkv(Hq=4, Hkv=2, N=16, D=64, dtype=torch.float16):
    g = torch.Generator().manual_seed(0)
    return (torch.randn(2, Hq, N, D, generator=g).to(dtype), torch.randn(2, Hkv, N, D, generator=g).to(dtype),
            torch.randn(2, Hkv, N, D, generator=g).to(dtype))


def test_sm_scale_must_be_positive():
    q, k, v = cpu_qkv()
    with pytest.raises(ValueError, match="sm_scale"):
        attention(q, k, v, sm_scale=-0.125)


def test_pack_gqa_needs_block_m_divisible_by_group():
    q, k, v = cpu_qkv(Hq=6, Hkv=2)
    with pytest.raises(ValueError, match="BLOCK_M"):
        attention(q, k, v, causal=True, pack_gqa=True)


def test_reference_asserts_kept():
    q, k, v = cpu_qkv()
    with pytest.raises(AssertionError):
        attention(q, k[:, :, :8], v[:, :, :8], causal=True)       # causal with N_q != N_kv
    with pytest.raises(AssertionError):                            # bottom-right: N_q > N_kv
        attention(q, k[:, :, :8], v[:, :, :8], causal=True, causal_align="bottom_right")
    with pytest.raises(AssertionError):
        attention(q, k, v, causal=True, causal_align="diagonal")
    with pytest.raises(AssertionError):
        attention(q.float(), k.float(), v.float())                 # fp32 is not supported
    with pytest.raises(AssertionError):
        attention(*cpu_qkv(D=48))                                  # head_dim not a power of two
    with pytest.raises(AssertionError):
        attention(*cpu_qkv(Hq=6, Hkv=4))                           # H_q % H_kv


def test_no_cpu_path():
    """The product path has no CPU fallback: CPU tensors are rejected loudly."""
    q, k, v = cpu_qkv()
    with pytest.raises(RuntimeError, match="sm_100"):
        attention(q, k, v)


def test_workspace_validation_and_size():
    p = params(causal=0, Nq=4, Nkv=4096, num_splits=4)
    need = _lib.workspace_bytes(p)
    # 4 splits x (B * Hq) row slices x 256 padded rows x (D + 1) fp32 + 256
    assert need == 4 * (2 * 8) * 256 * 129 * 4 + 256
    assert _lib.check(p) == _lib.FA2_ERR_WORKSPACE                       # no workspace
    p2 = params(causal=0, Nq=4, Nkv=4096, num_splits=4, workspace=0x10000, workspace_bytes=need - 1)
    assert _lib.check(p2) == _lib.FA2_ERR_WORKSPACE                      # too small
    p3 = params(causal=0, Nq=4, Nkv=4096, num_splits=4, workspace=0x10008, workspace_bytes=need)
    assert _lib.check(p3) == _lib.FA2_ERR_WORKSPACE                      # misaligned
    p4 = params(causal=0, Nq=4, Nkv=4096, num_splits=4, workspace=0x10000, workspace_bytes=need)
    assert _lib.check(p4) == _lib.FA2_OK
    assert _lib.workspace_bytes(params()) == 0                           # no split, no workspace
    # head_dim 16 / 32: the partials have the 64 build's columns
    d16 = params(causal=0, Nq=4, Nkv=4096, num_splits=4, D=16)
    assert _lib.workspace_bytes(d16) == 4 * (2 * 8) * 256 * 65 * 4 + 256


def test_auto_num_splits():
    from fa2.kernel import auto_num_splits
    assert auto_num_splits(2, 32, 8192, 8192, 4, 1, True) == 1          # causal prefill: never
    assert auto_num_splits(2, 32, 8192, 8192, 4, 1, False) == 1         # GPU already full
    assert auto_num_splits(16, 32, 1, 4096, 4, 4, False) == 2           # decode: one split pair per CTA
    assert auto_num_splits(4, 32, 1, 65536, 4, 4, False) == 8           # 32 CTAs -> 4 pairs each
    assert auto_num_splits(2, 8, 200, 8192, 1, 1, False) == 9           # 200 rows (no pairs): 16 CTAs -> 144
    assert auto_num_splits(1, 8, 1, 512, 8, 8, False) == 1              # too few K/V tiles
    # bottom-right causal decode / chunked prefill splits like the unmasked case
    assert auto_num_splits(4, 32, 1, 65536, 4, 4, True, causal_align="bottom_right") == 8
    assert auto_num_splits(4, 32, 1, 65536, 4, 4, True) == 1            # top-left: N_q == N_kv only


def test_ablation_switches_exist_in_the_kernel_source():
    """Every compile-time switch the design-choice ablation passes is a macro the kernel source
    actually tests, so a renamed switch cannot silently build the shipped kernel twice."""
    import re

    import ablation
    import build as fa2_build

    src = "".join(open(p).read() for p in fa2_build.DEPENDS if p.endswith((".cu", ".cuh")))
    for name, flags in ablation.COMPILED.items():
        for f in flags:
            macro = re.match(r"-D(\w+)=", f).group(1)
            assert f"#ifndef {macro}" in src, (name, macro)
    for name, (lib, cfg, kwargs) in ablation.RUNTIME.items():
        assert lib in ablation.COMPILED
        assert set(kwargs) <= {"pack_gqa", "num_splits"}


def test_profile_target_configs_cover_the_ablation():
    import ablation
    from profile_target import CONFIGS

    for _, (_, cfg, _) in ablation.RUNTIME.items():
        assert cfg in CONFIGS
    for cfg in ("headline", "mha_causal", "full_long", "pack_tail", "decode"):
        assert cfg in CONFIGS


@pytest.mark.parametrize("flag", ["-DFA2_ROW_SPLIT=2", "-DFA2_PAIR=1"])
def test_alternative_layouts_build(tmp_path, flag):
    """The alternatives the shipped library leaves out still compile for sm_100a, so their
    register and shared-memory budgets (static_asserts) and code stay checked: the 20-warp layout
    (two softmax warps per row quadrant) and the CTA-pair kernel (cta_group::2, fa2_pair_sm100.cuh).
    Compilation only: no GPU."""
    import shutil
    import subprocess

    import build as fa2_build

    nvcc = fa2_build.nvcc_path()
    if shutil.which(nvcc) is None and not os.path.exists(nvcc):
        pytest.skip("nvcc not available")
    out = tmp_path / "libfa2_variant.so"
    cmd = [nvcc, *fa2_build.NVCC_FLAGS, flag, "-I", fa2_build.INCLUDE, "-I", fa2_build.CSRC,
           "-o", str(out), *fa2_build.SOURCES]
    res = subprocess.run(cmd, capture_output=True, text=True)
    assert res.returncode == 0, res.stderr[-3000:]
    assert out.stat().st_size > 0


def test_integration_doc_ctypes_mirror_matches_the_library():
    """The ctypes struct that INTEGRATION.md tells a maintainer to paste is exec'd against the
    built library: its size must be the library's sizeof(Fa2FwdParams)."""
    doc = open(os.path.join(os.path.dirname(HEADER), "..", "INTEGRATION.md")).read()
    blocks = re.findall(r"```python\n(.*?)```", doc, flags=re.S)
    mirror = [b for b in blocks if "class Fa2FwdParams" in b]
    assert len(mirror) == 1
    ns = {"LIB_PATH": _lib.LIB_PATH}
    exec(mirror[0], ns)  # runs the snippet's own size assertion
    assert ctypes.sizeof(ns["Fa2FwdParams"]) == ctypes.sizeof(_lib.Fa2FwdParams)
    assert [f[0] for f in ns["Fa2FwdParams"]._fields_] == [f[0] for f in _lib.Fa2FwdParams._fields_]
