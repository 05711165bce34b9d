"""Design-choice ablation: each choice of the sm_100a kernel against its alternative, timed
on the BASELINE configs (the role of the reference's bench/ablation.py).

Every variant computes the full attention (no work is skipped); they differ only in how:

  shipped        the library as built by build.py
  no_persistent  one CTA per 256-row work unit (FA2_PERSISTENT=0) instead of one CTA per SM
                 walking the units
  all_mufu       every exp2 on the MUFU (shipped: 12.5%, pairs 7 and 15, on the FMA pipe at D=128; at D=64 12.5%
                 for bf16 and none for fp16)
  emu_25         25% of the exp2 (pairs 3, 7, 11, 15) on the FMA pipe at both head dims
  emu_50         half of the exp2 on the FMA pipe at both head dims
  emu_25_pairs_0/1/2/3   25% at D=128 on pairs 0,4,8,12 / 1,5,9,13 / 2,6,10,14 / 3,7,11,15 of
                 each chunk (the last shipped before the warp-voted waits; shipped: 7, 15)
  d64_fp16_all_mufu   every exp2 on the MUFU at D=64 fp16 (shipped: pairs 7, 15 on the FMA pipe)
  d64_emu_pairs_3_11, d64_emu_3pairs   at D=64, pairs 3, 11 (12.5%) or 5, 10, 15 (18.75%) on the
                 FMA pipe instead of 7, 15
  d64_bf16_all_mufu   every exp2 on the MUFU at D=64 bf16
  emu_12, emu_37 12.5% on pairs 1, 9 or 37.5% on the FMA pipe at D=128 (emu_12_pairs_7 = shipped)
  p_split_2      P handed to the MMA warp after 64 of 128 columns (FA2_P_SPLIT=2) instead of 96
  no_spec_max    the row max taken before any exp2 at both head dims (shipped: at D=128 only)
  spec_max       P's first chunks computed with the current reference max while the row max is
                 taken, with a redo when a max moves, at both head dims (shipped: at D=64 only)
  two_issuers    one MMA-issuing thread per Q tile (FA2_TWO_ISSUERS=1) instead of one for both
  stages_4, stages_2   K/V ring of 4 (2) slots at D=128, 8 (4) at D=64 (shipped: 3 and 8); the
                 4-slot ring only fits with one O staging chunk per warp
  stg_chunk      O staged one 64-column chunk at a time per warp (FA2_STG_FULL=0) instead of whole
  no_l2_hints    TMA loads with evict_normal in L2 (FA2_L2_HINTS=0) instead of K/V evict_last, Q evict_first
  mma_spin       the MMA thread polls its barriers without suspending (FA2_MMA_SPIN=1)
  rescale_th_12  the running max moves only past 2^12 (FA2_RESCALE_TH=12) instead of 2^8
  regs_208       softmax warps at 208 registers, the MMA/TMA warpgroup at 88 (shipped: 200 / 104)
  s_load_x64     a softmax warp's scores loaded from TMEM in 64-column tcgen05.ld instructions
                 (shipped: four of 32 columns at D=128, one of 128 at D=64)
  d128_s_load_x128, d64_s_load_x32   the other load width at one head dim
  d64_regs_208   208 / 88 registers at D=64 only
  fp16_poly_deg4 the degree-4 exp2 polynomial for fp16 P (shipped: degree 3, as for bf16)
  row_split_2    two softmax warps per row quadrant, 64 scores each, exchanging the row max and
                 row sum through TMEM (FA2_ROW_SPLIT=2: 20 warps, setmaxnreg 104/64) instead of
                 one warp taking all 128 scores (12 warps, 200/104)
  row_major_noncausal   without a causal mask, the persistent CTAs walk the units row block by
                 row block (FA2_HEAD_MAJOR=0) instead of (batch, head) slice by slice
  defer_epi      a unit's output written during the next unit's first step, after its P hand-off
                 (FA2_DEFER_EPI=1) instead of when the unit ends
  d64_sep_p      at D=64, P in TMEM columns of its own and the next QK of a tile issued as soon as
                 its scores are read (FA2_SEP_P_D64=1) instead of P overwriting S_t
  seq_exp        the two softmax warps of a lane quadrant take turns on the exponential phase of
                 a step (FA2_SEQ_EXP=1, a bounded mbarrier hand-shake) instead of running freely
  ffma_pass      s * qk_scale - m for the whole row in one FMA pass before the exponentials
                 (FA2_FFMA_PASS=1) instead of fused into the per-chunk loop
  seq_exp_ffma_pass   both
  lane_waits     at D=128 each softmax lane runs its own probe loop for S and O and the warp votes
                 once at the end (FA2_WARP_WAIT_D128=0) instead of warp-voted probes
  probe8         mbarrier waits probe 8 times per loop iteration in one PTX block (FA2_WAIT_UNROLL=8)
  wait_suspend_20us   mbarrier waits with a 20 us suspend-time hint (FA2_WAIT_SUSPEND_NS=20000)
                 instead of the default, as CUTLASS's barriers use (with 10 ms)
  pair           CTA pairs at D=128 (FA2_PAIR=1: fixed-length launches without split-KV of at
                 least 1024 packed rows per head block run fa2_fwd_pair_kernel, one M = 256
                 cta_group::2 MMA over two SMs with K/V split between them) instead of one CTA
  pack_off       (runtime) GQA head packing forced off, on the pack_tail config (the wrapper
                 packs whenever the group divides 128; the reference's rule would not pack here)
  pack_off_headline, pack_off_mqa   the same on the headline and on an MQA shape
  splitkv_off    (runtime) split-KV off (num_splits=1), on the decode config

    python triton-fa2-forward_b200/ablation.py [--variants shipped,all_mufu] [--configs headline]

Variant libraries are compiled into triton-fa2-forward_b200/_build/ablation/ and each runs in a
child process. Timing: 3 warm-up calls, then the median of 20 calls with a 256 MiB L2 flush
before each, CUDA events on the current stream. Prints one JSON line per (variant, config).
"""

import argparse
import json
import os
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, PKG_DIR)

import build as fa2_build  # noqa: E402

BUILD_DIR = os.path.join(PKG_DIR, "_build", "ablation")

COMPILED = {
    "shipped": [],
    "no_persistent": ["-DFA2_PERSISTENT=0"],
    "all_mufu": ["-DFA2_EMU_MASK_D128=0x0u", "-DFA2_EMU_MASK_D64=0x0u", "-DFA2_EMU_MASK_D64_BF16=0x0u"],
    "emu_25": ["-DFA2_EMU_MASK_D128=0x8888u", "-DFA2_EMU_MASK_D64=0x8888u", "-DFA2_EMU_MASK_D64_BF16=0x8888u"],
    "emu_50": ["-DFA2_EMU_MASK_D128=0x5555u", "-DFA2_EMU_MASK_D64=0x5555u", "-DFA2_EMU_MASK_D64_BF16=0x5555u"],
    "emu_25_pairs_0": ["-DFA2_EMU_MASK_D128=0x1111u"],
    "emu_25_pairs_1": ["-DFA2_EMU_MASK_D128=0x2222u"],
    "emu_25_pairs_2": ["-DFA2_EMU_MASK_D128=0x4444u"],
    "emu_25_pairs_3": ["-DFA2_EMU_MASK_D128=0x8888u"],
    "emu_12": ["-DFA2_EMU_MASK_D128=0x0202u"],
    "emu_12_pairs_7": ["-DFA2_EMU_MASK_D128=0x8080u"],
    "d64_fp16_all_mufu": ["-DFA2_EMU_MASK_D64=0x0u"],
    "d64_emu_pairs_3_11": ["-DFA2_EMU_MASK_D64=0x0808u", "-DFA2_EMU_MASK_D64_BF16=0x0808u"],
    "d64_emu_3pairs": ["-DFA2_EMU_MASK_D64=0x8420u", "-DFA2_EMU_MASK_D64_BF16=0x8420u"],
    "d64_bf16_all_mufu": ["-DFA2_EMU_MASK_D64_BF16=0x0u"],
    "emu_37": ["-DFA2_EMU_MASK_D128=0x2A2Au"],
    "p_split_2": ["-DFA2_P_SPLIT=2"],
    "no_spec_max": ["-DFA2_SPEC_MAX_D128=0", "-DFA2_SPEC_MAX_D64=0"],
    "spec_max": ["-DFA2_SPEC_MAX_D128=1", "-DFA2_SPEC_MAX_D64=1"],
    "two_issuers": ["-DFA2_TWO_ISSUERS=1"],
    "stages_4": ["-DFA2_STAGES_D128=4", "-DFA2_STAGES_D64=8", "-DFA2_STG_FULL=0"],
    "stages_2": ["-DFA2_STAGES_D128=2", "-DFA2_STAGES_D64=4"],
    "stg_chunk": ["-DFA2_STG_FULL=0"],
    "no_l2_hints": ["-DFA2_L2_HINTS=0"],
    "mma_spin": ["-DFA2_MMA_SPIN=1"],
    "rescale_th_12": ["-DFA2_RESCALE_TH=12.0f"],
    "row_split_2": ["-DFA2_ROW_SPLIT=2"],
    "regs_208": ["-DFA2_REGS_SOFTMAX_D128=208", "-DFA2_REGS_SOFTMAX_D64=208"],
    "s_load_x64": ["-DFA2_S_LOAD_X_D128=64", "-DFA2_S_LOAD_X_D64=64"],
    "d128_s_load_x128": ["-DFA2_S_LOAD_X_D128=128"],
    "d64_s_load_x32": ["-DFA2_S_LOAD_X_D64=32"],
    "d64_regs_208": ["-DFA2_REGS_SOFTMAX_D64=208"],
    "fp16_poly_deg4": ["-DFA2_POLY_DEG_FP16=4"],
    "seq_exp": ["-DFA2_SEQ_EXP=1"],
    "d64_sep_p": ["-DFA2_SEP_P_D64=1"],
    "defer_epi": ["-DFA2_DEFER_EPI=1"],
    "row_major_noncausal": ["-DFA2_HEAD_MAJOR=0"],
    "ffma_pass": ["-DFA2_FFMA_PASS=1"],
    "seq_exp_ffma_pass": ["-DFA2_SEQ_EXP=1", "-DFA2_FFMA_PASS=1"],
    "pair": ["-DFA2_PAIR=1"],
    "probe8": ["-DFA2_WAIT_UNROLL=8"],
    "lane_waits": ["-DFA2_WARP_WAIT_D128=0"],
    "wait_suspend_20us": ["-DFA2_WAIT_SUSPEND_NS=20000"],
}
RUNTIME = {
    # name: (library variant, config it applies to, attention() keyword arguments)
    "pack_off": ("shipped", "pack_tail", {"pack_gqa": False}),
    "pack_off_headline": ("shipped", "headline", {"pack_gqa": False}),
    "pack_off_mqa": ("shipped", "mqa_causal", {"pack_gqa": False}),
    "splitkv_off": ("shipped", "decode", {"num_splits": 1}),
}


def lib_path(name):
    return os.path.join(BUILD_DIR, f"libfa2_sm100_{name}.so")


def build_variant(name):
    """Compile one variant library (skipped when it is newer than every source)."""
    os.makedirs(BUILD_DIR, exist_ok=True)
    out = lib_path(name)
    if fa2_build.up_to_date(out=out):
        return out
    cmd = [fa2_build.nvcc_path(), *fa2_build.NVCC_FLAGS, *COMPILED[name], "-I", fa2_build.INCLUDE,
           "-I", fa2_build.CSRC, "-o", out, *fa2_build.SOURCES]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {name}:\n{res.stderr}")
    return out


def child(lib, config, kwargs_json):
    """Runs in a fresh process: time `config` with library `lib`, print one JSON line."""
    from fa2 import _lib

    _lib.LIB_PATH = lib
    import torch

    from fa2.kernel import attention, check_device_errors
    from profile_target import CONFIGS as SHAPES

    kwargs = json.loads(kwargs_json)
    B, Hq, Hkv, N, D, dt, causal, scale = SHAPES[config]
    n_q, n_kv = N if isinstance(N, tuple) else (N, N)
    g = torch.Generator(device="cuda").manual_seed(0)
    q = torch.randn(B, Hq, n_q, D, device="cuda", dtype=dt, generator=g) * scale
    k = torch.randn(B, Hkv, n_kv, D, device="cuda", dtype=dt, generator=g) * scale
    v = torch.randn(B, Hkv, n_kv, D, device="cuda", dtype=dt, generator=g) * scale
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    for _ in range(3):
        attention(q, k, v, causal=causal, **kwargs)
    torch.cuda.synchronize()
    ts = []
    for _ in range(20):
        flush.fill_(1)
        torch.cuda._sleep(200_000)  # keeps the stream ahead of the host's launch
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        attention(q, k, v, causal=causal, **kwargs)
        e.record()
        torch.cuda.synchronize()
        ts.append(s.elapsed_time(e))
    check_device_errors()
    ts.sort()
    ms = ts[len(ts) // 2]
    pairs = n_q * (n_q + 1) / 2 if causal else n_q * n_kv
    tflops = 4 * B * Hq * pairs * D / (ms * 1e-3) / 1e12
    nbytes = (q.numel() * 2 + k.numel() + v.numel()) * q.element_size()
    print(json.dumps({"config": config, "ms": ms, "tflops": tflops,
                      "gbs": nbytes / (ms * 1e-3) / 1e9, "iqr_ms": ts[15] - ts[5]}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--variants", default=",".join(list(COMPILED) + list(RUNTIME)))
    ap.add_argument("--configs", default="headline,mha_causal,full_long")
    ap.add_argument("--child", nargs=3, metavar=("LIB", "CONFIG", "KWARGS"))
    ap.add_argument("--build-only", action="store_true")
    args = ap.parse_args()
    if args.child:
        child(*args.child)
        return 0
    variants = [v for v in args.variants.split(",") if v]
    for v in variants:
        build_variant(RUNTIME[v][0] if v in RUNTIME else v)
    if args.build_only:
        return 0
    rc = 0
    for v in variants:
        if v in RUNTIME:
            libname, cfg, kw = RUNTIME[v]
            runs = [("shipped", cfg, {}), (v, cfg, kw)]
        else:
            libname = v
            runs = [(v, c, {}) for c in args.configs.split(",") if c]
        for name, cfg, kw in runs:
            res = subprocess.run([sys.executable, os.path.abspath(__file__), "--child", lib_path(libname), cfg,
                                  json.dumps(kw)], capture_output=True, text=True, timeout=600)
            line = [ln for ln in res.stdout.splitlines() if ln.startswith("{")]
            if res.returncode != 0 or not line:
                print(json.dumps({"variant": name, "config": cfg, "error": res.stderr[-400:]}), flush=True)
                rc = 1
                continue
            d = json.loads(line[0])
            d["variant"] = name
            print(json.dumps(d), flush=True)
    return rc


if __name__ == "__main__":
    sys.exit(main())
