"""Where one K/V step's cycles go: builds the library with FA2_TRACE=1 (SM-clock stamps of CTA 0 at
the hand-off points of the softmax warps and the MMA thread, see FA2_STAMP in
csrc/fa2_fwd_sm100.cu), runs a config and prints, per Q tile, the median time of each event
relative to that tile's S being seen by its softmax warps, over the steady-state steps of one unit.

    python triton-fa2-forward_b200/step_trace.py [--config headline] [--unit 0]

The stamps are clock64 reads plus one global store each, taken by one lane; they perturb the
schedule slightly, so the step time here is close to, not equal to, the untraced kernel's. The
library is built into triton-fa2-forward_b200/_build/trace/ (no GPU needed to build).
"""

import argparse
import ctypes
import os
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, PKG_DIR)

import build as fa2_build  # noqa: E402

TRACE_LIB = os.path.join(PKG_DIR, "_build", "trace", "libfa2_sm100_trace.so")
UNITS, STEPS, EVENTS = 4, 80, 32
# event ids of FA2_STAMP (per unit n, step j, tile t)
SOFTMAX = {0: "S seen", 1: "S in registers", 2: "row max", 3: "first P hand-off", 4: "last P hand-off",
           5: "row sum done"}
MMA = {6: "V_j landed (tile 0)", 7: "first P hand-off seen", 8: "first PV part issued", 9: "last P hand-off seen",
       10: "second PV part issued", 11: "next K landed", 12: "next QK issued and committed"}


def build_trace_lib():
    if fa2_build.up_to_date(out=TRACE_LIB):
        return TRACE_LIB
    os.makedirs(os.path.dirname(TRACE_LIB), exist_ok=True)
    cmd = [fa2_build.nvcc_path(), *fa2_build.NVCC_FLAGS, "-DFA2_TRACE=1", "-I", fa2_build.INCLUDE, "-I",
           fa2_build.CSRC, "-o", TRACE_LIB, *fa2_build.SOURCES]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed:\n{res.stderr}")
    return TRACE_LIB


def summarize(buf, unit):
    """Per tile, medians over the unit's steady-state steps (the first and last 3 left out)."""
    import numpy as np

    T = buf[unit].astype(np.float64)  # [step, tile, event]
    J = int((T[:, 0, 0] != 0).sum())
    if J < 8:
        return f"unit {unit}: {J} steps stamped, too few for a steady state"
    js = list(range(3, J - 3))
    lines = [f"unit {unit}: {J} K/V steps; step time (tile 0 S seen to the next) median "
             f"{np.median(np.diff(T[3:J - 3, 0, 0])):.0f} cycles"]
    for t in range(2):
        def rel(e):
            vals = [T[j, t, e] - T[j, t, 0] for j in js if T[j, t, e] != 0 and T[j, t, 0] != 0]
            return np.median(vals) if vals else float("nan")
        lines.append(f" Q tile {t} (cycles after its S is seen):")
        for e, name in SOFTMAX.items():
            lines.append(f"   softmax warp 0  {name:30s} {rel(e):8.0f}")
        for e, name in MMA.items():
            if e == 6 and t == 1:
                continue
            lines.append(f"   MMA thread      {name:30s} {rel(e):8.0f}")
        per_q = "  ".join(f"q{q}: {rel(20 + q):.0f} / {rel(24 + q):.0f}" for q in range(4))
        lines.append(f"   first / last P hand-off per warp   {per_q}")
    off = np.median([T[j, 1, 0] - T[j, 0, 0] for j in js])
    lines.append(f" tile 1 S seen - tile 0 S seen: {off:.0f} cycles")
    return "\n".join(lines)


def main():
    import numpy as np

    ap = argparse.ArgumentParser()
    ap.add_argument("--config", default="headline")
    ap.add_argument("--unit", type=int, default=0)
    args = ap.parse_args()
    lib = build_trace_lib()
    from fa2 import _lib
    _lib.LIB_PATH = lib
    import torch

    from fa2.kernel import attention, check_device_errors
    from profile_target import CONFIGS

    B, Hq, Hkv, N, D, dt, causal, scale = CONFIGS[args.config]
    n_q, n_kv = N if isinstance(N, tuple) else (N, N)
    g = torch.Generator(device="cuda").manual_seed(0)
    q = torch.randn(B, Hq, n_q, D, device="cuda", dtype=dt, generator=g) * scale
    k = torch.randn(B, Hkv, n_kv, D, device="cuda", dtype=dt, generator=g) * scale
    v = torch.randn(B, Hkv, n_kv, D, device="cuda", dtype=dt, generator=g) * scale
    L = _lib.lib()
    L.fa2_trace_read.argtypes = [ctypes.c_void_p, ctypes.c_int64]
    for _ in range(3):
        attention(q, k, v, causal=causal)
    torch.cuda.synchronize()
    assert L.fa2_trace_clear() == 0
    attention(q, k, v, causal=causal)
    torch.cuda.synchronize()
    check_device_errors()
    buf = np.zeros((UNITS, STEPS, 2, EVENTS), dtype=np.int64)
    assert L.fa2_trace_read(buf.ctypes.data, buf.nbytes) == 0
    print(f"{args.config}: CTA 0")
    print(summarize(buf, args.unit))


if __name__ == "__main__":
    main()
