"""Profiling target: a few warm-up launches of the FA2 forward on one config, then the
launch(es) a profiler captures (e.g. `ncu -k regex:fa2_fwd -s <warmup> -c 1`).
Mirrors the role of the reference's bench/profile_target.py.

    python triton-fa2-forward_b200/profile_target.py [--config headline] [--warmup 2] [--launches 1]
        [--lib path/to/libfa2_sm100_variant.so]   (a library built by ablation.py)
        [--impl fa4]   (the same shapes through vLLM's CuTe-DSL sm_100 forward, a same-box yardstick)

Configs are the BASELINE.json shapes; inputs are seeded N(0,1) generated on the device.
The headline config holds 470 MB (inputs 335 MB > 126 MB L2), so DRAM counters are meaningful.
"""

import argparse
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

import torch  # noqa: E402

CONFIGS = {
    "plumbing": (1, 2, 2, 256, 64, torch.float16, True, 1.0),
    "mha_causal": (4, 16, 16, 4096, 128, torch.bfloat16, True, 1.0),
    "headline": (2, 32, 8, 8192, 128, torch.bfloat16, True, 1.0),
    "full_long": (2, 32, 32, 16384, 64, torch.float16, False, 0.5),
    "pack_tail": (16, 64, 8, 1000, 128, torch.bfloat16, True, 1.0),
    # short query against a long K/V (decode): HBM-bound, GQA-packed, split-KV in pairs
    "decode": (4, 32, 8, (1, 65536), 128, torch.bfloat16, False, 1.0),
    # the other dtype at each head dim (design-choice ablation)
    "mha_causal_fp16": (4, 16, 16, 4096, 128, torch.float16, True, 1.0),
    "full_long_bf16": (2, 32, 32, 16384, 64, torch.bfloat16, False, 0.5),
    "mha_causal_d64": (4, 16, 16, 4096, 64, torch.bfloat16, True, 1.0),
    "mqa_causal": (2, 32, 1, 4096, 128, torch.bfloat16, True, 1.0),
    "noncausal_128": (2, 32, 8, 8192, 128, torch.bfloat16, False, 1.0),
}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", choices=list(CONFIGS), default="headline")
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--launches", type=int, default=1)
    ap.add_argument("--pack", choices=["auto", "on", "off"], default="auto")
    ap.add_argument("--lib", default=None, help="load this build of libfa2_sm100.so instead of the shipped one")
    ap.add_argument("--impl", choices=["fa2", "fa4"], default="fa2",
                    help="fa4: vLLM's CuTe-DSL FlashAttention forward on the same shapes (yardstick)")
    args = ap.parse_args()
    if args.impl == "fa4":
        run_fa4(args)
        return
    if args.lib:
        from fa2 import _lib
        _lib.LIB_PATH = os.path.abspath(args.lib)
    from fa2.kernel import attention, check_device_errors
    B, Hq, Hkv, N, D, dt, causal, scale = CONFIGS[args.config]
    n_q, n_kv = N if isinstance(N, tuple) else (N, N)
    g = torch.Generator(device="cuda").manual_seed(0)
    q = torch.randn(B, Hq, n_q, D, device="cuda", dtype=dt, generator=g) * scale
    k = torch.randn(B, Hkv, n_kv, D, device="cuda", dtype=dt, generator=g) * scale
    v = torch.randn(B, Hkv, n_kv, D, device="cuda", dtype=dt, generator=g) * scale
    pack = {"auto": None, "on": True, "off": False}[args.pack]
    for _ in range(args.warmup + args.launches):
        attention(q, k, v, causal=causal, pack_gqa=pack)
    torch.cuda.synchronize()
    check_device_errors()
    print(f"ok: {args.config} x{args.warmup + args.launches}")


def run_fa4(args):
    """The same seeded shapes through vLLM's FlashAttention-4 forward ([B, N, H, D] layout), for
    counter comparisons under a profiler. Library code, not part of this package's path."""
    from vllm.vllm_flash_attn.cute.interface import flash_attn_func
    B, Hq, Hkv, N, D, dt, causal, scale = CONFIGS[args.config]
    n_q, n_kv = N if isinstance(N, tuple) else (N, N)
    g = torch.Generator(device="cuda").manual_seed(0)
    q = (torch.randn(B, Hq, n_q, D, device="cuda", dtype=dt, generator=g) * scale).transpose(1, 2).contiguous()
    k = (torch.randn(B, Hkv, n_kv, D, device="cuda", dtype=dt, generator=g) * scale).transpose(1, 2).contiguous()
    v = (torch.randn(B, Hkv, n_kv, D, device="cuda", dtype=dt, generator=g) * scale).transpose(1, 2).contiguous()
    for _ in range(args.warmup + args.launches):
        flash_attn_func(q, k, v, causal=causal)
    torch.cuda.synchronize()
    print(f"ok: fa4 {args.config} x{args.warmup + args.launches}")


if __name__ == "__main__":
    main()
