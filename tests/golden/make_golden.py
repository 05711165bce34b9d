"""Generate the golden fixtures in tests/golden/*.pt from the reference implementation itself.

Runs only where a checkout of the reference (roy6n23/triton-fa2-forward) is available; its
root directory is the required argument. The committed .pt files are what the tests use on any
box. For each case it stores the seeded inputs and
  * ref_naive     fa2.reference.naive_attention on fp64 copies of the inputs (the
                  reference tests' ground truth, tests/test_correctness.py:93), as fp32
  * ref_blocked   fa2.reference.blocked_attention on the same fp64 inputs (fp32 state), as
                  fp32 (smallest cases only)
  * ref_triton    the reference's Triton kernel fa2.kernel.attention run by Triton's CPU
                  interpreter (TRITON_INTERPRET=1, as the reference CI does), in the input
                  dtype; omitted for bf16 (the interpreter's bf16 dot is wrong,
                  reference tests/test_correctness.py:116-121)

    python tests/golden/make_golden.py REFERENCE_ROOT
"""

import os
import sys

os.environ["TRITON_INTERPRET"] = "1"  # must precede the first triton import

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
if len(sys.argv) != 2 or not os.path.isdir(os.path.join(sys.argv[1], "fa2")):
    sys.exit("usage: python tests/golden/make_golden.py REFERENCE_ROOT  (the directory holding the reference's fa2/)")
REF_ROOT = sys.argv[1]

sys.path.insert(0, REPO)
import torch  # noqa: E402

from oracle.reference import make_qkv  # noqa: E402

# (name, B, H_q, H_kv, N_q, N_kv, D, dtype, causal, extra)
# The tiled mirror (ref_blocked) is stored only for the smallest cases to keep fixtures small.
WITH_BLOCKED = {"gqa_noncausal_ragged_d64", "gqa_pack_causal_d64", "d16_causal"}
CASES = [
    ("plumbing_fp16_causal_d64", 1, 2, 2, 256, 256, 64, torch.float16, True, {}),
    ("gqa_noncausal_ragged_d64", 1, 4, 2, 23, 70, 64, torch.float16, False, {}),
    ("gqa_pack_causal_d64", 1, 8, 2, 37, 37, 64, torch.float16, True, {"pack_gqa": True}),
    ("mqa_causal_d128", 1, 4, 1, 100, 100, 128, torch.float16, True, {}),
    ("d16_causal", 1, 4, 2, 37, 37, 16, torch.float16, True, {}),
    ("bf16_spiky_causal_d128", 1, 2, 1, 200, 200, 128, torch.bfloat16, True, {"spike_frac": 0.01}),
    ("bf16_noncausal_d64", 1, 4, 2, 100, 100, 64, torch.bfloat16, False, {}),
]


def main():
    sys.path.insert(0, REF_ROOT)
    from fa2.reference import blocked_attention, naive_attention  # the reference's own
    from fa2.kernel import attention as ref_kernel

    for name, B, Hq, Hkv, Nq, Nkv, D, dt, causal, extra in CASES:
        spike = extra.get("spike_frac", 0.0)
        q, k, v = make_qkv(B, Hq, Hkv, Nq, Nkv, D, dt, seed=0, spike_frac=spike)
        qd, kd, vd = q.double(), k.double(), v.double()
        rec = {
            "name": name, "causal": causal, "q": q, "k": k, "v": v,
            "pack_gqa": extra.get("pack_gqa"),
            "ref_naive": naive_attention(qd, kd, vd, causal=causal).float(),
        }
        if name in WITH_BLOCKED:
            rec["ref_blocked"] = blocked_attention(qd, kd, vd, causal=causal).float()
        if dt == torch.float16:
            kw = {"pack_gqa": extra["pack_gqa"]} if "pack_gqa" in extra else {}
            rec["ref_triton"] = ref_kernel(q, k, v, causal=causal, **kw)
        path = os.path.join(HERE, f"{name}.pt")
        torch.save(rec, path)
        print(f"{name}: {os.path.getsize(path) / 1024:.0f} KiB")


if __name__ == "__main__":
    main()
