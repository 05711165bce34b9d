"""Counters-only summaries of Nsight Compute output for the FA2 kernel.

Equivalent of the reference's bench/ncu_summary.py summary() (tensor pipe, DRAM, stall
reasons), restricted to the metric pages (`--page raw`); it never reads the source page.

    # one-kernel report (--set full or sections) -> key counters
    ncu -i prof.ncu-rep --page raw --csv > raw.csv
    python triton-fa2-forward_b200/ncu_summary.py kernel raw.csv [--flops F] [--peak-tflops P]

    # launch list (--metrics gpu__time_duration.sum --csv --log-file launches.csv)
    python triton-fa2-forward_b200/ncu_summary.py launches launches.csv
"""

import argparse
import collections
import csv
import sys

KEYS = [
    ("gpu__time_duration.sum", "duration"),
    ("sm__cycles_elapsed.avg.per_second", "SM clock"),
    ("sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_elapsed", "tensor pipe active % (elapsed)"),
    ("sm__inst_executed_pipe_xu.avg.pct_of_peak_sustained_active", "XU (MUFU) pipe %"),
    ("sm__pipe_fma_cycles_active.avg.pct_of_peak_sustained_active", "FMA pipe %"),
    ("sm__pipe_alu_cycles_active.avg.pct_of_peak_sustained_active", "ALU pipe %"),
    ("smsp__issue_active.avg.pct_of_peak_sustained_active", "issue active %"),
    ("smsp__inst_executed.sum", "warp instructions executed"),
    ("sm__pipe_shared_cycles_active.avg.pct_of_peak_sustained_elapsed", "shared pipe active % (elapsed)"),
    ("l1tex__data_pipe_tc_wavefronts_mem_shared.sum.pct_of_peak_sustained_elapsed", "smem wavefronts for tcgen05 %"),
    ("dram__bytes_read.sum", "DRAM read"),
    ("dram__bytes_write.sum", "DRAM write"),
    ("gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed", "DRAM throughput % of peak"),
    ("dram__bytes_read.sum.per_second", "DRAM read rate"),
    ("lts__t_sector_hit_rate.pct", "L2 hit rate %"),
    ("sm__warps_active.avg.pct_of_peak_sustained_active", "warps active %"),
    ("launch__registers_per_thread", "registers/thread (launch)"),
    ("launch__block_size", "block size"),
    ("launch__grid_size", "grid size"),
    ("launch__shared_mem_per_block_dynamic", "dynamic smem/block"),
]

UNIT_SCALE = {"byte": 1, "Kbyte": 1e3, "Mbyte": 1e6, "Gbyte": 1e9, "nsecond": 1e-9, "usecond": 1e-6,
              "msecond": 1e-3, "second": 1.0, "ns": 1e-9, "us": 1e-6, "ms": 1e-3, "s": 1.0}


def read_raw(path):
    rows = list(csv.reader(open(path)))
    hi = next(i for i, r in enumerate(rows) if "ID" in r or "Kernel Name" in r)
    header = rows[hi]
    # the raw-page export has a units row (empty ID) under the header; launch lists do not
    has_units = len(rows) > hi + 1 and rows[hi + 1] and rows[hi + 1][0] == ""
    units = rows[hi + 1] if has_units else [""] * len(header)
    data = [r for r in rows[hi + (2 if has_units else 1):] if len(r) == len(header)]
    return header, units, data


def kernel_summary(path, flops=None, peak_tflops=None):
    header, units, data = read_raw(path)
    col = {h: i for i, h in enumerate(header)}
    out = []
    for r in data:
        name = r[col["Kernel Name"]] if "Kernel Name" in col else "?"
        out.append(f"kernel: {name[:110]}")
        vals = {}
        for key, label in KEYS:
            if key in col and r[col[key]] not in ("", "n/a"):
                v, u = r[col[key]].replace(",", ""), units[col[key]]
                vals[key] = (float(v), u)
                out.append(f"  {label:34s} {v} {u}")
        stalls = [(h, r[i]) for h, i in col.items()
                  if h.startswith("smsp__average_warps_issue_stalled_") and h.endswith("_per_issue_active.ratio")
                  and r[i] not in ("", "0")]
        stalls = sorted(((h[len("smsp__average_warps_issue_stalled_"):-len("_per_issue_active.ratio")],
                          float(v.replace(",", ""))) for h, v in stalls), key=lambda x: -x[1])
        if stalls:
            out.append("  warp stall reasons (cycles per issued instruction):")
            for n, v in stalls[:10]:
                out.append(f"    {n:24s} {v:.3f}")
        # local-memory (register spill) traffic, when the capture has it
        for h in ("smsp__sass_inst_executed_op_local_ld.sum", "smsp__sass_inst_executed_op_local_st.sum"):
            if h in col and r[col[h]] not in ("", "n/a"):
                out.append(f"  {h:34s} {r[col[h]]}")
        if "dram__bytes_read.sum" in vals and "dram__bytes_write.sum" in vals:
            rd = vals["dram__bytes_read.sum"][0] * UNIT_SCALE.get(vals["dram__bytes_read.sum"][1], 1)
            wr = vals["dram__bytes_write.sum"][0] * UNIT_SCALE.get(vals["dram__bytes_write.sum"][1], 1)
            out.append(f"traffic_bytes_per_launch: {int(rd + wr)}")
        if flops and "gpu__time_duration.sum" in vals:
            t = vals["gpu__time_duration.sum"][0] * UNIT_SCALE.get(vals["gpu__time_duration.sum"][1], 1)
            tf = flops / t / 1e12
            line = f"  algorithmic {flops:.4e} FLOP / {t * 1e3:.3f} ms = {tf:.1f} TFLOP/s (under ncu)"
            if peak_tflops:
                line += f" = {tf / peak_tflops:.3f} of {peak_tflops} TFLOP/s"
            out.append(line)
    return "\n".join(out)


def launch_summary(path):
    header, units, data = read_raw(path)
    col = {h: i for i, h in enumerate(header)}
    agg = collections.defaultdict(lambda: [0, 0.0])
    for r in data:
        if r[col["Metric Name"]] != "gpu__time_duration.sum":
            continue
        v = float(r[col["Metric Value"]].replace(",", "")) * UNIT_SCALE.get(r[col["Metric Unit"]], 1e-9)
        name = r[col["Kernel Name"]]
        agg[name][0] += 1
        agg[name][1] += v
    tot = sum(t for _, t in agg.values())
    lines = [f"{'launches':>8} {'total ms':>10} {'share':>7}  kernel"]
    for name, (n, t) in sorted(agg.items(), key=lambda x: -x[1][1]):
        lines.append(f"{n:8d} {t * 1e3:10.3f} {100 * t / tot:6.2f}%  {name[:100]}")
    lines.append(f"total {tot * 1e3:.3f} ms over {sum(n for n, _ in agg.values())} launches")
    return "\n".join(lines)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("mode", choices=["kernel", "launches"])
    ap.add_argument("csv")
    ap.add_argument("--flops", type=float)
    ap.add_argument("--peak-tflops", type=float)
    a = ap.parse_args(argv)
    print(kernel_summary(a.csv, a.flops, a.peak_tflops) if a.mode == "kernel" else launch_summary(a.csv))


if __name__ == "__main__":
    sys.exit(main())
