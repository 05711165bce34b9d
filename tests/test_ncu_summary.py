"""The counters-only ncu summariser parses Nsight Compute CSV exports (both the raw-page
export of a single kernel and a launch list), as the reference's tests/test_ncu_summary.py
does for its summariser."""

import os
import sys

sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "triton-fa2-forward_b200"))

import ncu_summary  # noqa: E402

RAW = '''"ID","Kernel Name","gpu__time_duration.sum","dram__bytes_read.sum","dram__bytes_write.sum","sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_elapsed","smsp__average_warps_issue_stalled_wait_per_issue_active.ratio","smsp__average_warps_issue_stalled_barrier_per_issue_active.ratio"
"","","us","Mbyte","Mbyte","%","inst","inst"
"0","void fa2::fa2_fwd_kernel<128, 1, 1>(...)","954.24","330.644224","88.282112","59.3","1.555","1.240"
'''

LAUNCHES = '''"ID","Process ID","Process Name","Host Name","Kernel Name","Context","Stream","Block Size","Grid Size","Device","CC","Section Name","Metric Name","Metric Unit","Metric Value"
"0","1","python","h","void fa2::fa2_fwd_kernel<128, 1, 1>(...)","1","7","(384, 1, 1)","(64, 32, 1)","0","10.0","Command line profiler metrics","gpu__time_duration.sum","us","950.5"
"1","1","python","h","void at::fill(...)","1","7","(128, 1, 1)","(1024, 1, 1)","0","10.0","Command line profiler metrics","gpu__time_duration.sum","us","70.0"
"2","1","python","h","void fa2::fa2_fwd_kernel<128, 1, 1>(...)","1","7","(384, 1, 1)","(64, 32, 1)","0","10.0","Command line profiler metrics","gpu__time_duration.sum","ms","0.9495"
'''


def test_kernel_summary(tmp_path):
    p = tmp_path / "raw.csv"
    p.write_text(RAW)
    out = ncu_summary.kernel_summary(str(p), flops=1.0996e12, peak_tflops=1644.8)
    assert "traffic_bytes_per_launch: 418926336" in out
    assert "tensor pipe active" in out and "59.3" in out
    assert out.index("wait") < out.index("barrier")  # stalls sorted by weight
    assert "1152.3 TFLOP/s" in out


def test_launch_summary(tmp_path):
    p = tmp_path / "launches.csv"
    p.write_text(LAUNCHES)
    out = ncu_summary.launch_summary(str(p))
    first = out.splitlines()[1]
    assert "fa2_fwd_kernel" in first and first.split()[0] == "2"
    assert "96.4" in first  # 1900 us of 1970 us


def test_step_trace_summary_reads_stamps():
    """step_trace.summarize turns FA2_TRACE stamps into per-event medians relative to each tile's
    S being seen (synthetic stamps: a 1000-cycle step, events at fixed offsets)."""
    import numpy as np

    import step_trace

    buf = np.zeros((step_trace.UNITS, step_trace.STEPS, 2, step_trace.EVENTS), dtype=np.int64)
    for j in range(20):
        for t in range(2):
            base = 10_000 + 1000 * j + 400 * t
            for e, off in {0: 0, 1: 50, 2: 150, 3: 500, 4: 700, 5: 800, 7: 560, 8: 700, 9: 760, 10: 800,
                           11: 820, 12: 900}.items():
                buf[0, j, t, e] = base + off
            for q in range(4):
                buf[0, j, t, 20 + q] = base + 500 + 10 * q
                buf[0, j, t, 24 + q] = base + 700 + 10 * q
            buf[0, j, 0, 6] = 10_000 + 1000 * j + 300
    text = step_trace.summarize(buf, 0)
    assert "20 K/V steps" in text and "median 1000 cycles" in text
    assert "first P hand-off" in text and "q3: 530 / 730" in text
    assert "tile 1 S seen - tile 0 S seen: 400 cycles" in text
