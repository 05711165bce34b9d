"""Multi-GPU parity of the (batch, kv-head) sharding: one process per GPU over NCCL.

Each rank runs the sm_100a kernel on its unit block; the NCCL all-gather of O must
reproduce the single-GPU output bit for bit (the kernel computes every row the same way
whatever the shard). Needs >= 2 GPUs; skipped otherwise. NVLS is turned off (no multicast
objects) so a failing rank cannot leave NVLink faults behind.
"""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

NGPU = torch.cuda.device_count() if torch.cuda.is_available() else 0


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, result_dir):
    import datetime
    import sys

    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (repo, os.path.join(repo, "triton-fa2-forward_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch.distributed as dist

    from fa2.kernel import attention, check_device_errors
    from fa2.shard import sharded_attention
    from oracle.reference import make_qkv

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        ok = True
        for (B, Hq, Hkv, N, D, causal) in [(2, 32, 8, 1024, 128, True), (2, 8, 8, 777, 64, False),
                                            (1, 12, 3, 513, 128, True)]:
            q, k, v = make_qkv(B, Hq, Hkv, N, N, D, torch.bfloat16, seed=5, device=dev)
            full = attention(q, k, v, causal=causal)
            got = sharded_attention(q, k, v, causal=causal, replicate_out=True)
            torch.cuda.synchronize(dev)
            check_device_errors(dev)
            ok = ok and torch.equal(got, full)
        with open(os.path.join(result_dir, f"rank{rank}.txt"), "w") as f:
            f.write("1" if ok else "0")
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(NGPU < 2, reason="needs >= 2 GPUs")
@pytest.mark.parametrize("world", [2] + ([4] if NGPU >= 4 else []) + ([8] if NGPU >= 8 else []))
def test_sharded_allgather_matches_single_gpu(world, tmp_path):
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    for r in range(world):
        assert (tmp_path / f"rank{r}.txt").read_text() == "1", f"rank {r} mismatch"
