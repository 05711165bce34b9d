"""Multi-rank host logic of the (batch, kv-head) sharding, on CPU with the gloo backend
(world_size 2 and 4 processes). The per-shard compute is the oracle (CPU), so what is
tested is the partitioning, the shard slicing and the all-gather that reassembles O."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from fa2.shard import gather_output, shard_bounds, shard_qkv, sharded_attention


def test_bounds_cover_every_unit_once():
    for batch, hkv in ((2, 8), (1, 3), (16, 8), (4, 16), (1, 1)):
        units = batch * hkv
        for world in (1, 2, 3, 4, 8):
            seen = []
            for r in range(world):
                lo, hi = shard_bounds(batch, hkv, r, world)
                assert 0 <= lo <= hi <= units
                seen.extend(range(lo, hi))
            assert seen == list(range(units))
    with pytest.raises(ValueError):
        shard_bounds(2, 8, 2, 2)


def test_headline_shards_are_even_and_contiguous():
    # headline config: 16 units -> 2 per rank at 8 GPUs; a shard is a contiguous slab
    q = torch.zeros(2, 32, 64, 128)
    k = torch.zeros(2, 8, 64, 128)
    for world in (1, 2, 4, 8):
        for r in range(world):
            qs, ks, vs = shard_qkv(q, k, k, r, world)
            assert qs.shape == (1, 64 // world, 64, 128) and ks.shape == (1, 16 // world, 64, 128)
            assert qs.is_contiguous() and ks.is_contiguous()


def _oracle_fn(q, k, v, causal=True, sm_scale=None, pack_gqa=None):
    from oracle.reference import naive_attention
    return naive_attention(q, k, v, causal=causal, sm_scale=sm_scale)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, shapes, result_path):
    import sys
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (repo, os.path.join(repo, "triton-fa2-forward_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    from oracle.reference import make_qkv, naive_attention

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        worst = 0.0
        for B, Hq, Hkv, N, causal in shapes:
            q, k, v = make_qkv(B, Hq, Hkv, N, N, 32, torch.float64, seed=3)
            full = sharded_attention(q, k, v, causal=causal, replicate_out=True, fn=_oracle_fn)
            ref = naive_attention(q, k, v, causal=causal)
            worst = max(worst, (full - ref).abs().max().item())
            local = sharded_attention(q, k, v, causal=causal, replicate_out=False, fn=_oracle_fn)
            lo, hi = shard_bounds(B, Hkv, rank, world)
            G = Hq // Hkv
            expect = ref.reshape(B * Hq, N, 32)[lo * G:hi * G]
            assert local[0].shape == expect.shape
            if expect.numel():
                worst = max(worst, (local[0] - expect).abs().max().item())
        if rank == 0:
            with open(result_path, "w") as f:
                f.write(repr(worst))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_forward_gloo(world, tmp_path):
    shapes = [(2, 8, 2, 24, True), (1, 6, 3, 17, False), (3, 4, 4, 9, True)]  # even and uneven
    out = tmp_path / "worst.txt"
    mp.start_processes(_worker, args=(world, _free_port(), shapes, str(out)), nprocs=world,
                       join=True, start_method="spawn")
    assert float(out.read_text()) < 1e-12


def _gather_worker(rank, world, port, result_path):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        B, Hq, Hkv, N, D = 1, 6, 3, 4, 8  # 3 units over 2 ranks: uneven gather path
        lo, hi = shard_bounds(B, Hkv, rank, world)
        G = Hq // Hkv
        shard = torch.arange((hi - lo) * G * N * D, dtype=torch.float32).view(1, (hi - lo) * G, N, D) + 1000 * rank
        full = gather_output(shard, B, Hq, Hkv)
        ok = full.shape == (B, Hq, N, D)
        for r in range(world):
            l2, h2 = shard_bounds(B, Hkv, r, world)
            exp = torch.arange((h2 - l2) * G * N * D, dtype=torch.float32).view((h2 - l2) * G, N, D) + 1000 * r
            ok = ok and torch.equal(full.view(B * Hq, N, D)[l2 * G:h2 * G], exp)
        if rank == 0:
            with open(result_path, "w") as f:
                f.write("1" if ok else "0")
    finally:
        dist.destroy_process_group()


def test_uneven_gather_gloo(tmp_path):
    out = tmp_path / "ok.txt"
    mp.start_processes(_gather_worker, args=(2, _free_port(), str(out)), nprocs=2, join=True,
                       start_method="spawn")
    assert out.read_text() == "1"
