"""Multi-GPU partitioning of the FA2 forward: one process per GPU, no traffic in the kernel.

The reference is single-GPU (its only parallelism is the CUDA grid, fa2/kernel.py:24-26).
The forward shards naturally by work unit u = b * H_kv + h_kv: a unit owns query heads
[h_kv * G, (h_kv + 1) * G) of batch b and their K/V head, and no unit reads another's K/V.
Rank r of W takes the contiguous unit block [lo, hi) with lo = floor(r * U / W).

In [B, H, N, D] storage with the (b, h) dimensions flattened, a contiguous unit block is a
contiguous slab of q/out (G heads per unit) and of k/v (one head per unit), so a rank's
shard is a plain slice, it runs as a batch-1 problem with (hi - lo) * G query heads and
(hi - lo) K/V heads, and its output rows land at offset lo * G of the flattened output.
The only collective is the optional all-gather of O when the caller wants it replicated
(torch.distributed, NCCL over NVLink on GPUs; any backend works for the host logic).
"""

import torch
import torch.distributed as dist


def shard_bounds(batch, heads_kv, rank, world):
    """Unit range [lo, hi) of `rank` among `world` ranks (units = batch * heads_kv)."""
    if world < 1 or not (0 <= rank < world):
        raise ValueError(f"bad rank {rank} / world {world}")
    units = batch * heads_kv
    return (rank * units) // world, ((rank + 1) * units) // world


def shard_qkv(q, k, v, rank, world):
    """(q, k, v) shards of `rank`: views [1, (hi-lo)*G, N_q, D] and [1, hi-lo, N_kv, D]."""
    B, H_q, N_q, D = q.shape
    H_kv = k.shape[1]
    G = H_q // H_kv
    lo, hi = shard_bounds(B, H_kv, rank, world)
    qs = q.reshape(B * H_q, N_q, D)[lo * G:hi * G].unsqueeze(0)
    ks = k.reshape(B * H_kv, k.shape[2], D)[lo:hi].unsqueeze(0)
    vs = v.reshape(B * H_kv, v.shape[2], D)[lo:hi].unsqueeze(0)
    return qs, ks, vs


def attention_shard(q_shard, k_shard, v_shard, causal=True, sm_scale=None, pack_gqa=None, fn=None):
    """Run the forward on one rank's shard (any callable with attention()'s signature).
    A rank with no units (more ranks than units) gets an empty output."""
    if k_shard.shape[1] == 0:
        return q_shard.new_empty(q_shard.shape)
    if fn is None:
        from .kernel import attention as fn
    return fn(q_shard, k_shard, v_shard, causal=causal, sm_scale=sm_scale, pack_gqa=pack_gqa)


def gather_output(out_shard, batch, heads_q, heads_kv, group=None):
    """All-gather every rank's [1, (hi-lo)*G, N, D] output shard into the full
    [B, H_q, N, D] tensor on every rank (rank order == memory order of the units)."""
    world = dist.get_world_size(group)
    G = heads_q // heads_kv
    _, _, N, D = out_shard.shape
    bounds = [shard_bounds(batch, heads_kv, r, world) for r in range(world)]
    sizes = [(hi - lo) * G for lo, hi in bounds]
    full = torch.empty(batch * heads_q, N, D, dtype=out_shard.dtype, device=out_shard.device)
    mine = out_shard.reshape(-1, N, D).contiguous()
    if len(set(sizes)) == 1:
        dist.all_gather_into_tensor(full, mine, group=group)
    else:
        # Uneven blocks (units % world != 0): gather padded blocks, then compact.
        m = max(sizes)
        padded = torch.zeros(m, N, D, dtype=mine.dtype, device=mine.device)
        padded[: mine.shape[0]] = mine
        buf = torch.empty(world * m, N, D, dtype=mine.dtype, device=mine.device)
        dist.all_gather_into_tensor(buf, padded, group=group)
        off = 0
        for r, s in enumerate(sizes):
            full[off:off + s] = buf[r * m:r * m + s]
            off += s
    return full.view(batch, heads_q, N, D)


def sharded_attention(q, k, v, causal=True, sm_scale=None, pack_gqa=None, replicate_out=False,
                      group=None, fn=None):
    """Forward of the full problem split over the process group: every rank computes its
    unit block; returns the local output shard, or the full output on every rank when
    `replicate_out` (one all-gather). q/k/v may be full tensors or already the same on every
    rank; only the rank's slice is read."""
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    qs, ks, vs = shard_qkv(q, k, v, rank, world)
    out = attention_shard(qs, ks, vs, causal=causal, sm_scale=sm_scale, pack_gqa=pack_gqa, fn=fn)
    if not replicate_out:
        return out
    return gather_output(out, q.shape[0], q.shape[1], k.shape[1], group=group)
