"""KV-head sharding of the decode step across ranks (one process per GPU).

(batch, KV head) units are independent for scores, softmax and p.V, and a
query head reads only its own KV head, so rank r owns the contiguous KV heads
[h0, h0 + n) of every layer together with their query heads, runs the decode
kernels on that shard, and the per-head outputs are gathered with one
all-gather per layer. The key calibration (per channel) is local to the shard;
the value statistics are per token over all channels, so each rank quantizes
its value shard from the full v_proj row (quantize_values with h0/n_heads).
"""
from __future__ import annotations

import torch


def shard_heads(n_kv_heads: int, world: int, rank: int) -> tuple[int, int]:
    """(h0, n) of rank `rank`: equal contiguous blocks of KV heads."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if n_kv_heads % world:
        raise ValueError(f"{n_kv_heads} KV heads do not split over {world} ranks")
    n = n_kv_heads // world
    return rank * n, n


def gather_buffer(local_out: torch.Tensor, world: int) -> torch.Tensor:
    """Receive buffer [world * B, Hq_local, D] (rank-major) for gather_head_outputs."""
    B = local_out.shape[0]
    return torch.empty((world * B, *local_out.shape[1:]), dtype=local_out.dtype,
                       device=local_out.device)


def gather_head_outputs(local_out: torch.Tensor, buf: torch.Tensor, group=None,
                        async_op: bool = False):
    """All-gathers each rank's [B, Hq_local, D] decode output into buf (rank-major).

    Returns the work handle when async_op, else None. full_heads(buf, world)
    turns the buffer into the [B, Hq, D] output in global query-head order.
    """
    import torch.distributed as dist
    return dist.all_gather_into_tensor(buf, local_out.contiguous(), group=group,
                                       async_op=async_op)


def full_heads(buf: torch.Tensor, world: int) -> torch.Tensor:
    """[world * B, Hq_local, D] -> [B, world * Hq_local, D] (global query-head order)."""
    wb, hl, D = buf.shape
    B = wb // world
    return buf.view(world, B, hl, D).permute(1, 0, 2, 3).reshape(B, world * hl, D)
