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


# ---------------------------------------------------------------------------
# Token-range sharding: every rank keeps all KV heads for a contiguous range of
# cached positions. The key kernel shares each 16-token block's exact-angle
# RoPE twiddles across the units of a work item, so it runs best with many
# heads per rank; with few heads (8 ranks over 32 KV heads) token ranges keep
# all 32 units on every rank. Each rank's decode gives its range's output and
# softmax row stats, which are all-gathered and merged (merge_shards) into the
# output over the whole context.
# ---------------------------------------------------------------------------
def shard_tokens(n_tokens: int, world: int, rank: int, align: int = 256) -> tuple[int, int]:
    """(t0, t1) of rank `rank`: contiguous ranges of whole `align`-token chunks."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    chunks = -(-n_tokens // align)
    if chunks < world:
        raise ValueError(f"{n_tokens} tokens do not split into {world} ranges of {align}")
    c0 = chunks * rank // world
    c1 = chunks * (rank + 1) // world
    return c0 * align, min(n_tokens, c1 * align)


def gather_shard_partials(o: torch.Tensor, ml: torch.Tensor, o_buf: torch.Tensor,
                          ml_buf: torch.Tensor, group=None, async_op: bool = False):
    """All-gathers each rank's shard output o [B, Hq, D] fp16 and row stats ml
    [B*Hq, 2] fp32 into o_buf [world, B, Hq, D] and ml_buf [world, B*Hq, 2]
    (rank-major), the inputs of kvquant.kernels.merge_shards. Returns the two
    work handles when async_op."""
    import torch.distributed as dist
    h1 = dist.all_gather_into_tensor(o_buf.view(-1, *o.shape[1:]), o.contiguous(), group=group,
                                     async_op=async_op)
    h2 = dist.all_gather_into_tensor(ml_buf.view(-1, 2), ml.contiguous(), group=group,
                                     async_op=async_op)
    return (h1, h2) if async_op else None
