"""Multi-GPU partitioning of the paged-KV path (new: the reference is
single-device, src/nanovllm_ascend/model_runner.py:31).

Two schemes, one process per GPU:

* sequence sharding (decode): rank r serves a contiguous slice of the batch
  with its own BlockManager + PagedKVCache; no collective on the data path.
* KV-head sharding (large-model config): rank r holds KV heads
  [r*KVH/W, (r+1)*KVH/W) and the query heads of those GQA groups; after
  attention the per-rank outputs [B, H/W, D] are all-gathered and laid out as
  [B, H, D] (query-head order) for the output projection.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def sequence_shard(num_seqs: int, world_size: int, rank: int) -> range:
    """Contiguous, balanced slice of ``num_seqs`` sequences for ``rank``."""
    if world_size <= 0 or not 0 <= rank < world_size:
        raise ValueError(f"bad rank {rank} for world size {world_size}")
    base, extra = divmod(num_seqs, world_size)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def token_balanced_shard(lengths: list[int], world_size: int, rank: int) -> list[int]:
    """Indices (ascending) of the sequences ``rank`` decodes when the batch is
    split by context length instead of by position: longest first, each to
    the rank holding the fewest tokens so far (lowest rank on ties). A decode
    step reads every token's K and V once, so equal token totals mean equal
    step times; the ranks' totals differ by at most one sequence's length.
    Deterministic: every rank computes the same assignment."""
    if world_size <= 0 or not 0 <= rank < world_size:
        raise ValueError(f"bad rank {rank} for world size {world_size}")
    totals = [0] * world_size
    mine = []
    for i in sorted(range(len(lengths)), key=lambda j: (-lengths[j], j)):
        r = min(range(world_size), key=lambda k: (totals[k], k))
        totals[r] += lengths[i]
        if r == rank:
            mine.append(i)
    return sorted(mine)


def kv_head_shard(num_heads: int, num_kv_heads: int, world_size: int, rank: int) -> tuple[range, range]:
    """(kv-head range, query-head range) owned by ``rank``."""
    if num_kv_heads % world_size != 0:
        raise ValueError(f"num_kv_heads {num_kv_heads} is not divisible by world size {world_size}")
    if num_heads % num_kv_heads != 0:
        raise ValueError(f"num_heads {num_heads} is not a multiple of num_kv_heads {num_kv_heads}")
    kv_per = num_kv_heads // world_size
    q_per = kv_per * (num_heads // num_kv_heads)
    return range(rank * kv_per, (rank + 1) * kv_per), range(rank * q_per, (rank + 1) * q_per)


def gather_head_shards(local_out: torch.Tensor, group=None, out: torch.Tensor | None = None) -> torch.Tensor:
    """All-gathers [B, Hl, D] shards from every rank into [B, W*Hl, D].

    NCCL path: one ``all_gather_into_tensor`` into a [W, B, Hl, D] buffer
    (capturable in a CUDA graph), then one permuting copy. Other backends
    (gloo, for the CPU tests) use the list form.
    """
    world = dist.get_world_size(group)
    b, hl, d = local_out.shape
    local_out = local_out.contiguous()
    if dist.get_backend(group) == "nccl":
        buf = torch.empty((world, b, hl, d), dtype=local_out.dtype, device=local_out.device)
        dist.all_gather_into_tensor(buf, local_out, group=group)
    else:
        parts = [torch.empty_like(local_out) for _ in range(world)]
        dist.all_gather(parts, local_out, group=group)
        buf = torch.stack(parts, dim=0)
    if out is None:
        out = torch.empty((b, world * hl, d), dtype=local_out.dtype, device=local_out.device)
    out.view(b, world, hl, d).copy_(buf.permute(1, 0, 2, 3))
    return out
