"""Paged decode attention module (drop-in for
``nanovllm_ascend.layers.npu_paged_attention.NpuPagedAttention``,
src/nanovllm_ascend/layers/npu_paged_attention.py:14-100).

``forward(q, key_cache, value_cache, block_tables, context_lens)`` returns a
new [tokens, num_heads, head_dim] tensor like the reference. ``context_lens``
may be the reference's CPU int32 tensor (it is copied to the device, and its
values pick the split-K granularity) or a device tensor (the CUDA-graph path).
Inside a decode-graph capture the split-K workspace and split policy come
from the capturing graph entry, mirroring the per-task workspace of
src/nanovllm_ascend/npu/acl_graph.py:229-242.
"""

from __future__ import annotations

import math

import torch
from torch import nn

from . import ops
from .cuda_graph import PagedAttentionGraphTask, current_decode_graph_entry, record_paged_attention_task

_NUM_SMS: dict[int, int] = {}
_WORKSPACES: dict[int, torch.Tensor] = {}


def num_sms(device: torch.device) -> int:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _NUM_SMS:
        _NUM_SMS[idx] = torch.cuda.get_device_properties(idx).multi_processor_count
    return _NUM_SMS[idx]


def shared_workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """Eager-mode split-K workspace, one per device, grown (zero-filled) on demand.

    Calls ordered on one stream may share it: each decode call returns its
    arrival counters to zero.
    """
    idx = device.index if device.index is not None else torch.cuda.current_device()
    ws = _WORKSPACES.get(idx)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _WORKSPACES[idx] = ws
    return ws


class PagedAttention(nn.Module):
    def __init__(self, num_heads: int, num_key_value_heads: int, head_dim: int,
                 blocks_per_split: int | None = None):
        super().__init__()
        self.num_heads = num_heads
        self.num_key_value_heads = num_key_value_heads
        self.head_dim = head_dim
        self.scale = head_dim ** -0.5
        self.blocks_per_split = blocks_per_split

    def split_policy(self, device: torch.device, batch: int, block_size: int, block_tables: torch.Tensor,
                     context_lens: torch.Tensor) -> tuple[int, int]:
        width = block_tables.shape[1]
        if self.blocks_per_split is not None:
            bps = self.blocks_per_split
        else:
            total = None
            if not context_lens.is_cuda:
                total = int(((context_lens.to(torch.int64) + block_size - 1) // block_size).sum())
            bps = ops.choose_blocks_per_split(self.num_key_value_heads, width, total, batch, num_sms(device))
        return bps, math.ceil(width / bps)

    def forward(
        self,
        q: torch.Tensor,
        key_cache: torch.Tensor,
        value_cache: torch.Tensor,
        block_tables: torch.Tensor,
        context_lens: torch.Tensor,
    ) -> torch.Tensor:
        total_tokens, num_heads, head_dim = q.shape
        if num_heads != self.num_heads or head_dim != self.head_dim:
            raise ValueError(f"query shape mismatch: got {tuple(q.shape)}")
        output = torch.empty_like(q)
        if total_tokens == 0:
            return output
        device = q.device
        block_size = key_cache.shape[1]
        entry = current_decode_graph_entry()
        if entry is not None:
            bps, max_splits, workspace = entry.decode_plan(self, block_size, block_tables, context_lens)
        else:
            bps, max_splits = self.split_policy(device, total_tokens, block_size, block_tables, context_lens)
            workspace = shared_workspace(
                device, ops.decode_workspace_bytes(total_tokens, num_heads, self.num_key_value_heads, head_dim,
                                                   max_splits))
        ctx = context_lens if context_lens.is_cuda else context_lens.to(device=device, dtype=torch.int32)
        tables = block_tables if block_tables.is_cuda else block_tables.to(device)
        with torch.cuda.device(device):
            ops.paged_decode(output, q.contiguous(), key_cache, value_cache, tables.to(torch.int32),
                             ctx.to(torch.int32), self.scale, workspace, bps, max_splits)
        if entry is not None:
            record_paged_attention_task(PagedAttentionGraphTask(
                query=q, key_cache=key_cache, value_cache=value_cache, num_kv_heads=self.num_key_value_heads,
                num_heads=self.num_heads, scale=self.scale, block_tables=block_tables, context_lens=context_lens,
                output=output, workspace=workspace, blocks_per_split=bps))
        return output
