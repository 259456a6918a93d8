"""Paged decode attention module (drop-in for
``nanovllm_ascend.layers.npu_paged_attention.NpuPagedAttention``,
src/nanovllm_ascend/layers/npu_paged_attention.py:14-100).

``forward(q, key_cache, value_cache, block_tables, context_lens)`` returns a
new [tokens, num_heads, head_dim] tensor like the reference. ``context_lens``
may be the reference's CPU int32 tensor (it is copied to the device) or a
device tensor (the CUDA-graph path). Inside PagedKVCache.deferred_appends()
(the CUDA-graph decode runner) the layer's append is fused into the kernel. Inside a decode-graph capture the
workspace comes from the capturing graph entry, mirroring the per-task
workspace of src/nanovllm_ascend/npu/acl_graph.py:229-242.
"""

from __future__ import annotations

import torch
from torch import nn

from . import ops
from .cuda_graph import PagedAttentionGraphTask, current_decode_graph_entry, record_paged_attention_task
from .paged_kv_cache import take_deferred

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
    def __init__(self, num_heads: int, num_key_value_heads: int, head_dim: int, num_ctas: int = 0):
        super().__init__()
        self.num_heads = num_heads
        self.num_key_value_heads = num_key_value_heads
        self.head_dim = head_dim
        self.scale = head_dim ** -0.5
        self.num_ctas = num_ctas  # 0: one persistent CTA per SM

    def workspace_bytes(self, batch: int) -> int:
        return ops.decode_workspace_bytes(batch, self.num_heads, self.num_key_value_heads, self.head_dim,
                                          self.num_ctas)

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
        entry = current_decode_graph_entry()
        with torch.cuda.device(device):
            if entry is not None:
                workspace = entry.decode_workspace(self)
            else:
                workspace = shared_workspace(device, self.workspace_bytes(total_tokens))
            ctx = context_lens if context_lens.is_cuda else context_lens.to(device=device, dtype=torch.int32)
            tables = block_tables if block_tables.is_cuda else block_tables.to(device)
            # This layer's append, when PagedKVCache.deferred_appends() held it
            # back, is done by the decode kernel itself.
            pending = take_deferred(key_cache)
            if pending is not None and pending[0].shape[0] != total_tokens:
                ops.kv_append(key_cache, value_cache, *pending)  # not one row per sequence: plain append first
                pending = None
            new_key, new_value, slots = pending if pending is not None else (None, None, None)
            ops.paged_decode(output, q.contiguous(), key_cache, value_cache, tables.to(torch.int32),
                             ctx.to(torch.int32), self.scale, workspace, self.num_ctas, new_key=new_key,
                             new_value=new_value, slot_mapping=slots)
        if entry is not None:
            record_paged_attention_task(PagedAttentionGraphTask(
                query=q, key_cache=key_cache, value_cache=value_cache, num_kv_heads=self.num_key_value_heads,
                num_heads=self.num_heads, scale=self.scale, block_tables=block_tables, context_lens=context_lens,
                output=output, workspace=workspace))
        return output
