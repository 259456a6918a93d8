"""Paged decode attention module (drop-in for
``nanovllm_ascend.layers.npu_paged_attention.NpuPagedAttention``,
src/nanovllm_ascend/layers/npu_paged_attention.py:14-100).

``forward(q, key_cache, value_cache, block_tables, context_lens)`` returns a
new [tokens, num_heads, head_dim] tensor like the reference. ``context_lens``
may be the reference's CPU int32 tensor (it is copied to the device) or a
device tensor (the CUDA-graph path). Inside PagedKVCache.deferred_appends()
(the CUDA-graph decode runner) the layer's append is fused into the kernel.
While DecodeGraphRunner records a batch size, the split-K workspace is that
graph's own (cuda_graph.graph_workspace), as the reference gives each
captured task its workspace (src/nanovllm_ascend/npu/acl_graph.py:229-242).

Bad metadata raises like the reference: a CPU ``context_lens`` longer than
its block-table row raises ``RuntimeError("missing block ...")`` before the
launch (block_manager.py:194-205); what only the device can see (a block id
outside the pool, a device ``context_lens`` too long, a fused-append slot
that is not the sequence's last position) is reported through the decode
workspace's error word and raised by ``device_errors`` on a following call
or by ``device_errors.check_errors()``.
"""

from __future__ import annotations

import torch
from torch import nn

from . import device_errors, ops
from .cuda_graph import graph_workspace
from .paged_kv_cache import take_deferred

_NUM_SMS: dict[int, int] = {}
_WORKSPACES: dict[int, torch.Tensor] = {}
_SHAPES: dict[int, tuple] = {}  # per device: the shape of the last call on its workspace


def num_sms(device: torch.device) -> int:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _NUM_SMS:
        _NUM_SMS[idx] = torch.cuda.get_device_properties(idx).multi_processor_count
    return _NUM_SMS[idx]


def shared_workspace(device: torch.device, nbytes: int, shape: tuple = ()) -> torch.Tensor:
    """Eager-mode split-K workspace, one per device, grown (zero-filled) on demand.

    Calls ordered on one stream may share it: each decode call returns its
    arrival tickets to zero. Where the tickets lie depends on the call's
    ``shape`` (batch, heads, KV heads, CTAs), and a call of another shape
    would find the previous call's partial results there, so the workspace
    is zeroed again, in stream order, whenever the shape changes.
    """
    idx = device.index if device.index is not None else torch.cuda.current_device()
    ws = _WORKSPACES.get(idx)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _WORKSPACES[idx] = ws
    elif _SHAPES.get(idx) != shape:
        ws[:nbytes].zero_()
    _SHAPES[idx] = shape
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
        if not context_lens.is_cuda and context_lens.numel() and block_tables.dim() == 2:
            longest = int(context_lens.max())
            if longest > block_tables.shape[1] * key_cache.shape[1]:
                raise RuntimeError(f"missing block: context length {longest} exceeds the "
                                   f"{block_tables.shape[1]}-block table")
        with torch.cuda.device(device):
            errors = device_errors.state(device)
            errors.raise_if_flagged()
            workspace = graph_workspace(self, total_tokens)
            if workspace is not None:
                word = None  # the graph runner reads its slot's word after each replay
            else:
                workspace = shared_workspace(device, self.workspace_bytes(total_tokens),
                                             (total_tokens, self.num_heads, self.num_key_value_heads, self.num_ctas))
                word = errors.watch("paged decode", workspace)
            ctx = context_lens if context_lens.is_cuda else context_lens.to(device=device, dtype=torch.int32)
            tables = block_tables if block_tables.is_cuda else block_tables.to(device)
            # This layer's append, when PagedKVCache.deferred_appends() held it
            # back, is done by the decode kernel itself.
            pending = take_deferred(key_cache)
            if pending is not None and pending[0].shape[0] != total_tokens:
                # not one row per sequence: plain append first
                ops.kv_append(key_cache, value_cache, *pending, error_word=errors.word)
                errors.launched()
                pending = None
            new_key, new_value, slots = pending if pending is not None else (None, None, None)
            ops.paged_decode(output, q.contiguous(), key_cache, value_cache, tables.to(torch.int32),
                             ctx.to(torch.int32), self.scale, workspace, self.num_ctas, new_key=new_key,
                             new_value=new_value, slot_mapping=slots)
            if word is not None:
                errors.launched(word)
        return output
