"""KV-pool sizing from free HBM (src/nanovllm_ascend/model_runner.py:113-125)."""

from __future__ import annotations

import torch


def bytes_per_block(num_layers: int, block_size: int, num_kv_heads: int, head_dim: int,
                    dtype: torch.dtype = torch.bfloat16) -> int:
    """K and V bytes of one pool block across all layers."""
    return 2 * num_layers * block_size * num_kv_heads * head_dim * torch.tensor([], dtype=dtype).element_size()


def num_blocks_for_budget(free_bytes: int, total_bytes: int, memory_utilization: float, num_layers: int,
                          block_size: int, num_kv_heads: int, head_dim: int,
                          dtype: torch.dtype = torch.bfloat16) -> int:
    """(total * utilization - used) // bytes_per_block, as the reference sizes its pool."""
    used = total_bytes - free_bytes
    budget = int(total_bytes * memory_utilization) - used
    return max(0, budget // bytes_per_block(num_layers, block_size, num_kv_heads, head_dim, dtype))


def num_blocks_from_memory(memory_utilization: float, num_layers: int, block_size: int, num_kv_heads: int,
                           head_dim: int, dtype: torch.dtype = torch.bfloat16,
                           device: torch.device | str | None = None) -> int:
    free, total = torch.cuda.mem_get_info(device)
    return num_blocks_for_budget(free, total, memory_utilization, num_layers, block_size, num_kv_heads, head_dim,
                                 dtype)
