"""Physical KV pool with a CUDA append (drop-in for
``nanovllm_ascend.npu.paged_kv_cache.PagedKVCache``,
src/nanovllm_ascend/npu/paged_kv_cache.py:6-72).

Layout (unchanged from the reference, so slot numbers and per-layer views are
interchangeable): ``key_cache``/``value_cache`` are
[num_layers, num_blocks, block_size, num_kv_heads, head_dim]. One layer is a
contiguous [num_blocks * block_size, num_kv_heads, head_dim] row array whose
row s is token slot s.
"""

from __future__ import annotations

import torch

from . import ops


class PagedKVCache:
    def __init__(
        self,
        num_layers: int,
        num_blocks: int,
        block_size: int,
        num_kv_heads: int,
        head_dim: int,
        dtype: torch.dtype,
        device: torch.device | str,
    ):
        self.num_layers = num_layers
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.dtype = dtype
        self.device = torch.device(device)
        shape = (num_layers, num_blocks, block_size, num_kv_heads, head_dim)
        self.key_cache = torch.empty(shape, dtype=dtype, device=self.device)
        self.value_cache = torch.empty(shape, dtype=dtype, device=self.device)

    @property
    def bytes_per_block(self) -> int:
        """K + V bytes of one block across all layers (model_runner.py:117-124)."""
        return 2 * self.num_layers * self.block_size * self.num_kv_heads * self.head_dim * self.key_cache.element_size()

    def write(
        self,
        layer_idx: int,
        key_states: torch.Tensor,
        value_states: torch.Tensor,
        slot_mapping: torch.Tensor,
    ) -> None:
        """Appends rows: pool[layer].view(-1, KVH, D)[slot_mapping[t]] = key_states[t] (and V)."""
        total_tokens, num_kv_heads, head_dim = key_states.shape
        if num_kv_heads != self.num_kv_heads or head_dim != self.head_dim:
            raise ValueError(f"kv shape mismatch: got {tuple(key_states.shape)}")
        if slot_mapping.numel() != total_tokens:
            raise ValueError(f"slot_mapping numel {slot_mapping.numel()} != total_tokens {total_tokens}")
        if value_states.shape != key_states.shape:
            raise ValueError(f"kv shape mismatch: got {tuple(value_states.shape)}")
        if total_tokens == 0:
            return
        slot_mapping = slot_mapping.to(device=self.device, dtype=torch.long)
        key_states = _packed_rows(key_states.to(self.device))
        value_states = _packed_rows(value_states.to(self.device))
        with torch.cuda.device(self.device):
            ops.kv_append(self.key_cache[layer_idx], self.value_cache[layer_idx], key_states, value_states,
                          slot_mapping)

    def get_physical_cache(self, layer_idx: int) -> tuple[torch.Tensor, torch.Tensor]:
        return self.key_cache[layer_idx], self.value_cache[layer_idx]


def _packed_rows(t: torch.Tensor) -> torch.Tensor:
    """Keeps strided token rows (e.g. a slice of a fused QKV output) as they are;
    copies only when heads/dims are not packed or rows are misaligned."""
    if t.stride(2) == 1 and t.stride(1) == t.shape[2] and (t.stride(0) * t.element_size()) % 16 == 0 \
            and t.data_ptr() % 16 == 0:
        return t
    return t.contiguous()
