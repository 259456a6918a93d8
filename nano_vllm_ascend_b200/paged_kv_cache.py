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

from contextlib import contextmanager
from typing import Iterator

import torch

from . import ops

# Deferred decode appends, by the data pointer of the layer's key view:
# (cache, layer). PagedAttention takes them to fuse the append into decode.
_DEFERRED: dict[int, tuple["PagedKVCache", int]] = {}


def take_deferred(key_cache: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor] | None:
    """Removes and returns the (key, value, slot_mapping) rows deferred for
    the layer whose key view is ``key_cache``, or None."""
    entry = _DEFERRED.pop(key_cache.data_ptr(), None)
    if entry is None:
        return None
    cache, layer = entry
    return cache._pending.pop(layer, None)


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
        self._deferring = False
        self._pending: dict[int, tuple[torch.Tensor, torch.Tensor, torch.Tensor]] = {}

    @contextmanager
    def deferred_appends(self) -> Iterator["PagedKVCache"]:
        """Decode only: inside the block, write() records each layer's rows
        instead of launching the append, and the decode attention over that
        layer (PagedAttention.forward) writes them inside its own kernel
        (nvk_paged_decode_append) -- one launch per layer instead of two, same
        pool contents and outputs. Rows no attention call took are appended
        when the block exits. Nothing may read the pool between a write() and
        the attention of that layer, which the reference's call order
        (qwen3.py:91-117) guarantees."""
        prev = self._deferring
        self._deferring = True
        try:
            yield self
        finally:
            self._deferring = prev
            if not prev:
                self.flush_pending()

    def flush_pending(self) -> None:
        """Appends every deferred layer's rows now (standalone append kernel)."""
        for layer, (k, v, slots) in list(self._pending.items()):
            _DEFERRED.pop(self.key_cache[layer].data_ptr(), None)
            with torch.cuda.device(self.device):
                ops.kv_append(self.key_cache[layer], self.value_cache[layer], k, v, slots)
        self._pending.clear()

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
        if self._deferring:
            if layer_idx in self._pending:  # a second write before attention: the first one lands now
                k0, v0, s0 = self._pending.pop(layer_idx)
                with torch.cuda.device(self.device):
                    ops.kv_append(self.key_cache[layer_idx], self.value_cache[layer_idx], k0, v0, s0)
            self._pending[layer_idx] = (key_states, value_states, slot_mapping)
            _DEFERRED[self.key_cache[layer_idx].data_ptr()] = (self, layer_idx)
            return
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
