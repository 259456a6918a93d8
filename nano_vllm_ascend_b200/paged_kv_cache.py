"""Physical KV pool with a CUDA append (drop-in for
``nanovllm_ascend.npu.paged_kv_cache.PagedKVCache``,
src/nanovllm_ascend/npu/paged_kv_cache.py:6-72).

Layout (unchanged from the reference, so slot numbers and per-layer views are
interchangeable): ``key_cache``/``value_cache`` are
[num_layers, num_blocks, block_size, num_kv_heads, head_dim]. One layer is a
contiguous [num_blocks * block_size, num_kv_heads, head_dim] row array whose
row s is token slot s.

A slot outside the pool raises ``IndexError`` as the reference's
``index_copy_`` does: at once when ``slot_mapping`` is a host tensor,
otherwise through the device's error word (``device_errors``) on a following
call or at ``device_errors.check_errors()``.
"""

from __future__ import annotations

from contextlib import contextmanager
from typing import Iterator

import torch

from . import device_errors, ops

# Caches inside deferred_appends(); PagedAttention asks them for the rows
# held back for the layer it attends over (a decode step touches one or two).
_DEFERRING: list["PagedKVCache"] = []


def take_deferred(key_cache: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor] | None:
    """Removes and returns the (key, value, slot_mapping) rows deferred for the
    layer whose key view is ``key_cache``, or None. The owner is found by
    address: the deferring cache whose key pool holds ``key_cache`` as one
    whole layer."""
    for cache in _DEFERRING:
        layer = cache.layer_of(key_cache)
        if layer is not None:
            return cache._pending.pop(layer, None)
    return None


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
        # Zero-filled (the reference allocates with torch.empty): the attention
        # kernels stage whole tiles, so rows of a block past a sequence's end are
        # read with probability 0, and 0 * V must stay 0 -- a never-written row
        # holding a NaN bit pattern would make it NaN.
        self.key_cache = torch.zeros(shape, dtype=dtype, device=self.device)
        self.value_cache = torch.zeros(shape, dtype=dtype, device=self.device)
        self._deferring = False
        self._pending: dict[int, tuple[torch.Tensor, torch.Tensor, torch.Tensor]] = {}

    @contextmanager
    def deferred_appends(self) -> Iterator["PagedKVCache"]:
        """Decode only: inside the block, write() records each layer's rows
        instead of launching the append, and the decode attention over that
        layer (PagedAttention.forward) writes them inside its own kernel
        (nvk_paged_decode_append) -- one launch per layer instead of two, same
        pool contents and outputs. Nothing may read the pool between a write()
        and the attention of that layer, which the reference's call order
        (qwen3.py:91-117) guarantees; rows that no attention call took are a
        broken contract: they are appended when the block exits and the exit
        raises RuntimeError."""
        prev = self._deferring
        self._deferring = True
        if not prev:
            _DEFERRING.append(self)
        try:
            yield self
        finally:
            self._deferring = prev
            if not prev:
                _DEFERRING.remove(self)
                left = sorted(self._pending)
                self.flush_pending()
                if left:
                    raise RuntimeError(f"deferred KV append of layer(s) {left} was not consumed by a decode "
                                       "attention call inside deferred_appends() (appended at exit)")

    def layer_of(self, key_view: torch.Tensor) -> int | None:
        """The layer whose key view ``key_view`` is (same storage address and
        shape as ``key_cache[layer]``), or None."""
        layer_bytes = self.key_cache[0].numel() * self.key_cache.element_size()
        off = key_view.data_ptr() - self.key_cache.data_ptr()
        if off < 0 or off % layer_bytes or off // layer_bytes >= self.num_layers:
            return None
        if key_view.shape != self.key_cache.shape[1:]:
            return None
        return off // layer_bytes

    def flush_pending(self) -> None:
        """Appends every deferred layer's rows now (standalone append kernel)."""
        pending, self._pending = self._pending, {}
        for layer, (k, v, slots) in pending.items():
            self._append(layer, k, v, slots)

    def _append(self, layer: int, key: torch.Tensor, value: torch.Tensor, slots: torch.Tensor) -> None:
        with torch.cuda.device(self.device):
            errors = device_errors.state(self.device)
            errors.raise_if_flagged()
            ops.kv_append(self.key_cache[layer], self.value_cache[layer], key, value, slots,
                          error_word=errors.word)
            errors.launched()

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
        if not slot_mapping.is_cuda:
            lo, hi = int(slot_mapping.min()), int(slot_mapping.max())
            if lo < 0 or hi >= self.num_blocks * self.block_size:
                bad = lo if lo < 0 else hi
                raise IndexError(f"index_copy_(): index {bad} is out of bounds for dimension 0 with size "
                                 f"{self.num_blocks * self.block_size}")
        slot_mapping = slot_mapping.to(device=self.device, dtype=torch.long)
        key_states = _packed_rows(key_states.to(self.device))
        value_states = _packed_rows(value_states.to(self.device))
        if self._deferring:
            if layer_idx in self._pending:  # a second write before attention: the first one lands now
                self._append(layer_idx, *self._pending.pop(layer_idx))
            self._pending[layer_idx] = (key_states, value_states, slot_mapping)
            return
        self._append(layer_idx, key_states, value_states, slot_mapping)

    def get_physical_cache(self, layer_idx: int) -> tuple[torch.Tensor, torch.Tensor]:
        return self.key_cache[layer_idx], self.value_cache[layer_idx]


def _packed_rows(t: torch.Tensor) -> torch.Tensor:
    """Keeps strided token rows (e.g. a slice of a fused QKV output) as they are;
    copies only when heads/dims are not packed or rows are misaligned."""
    if t.stride(2) == 1 and t.stride(1) == t.shape[2] and (t.stride(0) * t.element_size()) % 16 == 0 \
            and t.data_ptr() % 16 == 0:
        return t
    return t.contiguous()
