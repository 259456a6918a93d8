"""Block pool, per-sequence block tables, slot mapping and prefix-cache reuse.

Drop-in for ``nanovllm_ascend.npu.block_manager`` (src/nanovllm_ascend/npu/
block_manager.py): same classes, methods, arguments, return values and error
types, producing bit-identical block tables, context lengths and slot
mappings for the same call sequence. The observable rules it keeps:

* allocation pops the FRONT of the free queue (block_manager.py:83-93); a
  released block goes to the BACK (:101-107); ``free_slot`` releases a table
  in reverse order (:181-185); retaining a free cached block removes it from
  wherever it sits in the queue (:95-99);
* a full block is keyed by its exact token ids chained to its parent block's
  key (:57-65); lookup returns the first block cached under a key (:136-152);
  reusing a physical block forgets its key (:76-81, :89);
* slot = block_table[pos // block_size] * block_size + pos % block_size, with
  ``RuntimeError`` for a missing block (:194-205).

Internals are new: the free queue is an insertion-ordered dict (O(1) pop-front,
push-back and removal by id instead of list.pop(0)/list.remove), and chain
keys are interned as integers with reference counts, so hashing a block costs
O(block_size) whatever its depth in the chain; a key lives exactly as long as
a block or a child key refers to it, which keeps lookups identical to keying
by the full nested content. By default the keys, the key -> blocks map and
the longest-prefix walk run in C++ (``nvk_prefix_*`` in libnvk_paged.so);
``native_prefix=False`` keeps the same rules in Python. Block tables are built
with one host-to-device copy instead of one per row.
"""

from __future__ import annotations

import ctypes
import math
from collections import OrderedDict
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib

ChainKey = int


@dataclass
class PagedKVCacheMetadata:
    """Per-step attention metadata (block_manager.py:12-20).

    block_tables: int32 [batch, max_blocks] on the manager's device, zero padded
      (0 is a valid block id: kernels bound reads by context_lens).
    context_lens: int32 [batch] on the CPU (the reference keeps it there);
      includes the tokens appended this step.
    slot_mapping: int64 [tokens] on the manager's device.
    """

    block_tables: torch.Tensor
    context_lens: torch.Tensor
    slot_mapping: torch.Tensor
    actual_seq_lengths_q: list[int] | None = None
    actual_seq_lengths_kv: list[int] | None = None
    query_lens: list[int] | None = None
    use_paged_prefill: bool = False


@dataclass
class BlockState:
    block_id: int
    ref_count: int = 0
    block_hash: ChainKey | None = None


class _FreeQueue:
    """FIFO of free block ids with O(1) pop-front, push-back and removal by id."""

    def __init__(self, ids) -> None:
        self._q: OrderedDict[int, None] = OrderedDict.fromkeys(int(i) for i in ids)

    def pop_front(self) -> int:
        return self._q.popitem(last=False)[0]

    def push_back(self, block_id: int) -> None:
        self._q[block_id] = None

    def remove(self, block_id: int) -> None:
        del self._q[block_id]

    def __len__(self) -> int:
        return len(self._q)

    def __iter__(self):
        return iter(self._q)


class _ChainKeys:
    """Interns (parent key, token tuple) pairs as integer keys.

    A key's reference count is the number of blocks that carry it plus the
    number of interned child keys whose parent it is; at zero it is dropped.
    Two chains get the same key iff their full token content is equal.
    """

    def __init__(self) -> None:
        self._ids: dict[tuple[ChainKey | None, tuple[int, ...]], ChainKey] = {}
        self._entries: dict[ChainKey, list] = {}  # key -> [(parent, tokens), refcount]
        self._next = 0

    def find(self, parent: ChainKey | None, tokens: tuple[int, ...]) -> ChainKey | None:
        return self._ids.get((parent, tokens))

    def acquire(self, parent: ChainKey | None, tokens: tuple[int, ...]) -> ChainKey:
        spec = (parent, tokens)
        key = self._ids.get(spec)
        if key is None:
            key = self._next
            self._next += 1
            self._ids[spec] = key
            self._entries[key] = [spec, 0]
            if parent is not None:
                self._entries[parent][1] += 1
        self._entries[key][1] += 1
        return key

    def release(self, key: ChainKey) -> None:
        while key is not None:
            entry = self._entries[key]
            entry[1] -= 1
            if entry[1] > 0:
                return
            spec = entry[0]
            del self._entries[key]
            del self._ids[spec]
            key = spec[0]

    def clear(self) -> None:
        self._ids.clear()
        self._entries.clear()

    def __len__(self) -> int:
        return len(self._entries)


def _token_array(token_ids) -> np.ndarray:
    if isinstance(token_ids, torch.Tensor):
        token_ids = token_ids.detach().cpu().numpy()
    return np.ascontiguousarray(np.asarray(token_ids, dtype=np.int64).reshape(-1))


class _NativePrefixIndex:
    """The prefix-cache keys in C++ (nvk_prefix_*): same rules as _ChainKeys
    plus the key -> cached-blocks map and the per-block keys."""

    def __init__(self, num_blocks: int, block_size: int) -> None:
        self._lib = _lib.load()
        handle = ctypes.c_void_p()
        _lib.call("nvk_prefix_create", num_blocks, block_size, ctypes.byref(handle))
        self._h = handle

    def __del__(self) -> None:
        if getattr(self, "_h", None) is not None and self._h.value:
            self._lib.nvk_prefix_destroy(self._h)
            self._h = None

    def find_longest(self, token_ids, max_blocks: int) -> list[int]:
        if max_blocks <= 0:
            return []
        tokens = _token_array(token_ids)
        out = np.zeros(max_blocks, dtype=np.int32)
        count = ctypes.c_int(0)
        _lib.call("nvk_prefix_find_longest", self._h, tokens.ctypes.data, tokens.size, max_blocks, out.ctypes.data,
                  ctypes.byref(count))
        return [int(b) for b in out[: count.value]]

    def cache_blocks(self, table: list[int], num_cached: int, num_full: int, token_ids) -> None:
        tokens = _token_array(token_ids)
        tab = np.ascontiguousarray(np.asarray(table, dtype=np.int32))
        _lib.call("nvk_prefix_cache_blocks", self._h, tab.ctypes.data, tab.size, num_cached, num_full,
                  tokens.ctypes.data, tokens.size)

    def forget(self, block_id: int) -> None:
        _lib.call("nvk_prefix_forget_block", self._h, block_id)

    def key(self, block_id: int) -> int | None:
        k = int(self._lib.nvk_prefix_block_key(self._h, block_id))
        return None if k < 0 else k

    def clear(self) -> None:
        _lib.call("nvk_prefix_clear", self._h)

    def num_cached_keys(self) -> int:
        return int(self._lib.nvk_prefix_num_cached_keys(self._h))

    def __len__(self) -> int:  # interned keys (cached or parents of cached ones)
        return int(self._lib.nvk_prefix_num_keys(self._h))


class BlockManager:
    """Unified block pool for runtime allocation and prefix-cache reuse.

    Prefix-cached blocks stay in the free queue when their reference count
    reaches zero; their key is forgotten only when the physical block is
    handed out again.
    """

    def __init__(self, num_blocks: int, block_size: int, device: torch.device | str, *,
                 native_prefix: bool = True):
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.device = device
        self.blocks = [BlockState(block_id=i) for i in range(num_blocks)]
        self._free = _FreeQueue(range(num_blocks))
        self._native = _NativePrefixIndex(num_blocks, block_size) if native_prefix else None
        self._keys = self._native if native_prefix else _ChainKeys()
        self._cached: dict[ChainKey, list[int]] = {}
        self.block_tables: dict[int, list[int]] = {}
        self.seq_lens: dict[int, int] = {}

    # ------------------------------------------------------------ free queue --
    @property
    def free_block_ids(self) -> list[int]:
        """Snapshot of the free queue, front first."""
        return list(self._free)

    @free_block_ids.setter
    def free_block_ids(self, ids) -> None:
        """Replaces the free queue order (e.g. a seeded permutation of the pool)."""
        self._free = _FreeQueue(ids)

    def num_free_blocks(self) -> int:
        return len(self._free)

    # ------------------------------------------------------------ block keys --
    def _block_tokens(self, token_ids, block_idx: int) -> tuple[int, ...]:
        start = block_idx * self.block_size
        return tuple(int(v) for v in token_ids[start:start + self.block_size].tolist())

    def _forget_key(self, block_id: int) -> None:
        block = self.blocks[block_id]
        if self._native is not None:
            if block.block_hash is not None:
                self._native.forget(block_id)
                block.block_hash = None
            return
        key = block.block_hash
        if key is None:
            return
        holders = self._cached[key]
        holders.remove(block_id)
        if not holders:
            del self._cached[key]
        self._keys.release(key)
        block.block_hash = None

    # ------------------------------------------------------- ref counting --
    def _alloc_block(self) -> int:
        if len(self._free) == 0:
            raise RuntimeError("BlockManager out of free blocks")
        block_id = self._free.pop_front()
        self._forget_key(block_id)
        block = self.blocks[block_id]
        if block.ref_count != 0:
            raise RuntimeError(f"block {block_id} is not free")
        block.ref_count = 1
        return block_id

    def _retain_block(self, block_id: int) -> None:
        block = self.blocks[block_id]
        if block.ref_count == 0:
            self._free.remove(block_id)
        block.ref_count += 1

    def _release_block(self, block_id: int) -> None:
        block = self.blocks[block_id]
        if block.ref_count <= 0:
            raise RuntimeError(f"block {block_id} ref_count underflow")
        block.ref_count -= 1
        if block.ref_count == 0:
            self._free.push_back(block_id)

    def _num_required_blocks(self, end_pos: int) -> int:
        return 0 if end_pos <= 0 else math.ceil(end_pos / self.block_size)

    # --------------------------------------------------------- sequences --
    def _init_slot(self, slot: int, start_pos: int, prefix_block_ids: list[int]) -> None:
        if slot in self.block_tables:
            return
        table = [int(b) for b in (prefix_block_ids or [])]
        for block_id in table:
            self._retain_block(block_id)
        self.block_tables[slot] = table
        self.seq_lens[slot] = start_pos

    def ensure_blocks(self, slot: int, end_pos: int) -> None:
        table = self.block_tables[slot]
        need = self._num_required_blocks(end_pos)
        while len(table) < need:
            table.append(self._alloc_block())

    def free_slot(self, slot: int) -> None:
        table = self.block_tables.pop(slot, [])
        self.seq_lens.pop(slot, None)
        for block_id in reversed(table):
            self._release_block(block_id)

    # ------------------------------------------------------- prefix cache --
    def find_longest_prefix_blocks(self, token_ids, max_cache_blocks: int) -> list[int]:
        if self._native is not None:
            return self._native.find_longest(token_ids, max_cache_blocks)
        found: list[int] = []
        parent: ChainKey | None = None
        for block_idx in range(max_cache_blocks):
            key = self._keys.find(parent, self._block_tokens(token_ids, block_idx))
            holders = self._cached.get(key) if key is not None else None
            if not holders:
                break
            found.append(holders[0])
            parent = key
        return found

    def cache_full_blocks(self, slot: int, token_ids, num_cached_blocks: int = 0,
                          num_full_blocks: int | None = None) -> None:
        table = self.block_tables[slot]
        total_full = num_full_blocks
        if total_full is None:
            total_full = int(token_ids.numel()) // self.block_size
        if self._native is not None:
            self._native.cache_blocks(table, num_cached_blocks, total_full, token_ids)
            for block_id in table[num_cached_blocks:total_full]:
                self.blocks[block_id].block_hash = self._native.key(block_id)
            return
        parent: ChainKey | None = None
        if num_cached_blocks > 0:
            parent = self.blocks[table[num_cached_blocks - 1]].block_hash
        for block_idx in range(num_cached_blocks, total_full):
            block_id = table[block_idx]
            block = self.blocks[block_id]
            if block.block_hash is not None:
                parent = block.block_hash
                continue
            key = self._keys.acquire(parent, self._block_tokens(token_ids, block_idx))
            block.block_hash = key
            self._cached.setdefault(key, []).append(block_id)
            parent = key

    def clear_prefix_cache(self) -> None:
        if self.block_tables or any(block.ref_count > 0 for block in self.blocks):
            raise RuntimeError("cannot clear prefix cache with active sequences")
        self._cached.clear()
        self._keys.clear()  # the native index or the Python one
        for block in self.blocks:
            block.block_hash = None

    def num_cached_keys(self) -> int:
        if self._native is not None:
            return self._native.num_cached_keys()
        return len(self._cached)

    # ------------------------------------------------------------ metadata --
    def _physical_slot(self, slot: int, logical_pos: int) -> int:
        table = self.block_tables[slot]
        block_idx = logical_pos // self.block_size
        if block_idx >= len(table):
            raise RuntimeError(f"missing block: slot={slot}, logical_pos={logical_pos}")
        return table[block_idx] * self.block_size + logical_pos % self.block_size

    def get_block_tables_tensor(self, slots: list[int]) -> torch.Tensor:
        tables = [self.block_tables[slot] for slot in slots]
        width = max(len(t) for t in tables)
        host = np.zeros((len(slots), width), dtype=np.int32)
        for row, table in enumerate(tables):
            host[row, : len(table)] = table
        return torch.from_numpy(host).to(self.device)

    def get_context_lens_tensor(self, slots: list[int]) -> torch.Tensor:
        return torch.tensor([self.seq_lens[slot] for slot in slots], dtype=torch.int32, device="cpu")

    def get_slot_mapping(self, slots: list[int], start_positions: list[int],
                         num_tokens_per_seq: list[int]) -> torch.Tensor:
        parts = []
        bs = self.block_size
        for slot, start, count in zip(slots, start_positions, num_tokens_per_seq):
            if count <= 0:
                continue
            table = np.asarray(self.block_tables[slot], dtype=np.int64)
            pos = np.arange(start, start + count, dtype=np.int64)
            idx = pos // bs
            if idx[-1] >= len(table):
                first_missing = int(pos[np.argmax(idx >= len(table))])
                raise RuntimeError(f"missing block: slot={slot}, logical_pos={first_missing}")
            parts.append(table[idx] * bs + pos % bs)
        host = np.concatenate(parts) if parts else np.zeros((0,), dtype=np.int64)
        return torch.from_numpy(host).to(self.device)

    def prepare_prefill_metadata(self, slots: list[int], seq_lens: list[int], start_positions: list[int],
                                 prefix_block_ids: list[list[int]]) -> PagedKVCacheMetadata:
        if not (len(slots) == len(seq_lens) == len(start_positions) == len(prefix_block_ids)):
            raise ValueError("slots, seq_lens, start_positions and prefix_block_ids length mismatch")
        cu_q: list[int] = []
        cu_kv: list[int] = []
        total_q = total_kv = 0
        use_paged = any(start > 0 for start in start_positions)
        for slot, seq_len, start, prefix in zip(slots, seq_lens, start_positions, prefix_block_ids):
            self._init_slot(slot, start, prefix)
            end = start + seq_len
            self.ensure_blocks(slot, end)
            self.seq_lens[slot] = max(self.seq_lens[slot], end)
            total_q += seq_len
            total_kv += end
            cu_q.append(total_q)
            cu_kv.append(total_kv)
        return PagedKVCacheMetadata(
            block_tables=self.get_block_tables_tensor(slots),
            context_lens=self.get_context_lens_tensor(slots),
            slot_mapping=self.get_slot_mapping(slots, start_positions, seq_lens),
            actual_seq_lengths_q=cu_q,
            actual_seq_lengths_kv=cu_kv,
            query_lens=seq_lens,
            use_paged_prefill=use_paged,
        )

    def prepare_decode_metadata(self, slots: list[int], start_positions: list[int],
                                q_len: int) -> PagedKVCacheMetadata:
        if len(slots) != len(start_positions):
            raise ValueError("slots and start_positions length mismatch")
        for slot, start in zip(slots, start_positions):
            end = start + q_len
            self.ensure_blocks(slot, end)
            self.seq_lens[slot] = max(self.seq_lens[slot], end)
        return PagedKVCacheMetadata(
            block_tables=self.get_block_tables_tensor(slots),
            context_lens=self.get_context_lens_tensor(slots),
            slot_mapping=self.get_slot_mapping(slots, start_positions, [q_len] * len(slots)),
        )
