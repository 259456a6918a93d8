"""Decode metadata built on the device (the Python loops of
BlockManager.prepare_decode_metadata, src/nanovllm_ascend/npu/block_manager.py:304-328,
and of get_block_tables_tensor / get_slot_mapping, :207-250, moved into
nvk_decode_metadata).

``DeviceBlockTables`` keeps a persistent device mirror of a BlockManager's
per-sequence block tables. Each decode step it does the allocator's host
bookkeeping exactly as the BlockManager does (ensure_blocks, seq_lens), sends
only the table entries added since the previous step (a whole table for a new
or reused sequence slot) in one packed host-to-device copy, and one kernel
writes the padded block tables, context lengths and slot mapping -- bit for
bit what the host path returns, except that ``context_lens`` is a device
tensor (as the CUDA-graph path wants it).
"""

from __future__ import annotations

import torch

from . import _lib
from .block_manager import PagedKVCacheMetadata
from .ops import _ptr, _stream


class DeviceBlockTables:
    def __init__(self, block_manager, max_slots: int, max_blocks_per_seq: int, device=None):
        self.bm = block_manager
        self.device = torch.device(device if device is not None else block_manager.device)
        self.mirror = torch.zeros(max_slots, max_blocks_per_seq, dtype=torch.int32, device=self.device)
        # slot -> (the table list last sent, entries of it already on the device); holding the list
        # keeps its identity from being reused by a new table of a re-initialised slot
        self._synced: dict[int, tuple[list[int], int]] = {}
        self.error_word = torch.zeros(1, dtype=torch.int32, device=self.device)

    def _updates(self, slots: list[int]) -> tuple[list[int], list[int], list[int]]:
        offsets, idx, blk = [0], [], []
        for slot in slots:
            table = self.bm.block_tables[slot]
            sent, done = self._synced.get(slot, (None, 0))
            if sent is not table:
                done = 0
            idx.extend(range(done, len(table)))
            blk.extend(table[done:])
            offsets.append(len(idx))
            self._synced[slot] = (table, len(table))
        return offsets, idx, blk

    def forget(self, slot: int) -> None:
        """Drops what was sent for ``slot`` (optional: a new table is detected anyway)."""
        self._synced.pop(slot, None)

    def prepare_decode_metadata(self, slots: list[int], start_positions: list[int], q_len: int,
                                width: int | None = None) -> PagedKVCacheMetadata:
        """Same contract as BlockManager.prepare_decode_metadata; the tensors are built on the device.

        ``width`` pads the block tables to a fixed number of columns (e.g. the
        CUDA-graph runner's ceil(max_model_len / block_size)); default: the
        longest table of the batch, as the host path does.
        """
        if len(slots) != len(start_positions):
            raise ValueError("slots and start_positions length mismatch")
        bm = self.bm
        for slot, start in zip(slots, start_positions):
            end = start + q_len
            bm.ensure_blocks(slot, end)
            bm.seq_lens[slot] = max(bm.seq_lens[slot], end)
        rows, cols = self.mirror.shape
        for slot in slots:
            if not 0 <= slot < rows or len(bm.block_tables[slot]) > cols:
                raise ValueError(f"sequence slot {slot} (table of {len(bm.block_tables[slot])} blocks) outside the "
                                 f"device mirror [{rows}, {cols}]")
        offsets, idx, blk = self._updates(slots)
        b = len(slots)
        width = width or max(len(bm.block_tables[s]) for s in slots)
        # one packed copy: int32 [slots | offsets | idx | blk], then int64 starts
        n32 = b + (b + 1) + 2 * len(idx)
        n32_pad = (n32 + 1) // 2 * 2
        host = torch.empty(n32_pad // 2 + b, dtype=torch.int64)
        h32 = host[: n32_pad // 2].view(torch.int32)
        h32[:n32] = torch.tensor(list(slots) + offsets + idx + blk, dtype=torch.int32)
        host[n32_pad // 2:] = torch.tensor(list(start_positions), dtype=torch.int64)
        dev = host.to(self.device)
        d32 = dev[: n32_pad // 2].view(torch.int32)
        d_slots, d_off = d32[:b], d32[b: 2 * b + 1]
        d_idx, d_blk = d32[2 * b + 1: 2 * b + 1 + len(idx)], d32[2 * b + 1 + len(idx): n32]
        d_start = dev[n32_pad // 2:]
        tables = torch.empty(b, width, dtype=torch.int32, device=self.device)
        ctx = torch.empty(b, dtype=torch.int32, device=self.device)
        slot_mapping = torch.empty(b * q_len, dtype=torch.int64, device=self.device)
        _lib.call("nvk_decode_metadata", _ptr(self.mirror), cols, rows, _ptr(d_slots), _ptr(d_start), b, q_len,
                  bm.block_size, _ptr(d_off), _ptr(d_idx), _ptr(d_blk), _ptr(tables), width, width, _ptr(ctx),
                  _ptr(slot_mapping), _ptr(self.error_word), _stream(self.device))
        return PagedKVCacheMetadata(block_tables=tables, context_lens=ctx, slot_mapping=slot_mapping)
