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

import numpy as np
import torch

from . import _lib
from .block_manager import PagedKVCacheMetadata


_STAGING_BUFFERS = 4  # pinned host staging buffers used round robin


class DeviceBlockTables:
    def __init__(self, block_manager, max_slots: int, max_blocks_per_seq: int, device=None):
        self.bm = block_manager
        self.device = torch.device(device if device is not None else block_manager.device)
        self.mirror = torch.zeros(max_slots, max_blocks_per_seq, dtype=torch.int32, device=self.device)
        # slot -> (the table list last sent, entries of it already on the device); holding the list
        # keeps its identity from being reused by a new table of a re-initialised slot
        self._synced: dict[int, tuple[list[int], int]] = {}
        self.error_word = torch.zeros(1, dtype=torch.int32, device=self.device)
        # pinned int64 staging buffers; each one's event marks the end of the copy that last read it
        self._staging = [(torch.empty(0, dtype=torch.int64), np.empty(0, dtype=np.int64))] * _STAGING_BUFFERS
        self._events = [torch.cuda.Event() for _ in range(_STAGING_BUFFERS)]
        self._next = 0
        self._fn = _lib.load().nvk_decode_metadata

    def forget(self, slot: int) -> None:
        """Drops what was sent for ``slot`` (optional: a new table is detected anyway)."""
        self._synced.pop(slot, None)

    def _staging_buffer(self, words: int) -> tuple[torch.Tensor, np.ndarray, torch.cuda.Event]:
        """A pinned int64 buffer of at least ``words`` words whose previous copy has finished,
        and the event to record after the next copy from it."""
        i = self._next
        self._next = (i + 1) % _STAGING_BUFFERS
        event = self._events[i]
        event.synchronize()  # returns at once for an event never recorded
        host, view = self._staging[i]
        if view.shape[0] < words:
            host = torch.empty(max(words, 2 * view.shape[0], 1024), dtype=torch.int64, pin_memory=True)
            view = host.numpy()
            self._staging[i] = (host, view)
        return host, view, event

    def prepare_decode_metadata(self, slots: list[int], start_positions: list[int], q_len: int,
                                width: int | None = None, out=None) -> PagedKVCacheMetadata:
        """Same contract as BlockManager.prepare_decode_metadata; the tensors are built on the device.

        ``width`` pads the block tables to a fixed number of columns (e.g. the
        CUDA-graph runner's ceil(max_model_len / block_size)); default: the
        longest table of the batch, as the host path does.

        ``out`` (a metadata object whose block_tables [batch, W] int32 with
        unit column stride, context_lens int32 [batch] and slot_mapping int64
        [batch * q_len] live on this device) receives the results in place --
        a decode graph's static buffers, so that nothing is copied before its
        replay; the tables are then padded to W columns and ``out`` is returned.
        """
        if len(slots) != len(start_positions):
            raise ValueError("slots and start_positions length mismatch")
        bm = self.bm
        bs = bm.block_size
        tables, seq_lens, synced = bm.block_tables, bm.seq_lens, self._synced
        rows, cols = self.mirror.shape
        # the allocator's bookkeeping (ensure_blocks, seq_lens) and the update lists, in one pass.
        # What is sent is recorded only after the launch, so an error leaves the record as it was.
        # Each row carries the host path's context length (seq_lens[slot] after the pass) and
        # table size; a slot named twice gets its final ones, and the same updates, in both rows.
        offsets, idx, blk, ctxs, ns = [0], [], [], [], []
        widest, bad, twice = 0, None, False
        sending = {}
        for slot, start in zip(slots, start_positions):
            end = start + q_len
            table = tables[slot]
            if len(table) * bs < end:
                bm.ensure_blocks(slot, end)
            ctx = seq_lens[slot]
            if ctx < end:
                seq_lens[slot] = ctx = end
            n = len(table)
            if n > widest:
                widest = n
            if not 0 <= slot < rows or n > cols:
                if bad is None:
                    bad = slot
                continue
            if slot in sending:
                twice = True
            sent = synced.get(slot)
            done = sent[1] if sent is not None and sent[0] is table else 0
            if done < n:
                idx.extend(range(done, n))
                blk.extend(table[done:])
            offsets.append(len(idx))
            ctxs.append(ctx)
            ns.append(n)
            sending[slot] = (table, n)
        if bad is not None:
            raise ValueError(f"sequence slot {bad} (table of {len(tables[bad])} blocks) outside the "
                             f"device mirror [{rows}, {cols}]")
        if twice:
            offsets, idx, blk, ctxs, ns = [0], [], [], [], []
            for slot in slots:
                table = tables[slot]
                n = len(table)
                sent = synced.get(slot)
                done = sent[1] if sent is not None and sent[0] is table else 0
                idx.extend(range(done, n))
                blk.extend(table[done:])
                offsets.append(len(idx))
                ctxs.append(seq_lens[slot])
                ns.append(n)
        b, m = len(slots), len(idx)
        width = width or widest
        if out is not None:
            ot, oc, os_ = out.block_tables, out.context_lens, out.slot_mapping
            if ot.dtype != torch.int32 or ot.dim() != 2 or ot.shape[0] != b or ot.stride(1) != 1 \
                    or ot.shape[1] < widest or oc.dtype != torch.int32 or oc.numel() != b or not oc.is_contiguous() \
                    or os_.dtype != torch.int64 or os_.numel() != b * q_len or not os_.is_contiguous() \
                    or any(t.device != self.device for t in (ot, oc, os_)):
                raise ValueError("prepare_decode_metadata: out buffers must be int32 [batch, >= widest table] / "
                                 "int32 [batch] / int64 [batch * q_len] on the mirror's device")
            width = ot.shape[1]
        # device buffer, int64 words: staged inputs int32 [slots | offsets | idx | blk | ctxs | ns]
        # (even length) and int64 starts; then the outputs: int32 tables [b, width], int32 context
        # lengths, int64 slots
        n32 = 4 * b + 1 + 2 * m
        w_in32 = (n32 + 1) // 2
        w_in = w_in32 + b
        w_tab = (b * width + 1) // 2
        w_ctx = (b + 1) // 2
        host, view, event = self._staging_buffer(w_in)
        view.view(np.int32)[:n32] = list(slots) + offsets + idx + blk + ctxs + ns
        view[w_in32:w_in] = start_positions
        stream = torch.cuda.current_stream(self.device)
        words = w_in if out is not None else w_in + w_tab + w_ctx + b * q_len
        buf = torch.empty(words, dtype=torch.int64, device=self.device)
        buf[:w_in].copy_(host[:w_in], non_blocking=True)
        event.record(stream)
        if out is not None:
            block_tables, context_lens, slot_mapping = out.block_tables, out.context_lens, out.slot_mapping
            tab_stride = block_tables.stride(0)
        else:
            out32 = buf[w_in:w_in + w_tab + w_ctx].view(torch.int32)
            block_tables = out32[:b * width].view(b, width)
            context_lens = out32[2 * w_tab:2 * w_tab + b]
            slot_mapping = buf[w_in + w_tab + w_ctx:]
            tab_stride = width
        base = buf.data_ptr()
        p_off = base + 4 * b
        p_idx = p_off + 4 * (b + 1)
        p_ctx = p_idx + 8 * m
        _lib.check("nvk_decode_metadata", self._fn(
            self.mirror.data_ptr(), cols, rows, base, base + 8 * w_in32, p_ctx, p_ctx + 4 * b, b, q_len, bs,
            p_off, p_idx, p_idx + 4 * m, block_tables.data_ptr(), tab_stride, width, context_lens.data_ptr(),
            slot_mapping.data_ptr(), self.error_word.data_ptr(), stream.cuda_stream))
        synced.update(sending)  # after the launch: a refused launch leaves the record as it was
        if out is not None:
            return out
        return PagedKVCacheMetadata(block_tables=block_tables, context_lens=context_lens, slot_mapping=slot_mapping)
