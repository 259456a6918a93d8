"""CUDA-graph decode runner (drop-in for ``DecodeGraphRunner`` of
src/nanovllm_ascend/npu/acl_graph.py:110-267).

What a caller of the reference sees is kept: ``DecodeGraphRunner(model,
kv_cache, batch_sizes, max_model_len, block_size)``; ``forward(input_ids,
position_ids, attn_metadata)`` returns the logits of a replay, or None when
the batch size has no graph (the caller then runs the model eagerly,
model_runner.py:262-276); a batch size whose capture fails is disabled and
logged as ``[decode_graph] disable batch_size=N: <error>``; ``stats_dict()``
has the keys ``captures``, ``replays``, ``updates``, ``fallbacks`` and
``capture_failures``; ``copy_block_tables`` pads a table into a wider static
one (acl_graph.py:253-267).

How it works on CUDA:

* One ``GraphSlot`` per batch size owns everything its graph touches: the
  static inputs (token ids, positions), the static decode metadata (block
  tables padded to ``ceil(max_model_len / block_size)`` columns, DEVICE
  context lengths, slot mapping), one split-K workspace shared by every
  attention layer of the step, the graph itself (with its own memory pool)
  and the logits it leaves behind.
* Nothing is recorded per attention call. The decode kernel reads the
  context lengths from device memory, so a replay needs no per-layer
  re-parameterisation (the Ascend graph re-issues every attention task
  before each replay, acl_graph.py:221-247). While the runner records a
  slot, attention layers fetch the slot's workspace with
  ``graph_workspace()``, which also counts them: a model that made no
  attention call fails its capture.
* Before a replay the step's metadata is refreshed in place. Metadata built
  on the device straight into the slot's buffers (``slot.metadata()`` handed
  to ``DeviceBlockTables.prepare_decode_metadata(out=...)``) costs nothing
  here; other device tensors are copied device to device; a host
  ``context_lens`` (the reference BlockManager's CPU tensor) crosses through
  a pinned staging buffer without blocking the host. The table tail beyond
  the source width is zeroed only when the width shrinks (the kernels never
  read past a sequence's context, the zeros keep the reference's contents).
* After each replay the slot's device error word is read without blocking
  (``device_errors``); a flagged replay raises on the next call.
"""

from __future__ import annotations

import math
from contextlib import contextmanager, nullcontext
from typing import Any, Iterator

import torch

from . import device_errors
from .block_manager import PagedKVCacheMetadata

# The slot whose warm-up or capture is running (at most one at a time).
_recording: "GraphSlot | None" = None


def graph_workspace(attn, batch_size: int) -> torch.Tensor | None:
    """Called by an attention layer: the split-K workspace of the decode graph
    being recorded, or None outside a runner's warm-up and capture."""
    slot = _recording
    if slot is None:
        return None
    if batch_size != slot.batch_size:
        raise RuntimeError(f"attention over {batch_size} sequences inside the batch-{slot.batch_size} decode graph")
    slot.attention_calls += 1
    return slot.workspace_for(attn.workspace_bytes(batch_size))


def recording_slot() -> "GraphSlot | None":
    return _recording


@contextmanager
def _record(slot: "GraphSlot") -> Iterator[None]:
    global _recording
    if _recording is not None:
        raise RuntimeError("decode graphs cannot be recorded inside one another")
    _recording = slot
    try:
        yield
    finally:
        _recording = None


class CudaGraphBackend:
    """The CUDA operations the runner needs (tests substitute a CPU stand-in)."""

    def new_graph(self):
        return torch.cuda.CUDAGraph()

    def capture(self, graph):
        return torch.cuda.graph(graph)

    def replay(self, graph) -> None:
        graph.replay()

    def synchronize(self) -> None:
        torch.cuda.synchronize()

    def capturing(self) -> bool:
        return torch.cuda.is_current_stream_capturing()


class GraphSlot:
    """Static buffers, workspace, graph and output of one decode batch size."""

    def __init__(self, batch_size: int, input_ids: torch.Tensor, position_ids: torch.Tensor, attn_metadata,
                 table_width: int | None, device, backend: CudaGraphBackend):
        self.batch_size = batch_size
        self.backend = backend
        self.device = torch.device(device)
        self.input_ids = torch.empty_like(input_ids, device=self.device)
        self.position_ids = torch.empty_like(position_ids, device=self.device)
        src = attn_metadata.block_tables
        width = max(table_width or 0, src.shape[1])
        self.block_tables = torch.zeros((batch_size, width), dtype=src.dtype, device=self.device)
        self.context_lens = torch.zeros(batch_size, dtype=torch.int32, device=self.device)
        self.slot_mapping = torch.zeros(attn_metadata.slot_mapping.shape, dtype=torch.int64, device=self.device)
        self._table_cols = width  # columns that may hold non-zero entries
        self.workspace: torch.Tensor | None = None
        self.graph: Any = None
        self.logits: torch.Tensor | None = None
        self.attention_calls = 0
        self.error_name = f"decode graph batch {batch_size}"

    def workspace_for(self, nbytes: int) -> torch.Tensor:
        if self.workspace is None or self.workspace.numel() < nbytes:
            if self.backend.capturing():
                raise RuntimeError("decode workspace must be sized by the warm-up run before capture")
            self.workspace = torch.zeros(max(nbytes, 1), dtype=torch.uint8, device=self.device)
        return self.workspace

    def metadata(self, like=None):
        """The step metadata as the graph sees it (the static buffers), in the type of
        ``like`` (default PagedKVCacheMetadata). Metadata built on the device can be
        written straight into it (DeviceBlockTables.prepare_decode_metadata(out=...))."""
        return (PagedKVCacheMetadata if like is None else type(like))(
            block_tables=self.block_tables,
            context_lens=self.context_lens,
            slot_mapping=self.slot_mapping,
            actual_seq_lengths_q=getattr(like, "actual_seq_lengths_q", []),
            actual_seq_lengths_kv=getattr(like, "actual_seq_lengths_kv", []),
            query_lens=getattr(like, "query_lens", []),
            use_paged_prefill=False,
        )

    def load(self, input_ids: torch.Tensor, position_ids: torch.Tensor, attn_metadata) -> None:
        """Refreshes the static inputs and metadata for the next replay."""
        _refresh(self.input_ids, input_ids)
        _refresh(self.position_ids, position_ids)
        src = attn_metadata.block_tables
        if src is not self.block_tables and src.data_ptr() != self.block_tables.data_ptr():
            width = src.shape[1]
            if width > self.block_tables.shape[1]:
                raise RuntimeError(f"decode graph block table width {self.block_tables.shape[1]} is smaller "
                                   f"than runtime width {width}")
            _refresh(self.block_tables[:, :width], src)
            if width < self._table_cols:
                self.block_tables[:, width:self._table_cols].zero_()
            self._table_cols = width
        _refresh(self.context_lens, attn_metadata.context_lens)
        _refresh(self.slot_mapping, attn_metadata.slot_mapping)


def _refresh(static: torch.Tensor, step: torch.Tensor) -> None:
    """static <- step without blocking the host; nothing to do when ``step`` is ``static``."""
    if step is static or (static.is_cuda and step.is_cuda and step.data_ptr() == static.data_ptr()
                          and step.shape == static.shape):
        return
    if static.is_cuda and not step.is_cuda:
        # Staged through pinned memory, so the caller may reuse its tensor at
        # once; torch's pinned allocator keeps the stage until the copy ran.
        stage = torch.empty(step.shape, dtype=step.dtype, pin_memory=True)
        stage.copy_(step)
        step = stage
    static.copy_(step, non_blocking=True)


class DecodeGraphStats:
    """Counters with the reference's keys (acl_graph.py:58-73). ``updates``
    counts the metadata refreshes done before replays."""

    KEYS = ("captures", "replays", "updates", "fallbacks", "capture_failures")

    def __init__(self) -> None:
        for k in self.KEYS:
            setattr(self, k, 0)

    def as_dict(self) -> dict[str, int]:
        return {k: getattr(self, k) for k in self.KEYS}


class DecodeGraphRunner:
    """Replays ``model``'s decode step from one CUDA graph per batch size.

    ``model`` is called as ``model(input_ids_flat=..., position_ids_flat=...,
    kv_cache=..., attn_metadata=..., is_prefill=False)`` and returns an
    object with ``.logits`` (the reference's Qwen3ForCausalLM contract).
    With ``fuse_appends`` the step runs inside
    ``kv_cache.deferred_appends()``, so each layer's KV append happens inside
    its decode-attention kernel.
    """

    def __init__(self, model, kv_cache, batch_sizes: list[int], max_model_len: int | None = None,
                 block_size: int | None = None, device: torch.device | str | None = None,
                 fuse_appends: bool = True, backend: CudaGraphBackend | None = None) -> None:
        self.model = model
        self.kv_cache = kv_cache
        self.batch_sizes = set(batch_sizes)
        self.table_width = math.ceil(max_model_len / block_size) if max_model_len and block_size else None
        self.device = device
        self.fuse_appends = fuse_appends
        self.backend = backend or CudaGraphBackend()
        self.slots: dict[int, GraphSlot] = {}
        self.disabled_batch_sizes: set[int] = set()
        self.stats = DecodeGraphStats()

    @property
    def entries(self) -> dict[int, GraphSlot]:
        """The captured slots by batch size."""
        return self.slots

    def supports(self, batch_size: int) -> bool:
        return batch_size in self.batch_sizes and batch_size not in self.disabled_batch_sizes

    def slot(self, batch_size: int) -> GraphSlot | None:
        return self.slots.get(batch_size)

    def forward(self, input_ids: torch.Tensor, position_ids: torch.Tensor, attn_metadata) -> torch.Tensor | None:
        batch_size = int(input_ids.numel())
        if not self.supports(batch_size):
            self.stats.fallbacks += 1
            return None
        slot = self.slots.get(batch_size) or self._capture(batch_size, input_ids, position_ids, attn_metadata)
        if slot is None:
            self.stats.fallbacks += 1
            return None
        errors = self._errors(slot)
        if errors is not None:
            errors.raise_if_flagged()
        slot.load(input_ids, position_ids, attn_metadata)
        self.stats.updates += 1
        self.backend.replay(slot.graph)
        self.stats.replays += 1
        if errors is not None:
            errors.launched(slot.error_name, device_errors.SHARED)
        return slot.logits

    def _errors(self, slot: GraphSlot):
        if slot.device.type != "cuda" or slot.workspace is None:
            return None
        errors = device_errors.state(slot.device)
        errors.watch(slot.error_name, slot.workspace)
        return errors

    def _step(self, slot: GraphSlot, static_md):
        defer = getattr(self.kv_cache, "deferred_appends", None)
        fused = defer() if (self.fuse_appends and defer is not None) else nullcontext()
        with _record(slot), fused:
            return self.model(input_ids_flat=slot.input_ids, position_ids_flat=slot.position_ids,
                              kv_cache=self.kv_cache, attn_metadata=static_md, is_prefill=False)

    def _capture(self, batch_size: int, input_ids, position_ids, attn_metadata) -> GraphSlot | None:
        try:
            device = self.device or input_ids.device
            slot = GraphSlot(batch_size, input_ids, position_ids, attn_metadata, self.table_width, device,
                             self.backend)
            slot.load(input_ids, position_ids, attn_metadata)
            static_md = slot.metadata(attn_metadata)
            self.backend.synchronize()
            # Eager warm-up outside the capture: sizes the workspace and lets
            # every kernel set itself up. It repeats this step's appends (same
            # rows, same slots), so the pool is unchanged by it.
            self._step(slot, static_md)
            self.backend.synchronize()
            slot.attention_calls = 0
            slot.graph = self.backend.new_graph()
            with self.backend.capture(slot.graph):
                slot.logits = self._step(slot, static_md).logits
            if slot.attention_calls == 0:
                raise RuntimeError("decode graph captured no paged attention calls")
        except Exception as exc:  # a failed capture disables only this batch size
            self.disabled_batch_sizes.add(batch_size)
            self.stats.capture_failures += 1
            print(f"[decode_graph] disable batch_size={batch_size}: {exc}")
            return None
        self.slots[batch_size] = slot
        self.stats.captures += 1
        return slot

    def stats_dict(self) -> dict[str, int]:
        return self.stats.as_dict()

    def release(self) -> None:
        """Drops every captured graph (call before tearing down the process group)."""
        for slot in self.slots.values():
            if slot.device.type == "cuda":
                device_errors.state(slot.device).forget(slot.error_name)
        self.slots.clear()


def copy_block_tables(target: torch.Tensor, source: torch.Tensor) -> None:
    """Zero-fills ``target`` and copies ``source`` into its leading columns
    (a narrower step table into the graph's static one)."""
    if target.dim() != 2 or source.dim() != 2:
        target.copy_(source)
        return
    if source.shape[1] > target.shape[1]:
        raise RuntimeError(f"decode graph block table width {target.shape[1]} is smaller than runtime width "
                           f"{source.shape[1]}")
    target.zero_()
    _refresh(target[:, :source.shape[1]], source)
