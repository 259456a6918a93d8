"""CUDA-graph decode runner (replaces the ACL-graph runner of
src/nanovllm_ascend/npu/acl_graph.py:110-267).

Same contract as the reference: one graph per exact decode batch size in
``batch_sizes``, captured on first use; static input/metadata buffers with
block tables padded to ``ceil(max_model_len / block_size)`` columns
(:123-124, :208-219, :253-267); a batch size whose capture fails is disabled
and reported as a fallback (:184-202); the same statistics keys (:58-73).

What changes on CUDA: ``context_lens`` lives in a static DEVICE buffer that the
decode kernel reads, so a replay needs no per-layer "task update" (the
reference re-issues every paged-attention task before each replay,
:221-247). ``updates`` therefore counts the metadata refreshes done before a
replay. The decode workspace is fixed per entry at capture time (the
reference's per-task workspace, :229-242).
"""

from __future__ import annotations

import math
from contextlib import contextmanager, nullcontext
from dataclasses import dataclass, field
from typing import Any, Iterator

import torch

_active_decode_graph_entry: "DecodeGraphEntry | None" = None


@dataclass
class PagedAttentionGraphTask:
    query: torch.Tensor
    key_cache: torch.Tensor
    value_cache: torch.Tensor
    num_kv_heads: int
    num_heads: int
    scale: float
    block_tables: torch.Tensor
    context_lens: torch.Tensor
    output: torch.Tensor
    workspace: Any


@dataclass
class DecodeGraphEntry:
    batch_size: int
    input_ids: torch.Tensor
    position_ids: torch.Tensor
    block_tables: torch.Tensor
    context_lens: torch.Tensor
    slot_mapping: torch.Tensor
    graph: Any
    logits: torch.Tensor | None = None
    tasks: list[PagedAttentionGraphTask] = field(default_factory=list)
    workspace: torch.Tensor | None = None

    def copy_inputs(self, input_ids: torch.Tensor, position_ids: torch.Tensor, attn_metadata) -> None:
        copy_in(self.input_ids, input_ids)
        copy_in(self.position_ids, position_ids)
        copy_block_tables(self.block_tables, attn_metadata.block_tables)
        copy_in(self.context_lens, attn_metadata.context_lens)
        copy_in(self.slot_mapping, attn_metadata.slot_mapping)

    def decode_workspace(self, attn) -> torch.Tensor:
        """This entry's decode workspace, sized and zeroed by the eager warm-up
        run before capture so that captured kernels and replays share it."""
        need = attn.workspace_bytes(self.batch_size)
        if self.workspace is None or self.workspace.numel() < need:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("decode workspace must be sized by the warm-up run before capture")
            self.workspace = torch.zeros(need, dtype=torch.uint8, device=self.block_tables.device)
        return self.workspace


class DecodeGraphStats:
    def __init__(self) -> None:
        self.captures = 0
        self.replays = 0
        self.updates = 0
        self.fallbacks = 0
        self.capture_failures = 0

    def as_dict(self) -> dict[str, int]:
        return {
            "captures": self.captures,
            "replays": self.replays,
            "updates": self.updates,
            "fallbacks": self.fallbacks,
            "capture_failures": self.capture_failures,
        }


def current_decode_graph_entry() -> DecodeGraphEntry | None:
    return _active_decode_graph_entry


@contextmanager
def capture_decode_graph_tasks(entry: DecodeGraphEntry) -> Iterator[None]:
    global _active_decode_graph_entry
    previous = _active_decode_graph_entry
    _active_decode_graph_entry = entry
    try:
        yield
    finally:
        _active_decode_graph_entry = previous


def record_paged_attention_task(task: PagedAttentionGraphTask) -> None:
    entry = current_decode_graph_entry()
    if entry is None:
        raise RuntimeError("paged attention graph task recorded outside graph capture")
    entry.tasks.append(task)


class DecodeGraphRunner:
    """Captures ``model`` once per supported decode batch size and replays it.

    ``model`` is called as ``model(input_ids_flat=..., position_ids_flat=...,
    kv_cache=..., attn_metadata=..., is_prefill=False)`` and must return an
    object with ``.logits`` (the reference's Qwen3ForCausalLM contract).
    """

    def __init__(self, model, kv_cache, batch_sizes: list[int], max_model_len: int | None = None,
                 block_size: int | None = None, device: torch.device | str | None = None,
                 fuse_appends: bool = True) -> None:
        self.model = model
        self.kv_cache = kv_cache
        # Decode appends fused into the attention kernels (PagedKVCache.deferred_appends).
        self.fuse_appends = fuse_appends
        self.batch_sizes = set(batch_sizes)
        self.max_blocks_per_seq = None
        if max_model_len is not None and block_size is not None:
            self.max_blocks_per_seq = math.ceil(max_model_len / block_size)
        self.device = device
        self.entries: dict[int, DecodeGraphEntry] = {}
        self.disabled_batch_sizes: set[int] = set()
        self.stats = DecodeGraphStats()

    # Graph backend hooks (overridden by the CPU tests).
    def _new_graph(self):
        return torch.cuda.CUDAGraph()

    def _graph_context(self, graph):
        return torch.cuda.graph(graph)

    def _synchronize(self) -> None:
        torch.cuda.synchronize()

    def _replay(self, graph) -> None:
        graph.replay()

    def supports(self, batch_size: int) -> bool:
        return batch_size in self.batch_sizes and batch_size not in self.disabled_batch_sizes

    def forward(self, input_ids: torch.Tensor, position_ids: torch.Tensor, attn_metadata) -> torch.Tensor | None:
        batch_size = int(input_ids.numel())
        if not self.supports(batch_size):
            self.stats.fallbacks += 1
            return None
        entry = self.entries.get(batch_size)
        if entry is None:
            entry = self._capture(batch_size, input_ids, position_ids, attn_metadata)
            if entry is None:
                self.stats.fallbacks += 1
                return None
        entry.copy_inputs(input_ids, position_ids, attn_metadata)
        self.stats.updates += 1
        self._replay(entry.graph)
        self.stats.replays += 1
        return entry.logits

    def _static_metadata(self, entry: DecodeGraphEntry, attn_metadata):
        md_type = type(attn_metadata)
        return md_type(
            block_tables=entry.block_tables,
            context_lens=entry.context_lens,
            slot_mapping=entry.slot_mapping,
            actual_seq_lengths_q=attn_metadata.actual_seq_lengths_q,
            actual_seq_lengths_kv=attn_metadata.actual_seq_lengths_kv,
            query_lens=attn_metadata.query_lens,
            use_paged_prefill=attn_metadata.use_paged_prefill,
        )

    def _run_model(self, entry: DecodeGraphEntry, static_md):
        defer = getattr(self.kv_cache, "deferred_appends", None)
        fused = defer() if (self.fuse_appends and defer is not None) else nullcontext()
        with capture_decode_graph_tasks(entry), fused:
            return self.model(
                input_ids_flat=entry.input_ids,
                position_ids_flat=entry.position_ids,
                kv_cache=self.kv_cache,
                attn_metadata=static_md,
                is_prefill=False,
            )

    def _capture(self, batch_size: int, input_ids: torch.Tensor, position_ids: torch.Tensor,
                 attn_metadata) -> DecodeGraphEntry | None:
        try:
            device = self.device or input_ids.device
            graph = self._new_graph()
            ctx_dev = attn_metadata.context_lens
            if hasattr(ctx_dev, "to") and not getattr(ctx_dev, "is_cuda", True):
                ctx_dev = ctx_dev.to(device=device, dtype=torch.int32)
            entry = DecodeGraphEntry(
                batch_size=batch_size,
                input_ids=input_ids.clone(),
                position_ids=position_ids.clone(),
                block_tables=self._make_static_block_tables(batch_size, attn_metadata.block_tables),
                context_lens=ctx_dev.clone(),
                slot_mapping=attn_metadata.slot_mapping.clone(),
                graph=graph,
            )
            static_md = self._static_metadata(entry, attn_metadata)
            self._synchronize()
            # Eager warm-up: fixes the split policy and allocates the workspace
            # outside the capture. It repeats this step's appends with the same
            # rows into the same slots, so it does not change the pool.
            self._run_model(entry, static_md)
            entry.tasks.clear()
            self._synchronize()
            with self._graph_context(graph):
                outputs = self._run_model(entry, static_md)
                entry.logits = outputs.logits
            if not entry.tasks:
                raise RuntimeError("decode graph captured no paged attention tasks")
        except Exception as exc:  # capture failure disables only this batch size
            self.disabled_batch_sizes.add(batch_size)
            self.stats.capture_failures += 1
            print(f"[decode_graph] disable batch_size={batch_size}: {exc}")
            return None
        self.entries[batch_size] = entry
        self.stats.captures += 1
        return entry

    def _make_static_block_tables(self, batch_size: int, block_tables: torch.Tensor) -> torch.Tensor:
        if self.max_blocks_per_seq is None:
            return block_tables.clone()
        static = block_tables.new_zeros((batch_size, self.max_blocks_per_seq))
        copy_block_tables(static, block_tables)
        return static

    def stats_dict(self) -> dict[str, int]:
        return self.stats.as_dict()

    def release(self) -> None:
        """Drops every captured graph (call before tearing down the process group)."""
        self.entries.clear()


def copy_block_tables(target: torch.Tensor, source: torch.Tensor) -> None:
    """Zero-fills ``target`` and copies ``source`` into its leading columns."""
    target_shape = getattr(target, "shape", None)
    source_shape = getattr(source, "shape", None)
    if target_shape is None or source_shape is None or len(target_shape) != 2 or len(source_shape) != 2:
        target.copy_(source)
        return
    if source_shape[1] > target_shape[1]:
        raise RuntimeError(
            f"decode graph block table width {target_shape[1]} is smaller than runtime width {source_shape[1]}"
        )
    target.zero_()
    copy_in(target[:, : source_shape[1]], source)


def copy_in(target: torch.Tensor, source: torch.Tensor) -> None:
    """``target.copy_(source)`` without blocking the host. A host ``source`` bound
    for a CUDA ``target`` (``context_lens`` from the host BlockManager, for one)
    is first copied into a fresh pinned buffer, so the caller may change its
    tensor at once, and crosses asynchronously on the current stream; torch's
    pinned allocator keeps that buffer until the copy has run. A plain blocking
    copy would drain the stream before every replay."""
    if getattr(target, "is_cuda", False) and isinstance(source, torch.Tensor) and not source.is_cuda:
        staged = torch.empty(source.shape, dtype=source.dtype, pin_memory=True)
        staged.copy_(source)
        target.copy_(staged, non_blocking=True)
    else:
        target.copy_(source)
