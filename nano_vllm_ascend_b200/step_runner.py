"""Prefill and decode step drivers on the device path (drop-in for the step
drivers of ``ModelRunner``, src/nanovllm_ascend/model_runner.py:146-167,
199-294).

``StepRunner`` takes the reference's ``Sequence`` objects (duck-typed:
``seq_id``, ``prompt_token_ids``, ``sampling_params``, ``cache_position``,
``append_next_token()``, ``set_prefill_result()``, ``set_decode_result()``)
and offers the methods ``EngineCore`` calls: ``prepare_sequences``,
``prefill``, ``decode``, ``free_seq``, ``decode_graph_stats`` and
``clear_prefix_cache``. What changes against the reference is where the step
runs:

* decode metadata is built on the device (``DeviceBlockTables``) straight
  into the static buffers of the decode graph of the batch size, and the
  token ids and positions cross in one pinned copy: no other host-to-device
  traffic per step;
* one CUDA graph per batch size (``DecodeGraphRunner``) holds every layer's
  fused q/k RMSNorm + RoPE + KV append (``nvk_qk_norm_rope_append``), paged
  decode attention and, at the end, the LM head with the greedy argmax
  (``nvk_lm_head_argmax``), so the step reads back only the next token ids
  (8 bytes a sequence) instead of one ``.item()`` per sequence
  (model_runner.py:284-286); the device error words are read with them;
* prefill runs the same layers eagerly with prefix-aware paged prefill
  attention over the pool (cached prefix + the rows just appended).

The model is Qwen3-shaped with seeded random weights (``PathModel``; no
checkpoint is loaded -- model loading, model_runner.py:85-111, is not part
of this path). Its dense parts (embedding, RMSNorm of the hidden states,
projections, MLP) are plain torch / cuBLAS; only greedy sampling
(temperature 0, the reference's default) runs on the device.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from types import SimpleNamespace

import torch
import torch.nn.functional as F

from . import device_errors, ops
from .block_manager import BlockManager
from .cuda_graph import DecodeGraphRunner
from .device_metadata import DeviceBlockTables
from .paged_attention import PagedAttention
from .paged_kv_cache import PagedKVCache
from .pool import num_blocks_from_memory

DEFAULT_DECODE_GRAPH_BATCH_SIZES = [1, 2, 4, 8, 16, 32]


@dataclass
class ModelShape:
    """The config fields of a Qwen3 model that the step needs (Qwen3-0.6B by default)."""

    num_layers: int = 28
    hidden_size: int = 1024
    num_heads: int = 16
    num_kv_heads: int = 8
    head_dim: int = 128
    intermediate_size: int = 3072
    vocab_size: int = 151936
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1000000.0
    max_position: int = 40960


def _rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * weight.float()).to(x.dtype)


class PathModel:
    """Qwen3ForCausalLM's forward (src/nanovllm_ascend/models/qwen3.py:122-221)
    with the paged-KV path on this package's kernels and seeded random weights.

    Called like the reference model: ``model(input_ids_flat=...,
    position_ids_flat=..., kv_cache=..., attn_metadata=..., is_prefill=...,
    logits_indices=...)``; returns an object whose ``logits`` are the greedy
    next-token ids (int64, one per decoded sequence or per ``logits_indices``
    row) -- the LM head and argmax are one kernel, the logits are never
    materialised.
    """

    def __init__(self, shape: ModelShape, device, seed: int = 0):
        self.shape = s = shape
        self.device = torch.device(device)
        g = torch.Generator(device=self.device).manual_seed(seed)
        bf = torch.bfloat16

        def w(*dims, scale):
            return (torch.randn(*dims, generator=g, device=self.device) * scale).to(bf)

        hd, qkv = s.hidden_size, (s.num_heads + 2 * s.num_kv_heads) * s.head_dim
        self.embed = w(s.vocab_size, hd, scale=0.02)  # tied with the LM head, as in Qwen3-0.6B
        self.layers = []
        for _ in range(s.num_layers):
            self.layers.append(SimpleNamespace(
                in_norm=torch.ones(hd, dtype=bf, device=self.device),
                post_norm=torch.ones(hd, dtype=bf, device=self.device),
                qkv=w(qkv, hd, scale=hd ** -0.5),
                q_norm=(1 + 0.1 * torch.randn(s.head_dim, generator=g, device=self.device)).to(bf),
                k_norm=(1 + 0.1 * torch.randn(s.head_dim, generator=g, device=self.device)).to(bf),
                o=w(hd, s.num_heads * s.head_dim, scale=(s.num_heads * s.head_dim) ** -0.5 * 0.5),
                gate_up=w(2 * s.intermediate_size, hd, scale=hd ** -0.5),
                down=w(hd, s.intermediate_size, scale=s.intermediate_size ** -0.5 * 0.5),
            ))
        self.final_norm = torch.ones(hd, dtype=bf, device=self.device)
        inv = 1.0 / (s.rope_theta ** (torch.arange(0, s.head_dim, 2, dtype=torch.float32) / s.head_dim))
        freqs = torch.outer(torch.arange(s.max_position, dtype=torch.float32), inv)
        emb = torch.cat((freqs, freqs), dim=-1)  # RotaryEmbedding's tables, rotary_embedding.py:20-40
        self.cos, self.sin = emb.cos().to(self.device), emb.sin().to(self.device)
        self.paged_attn = PagedAttention(s.num_heads, s.num_kv_heads, s.head_dim)
        self._lm_workspaces: dict[int, torch.Tensor] = {}

    def _lm_workspace(self, rows: int) -> torch.Tensor:
        ws = self._lm_workspaces.get(rows)
        if ws is None:  # zeroed once (the kernel leaves it zeroed); sized by the eager warm-up
            ws = torch.zeros(ops.lm_head_argmax_workspace_bytes(rows), dtype=torch.uint8, device=self.device)
            self._lm_workspaces[rows] = ws
        return ws

    def __call__(self, input_ids_flat, position_ids_flat, kv_cache, attn_metadata, is_prefill: bool,
                 logits_indices: torch.Tensor | None = None):
        s = self.shape
        t = input_ids_flat.numel()
        errors = device_errors.state(self.device)
        md = attn_metadata
        if is_prefill:
            cu_q = torch.tensor([0] + list(md.actual_seq_lengths_q), dtype=torch.int32).to(self.device,
                                                                                            non_blocking=True)
            kv_lens = md.context_lens.to(device=self.device, dtype=torch.int32, non_blocking=True)
            tables = md.block_tables.to(device=self.device, dtype=torch.int32)
            max_q = max(md.query_lens) if md.query_lens else 0
        x = self.embed[input_ids_flat]
        h_all, kvh = s.num_heads + 2 * s.num_kv_heads, s.num_kv_heads
        for i, layer in enumerate(self.layers):
            h = _rms_norm(x, layer.in_norm, s.rms_norm_eps)
            qkv = F.linear(h, layer.qkv).view(t, h_all, s.head_dim)
            kc, vc = kv_cache.get_physical_cache(i)
            q = ops.qk_norm_rope_append(qkv[:, :s.num_heads], qkv[:, s.num_heads:s.num_heads + kvh],
                                        qkv[:, s.num_heads + kvh:], layer.q_norm, layer.k_norm, s.rms_norm_eps,
                                        self.cos, self.sin, position_ids_flat, kc, vc, md.slot_mapping,
                                        error_word=errors.word)
            if is_prefill:
                attn = torch.empty_like(q)
                ops.paged_prefill(attn, q, kc, vc, tables, cu_q, kv_lens, max_q, s.head_dim ** -0.5,
                                  error_word=errors.word)
            else:
                attn = self.paged_attn(q, kc, vc, md.block_tables, md.context_lens)
            x = x + F.linear(attn.view(t, -1), layer.o)
            h = _rms_norm(x, layer.post_norm, s.rms_norm_eps)
            gate, up = F.linear(h, layer.gate_up).chunk(2, dim=-1)
            x = x + F.linear(F.silu(gate) * up, layer.down)
        h = _rms_norm(x, self.final_norm, s.rms_norm_eps)
        if logits_indices is not None:
            h = h.index_select(0, logits_indices)
        ids = ops.lm_head_argmax(h, self.embed, self._lm_workspace(h.shape[0]), error_word=errors.word)
        errors.launched()
        return SimpleNamespace(logits=ids)


@dataclass
class StepSequence:
    """The part of the reference's ``Sequence`` (src/nanovllm_ascend/sequence.py:20-67)
    that the step drivers read and update, for callers without the reference's
    engine; the reference's own objects work the same way."""

    seq_id: int
    prompt_token_ids: torch.Tensor
    sampling_params: object = None
    next_token_id: int | None = None
    cache_position: int = 0

    def __post_init__(self):
        self.generated_token_ids: list[int] = []

    def set_prefill_result(self, next_token_id: int, prompt_len: int) -> None:
        self.next_token_id = next_token_id
        self.cache_position = prompt_len

    def append_next_token(self) -> int:
        if self.next_token_id is None:
            raise RuntimeError(f"seq {self.seq_id} has no next_token_id")
        self.generated_token_ids.append(self.next_token_id)
        return self.next_token_id

    def set_decode_result(self, next_token_id: int) -> None:
        self.next_token_id = next_token_id
        self.cache_position += 1

    def token_ids(self) -> torch.Tensor:
        """Prompt and generated tokens: every token whose K/V the pool holds after a step."""
        return torch.cat([self.prompt_token_ids.to(torch.int64),
                          torch.tensor(self.generated_token_ids, dtype=torch.int64)])


class StepRunner:
    """Prefill / decode steps of ``ModelRunner`` (model_runner.py:18-297) on the device path."""

    def __init__(self, shape: ModelShape | None = None, device="cuda", max_model_len: int = 2048,
                 num_blocks: int | None = None, block_size: int = 128, memory_utilization: float = 0.8,
                 max_num_seqs: int = 32, enable_prefix_cache: bool = False, enable_decode_graph: bool = True,
                 decode_graph_batch_sizes: list[int] | None = None, seed: int = 0):
        self.shape = shape or ModelShape()
        self.device = torch.device(device)
        self.max_model_len = max_model_len
        self.block_size = block_size
        self.enable_prefix_cache = enable_prefix_cache
        s = self.shape
        self.model = PathModel(self.shape, self.device, seed)
        self.num_blocks = num_blocks or num_blocks_from_memory(memory_utilization, s.num_layers, block_size,
                                                               s.num_kv_heads, s.head_dim, torch.bfloat16,
                                                               self.device)
        self.block_manager = BlockManager(self.num_blocks, block_size, self.device)
        self.kv_cache = PagedKVCache(s.num_layers, self.num_blocks, block_size, s.num_kv_heads, s.head_dim,
                                     torch.bfloat16, self.device)
        self.table_width = math.ceil(max_model_len / block_size)
        self.device_tables = DeviceBlockTables(self.block_manager, max_num_seqs, self.table_width, self.device)
        self.errors = device_errors.state(self.device)
        self.errors.watch("decode metadata", self.device_tables.error_word)
        self.decode_graph_runner = None
        if enable_decode_graph:
            self.decode_graph_runner = DecodeGraphRunner(
                self.model, self.kv_cache, batch_sizes=decode_graph_batch_sizes or DEFAULT_DECODE_GRAPH_BATCH_SIZES,
                max_model_len=max_model_len, block_size=block_size, device=self.device, fuse_appends=False)
        # sequence id -> row of the block manager and of the device table mirror
        self._rows: dict[int, int] = {}
        self._free_rows = list(range(max_num_seqs))
        self._io = torch.empty(2 * max_num_seqs, dtype=torch.int64, pin_memory=True)  # ids | positions
        self._tokens = torch.empty(max(max_num_seqs, 1), dtype=torch.int64, pin_memory=True)

    # ------------------------------------------------------------ prefill ---
    def prepare_sequences(self, seqs) -> None:
        """Prefix-cache lookup and the runtime prompt suffix (model_runner.py:146-167)."""
        for seq in seqs:
            seq.estimated_prompt_len = int(seq.prompt_token_ids.numel())
            if seq.estimated_prompt_len > self.max_model_len:
                raise ValueError(f"prompt length {seq.estimated_prompt_len} exceeds max_model_len "
                                 f"{self.max_model_len}")
            seq.cached_block_ids = []
            seq.cached_prefix_len = 0
            if self.enable_prefix_cache:
                full = seq.estimated_prompt_len // self.block_size
                limit = full - 1 if seq.estimated_prompt_len % self.block_size == 0 and full > 0 else full
                if limit > 0:
                    seq.cached_block_ids = self.block_manager.find_longest_prefix_blocks(
                        seq.prompt_token_ids, max_cache_blocks=limit)
                    seq.cached_prefix_len = len(seq.cached_block_ids) * self.block_size
            seq.runtime_prompt_token_ids = seq.prompt_token_ids[seq.cached_prefix_len:]
            seq.runtime_prompt_len = int(seq.runtime_prompt_token_ids.numel())
            if seq.runtime_prompt_len <= 0:
                raise ValueError(f"seq {seq.seq_id} has empty runtime prompt suffix")

    def _row(self, seq) -> int:
        row = self._rows.get(seq.seq_id)
        if row is None:
            if not self._free_rows:
                raise RuntimeError(f"more than {len(self._rows)} sequences in flight (max_num_seqs)")
            row = self._free_rows.pop(0)
            self._rows[seq.seq_id] = row
        return row

    @staticmethod
    def _check_greedy(seqs) -> None:
        for seq in seqs:
            params = getattr(seq, "sampling_params", None)
            if params is not None and getattr(params, "temperature", 0) not in (0, 0.0):
                raise ValueError("only greedy sampling (temperature=0) runs on the device path")

    def _read_tokens(self, ids: torch.Tensor) -> list[int]:
        n = ids.numel()
        host = self._tokens[:n] if n <= self._tokens.numel() else torch.empty(n, dtype=torch.int64,
                                                                               pin_memory=True)
        host.copy_(ids, non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        self.errors.raise_if_flagged()  # this step's error words were read behind its kernels
        return host.tolist()

    @torch.inference_mode()
    def prefill(self, seqs) -> None:
        """One prefill step (model_runner.py:199-238): prefix-aware paged attention over
        the pool, next tokens by the device argmax, full prompt blocks cached."""
        if not seqs:
            return
        self._check_greedy(seqs)
        rows = [self._row(seq) for seq in seqs]
        lens = [seq.runtime_prompt_len for seq in seqs]
        ids = torch.cat([seq.runtime_prompt_token_ids.to(torch.int64) for seq in seqs])
        pos = torch.cat([torch.arange(seq.cached_prefix_len, seq.cached_prefix_len + n, dtype=torch.int64)
                         for seq, n in zip(seqs, lens)])
        last = torch.tensor(lens, dtype=torch.int64).cumsum(0) - 1
        md = self.block_manager.prepare_prefill_metadata(
            slots=rows, seq_lens=lens, start_positions=[seq.cached_prefix_len for seq in seqs],
            prefix_block_ids=[seq.cached_block_ids for seq in seqs])
        with torch.cuda.device(self.device):
            stage = torch.cat([ids, pos, last]).pin_memory()
            dev = stage.to(self.device, non_blocking=True)
            t = ids.numel()
            out = self.model(input_ids_flat=dev[:t], position_ids_flat=dev[t:2 * t], kv_cache=self.kv_cache,
                             attn_metadata=md, is_prefill=True, logits_indices=dev[2 * t:])
            tokens = self._read_tokens(out.logits)
        for seq, token in zip(seqs, tokens):
            seq.set_prefill_result(next_token_id=token, prompt_len=seq.estimated_prompt_len)
            if self.enable_prefix_cache:
                self.block_manager.cache_full_blocks(
                    slot=self._rows[seq.seq_id], token_ids=seq.prompt_token_ids,
                    num_cached_blocks=len(seq.cached_block_ids),
                    num_full_blocks=seq.estimated_prompt_len // self.block_size)

    # ------------------------------------------------------------- decode ---
    @torch.inference_mode()
    def decode(self, seqs) -> None:
        """One decode step (model_runner.py:240-286) of every sequence in ``seqs``."""
        if not seqs:
            return
        self._check_greedy(seqs)
        token_ids = [seq.append_next_token() for seq in seqs]
        positions = [seq.cache_position for seq in seqs]
        rows = [self._rows[seq.seq_id] for seq in seqs]
        b = len(seqs)
        with torch.cuda.device(self.device):
            io = self._io[:2 * b] if 2 * b <= self._io.numel() else torch.empty(2 * b, dtype=torch.int64,
                                                                                 pin_memory=True)
            io[:b] = torch.tensor(token_ids, dtype=torch.int64)
            io[b:] = torch.tensor(positions, dtype=torch.int64)
            runner = self.decode_graph_runner
            slot = runner.slot(b) if runner is not None else None
            if slot is not None:
                # the graph's own buffers receive this step's inputs and metadata
                slot.input_ids.copy_(io[:b], non_blocking=True)
                slot.position_ids.copy_(io[b:], non_blocking=True)
                md = self.device_tables.prepare_decode_metadata(rows, positions, 1, out=slot.metadata())
                ids, pos = slot.input_ids, slot.position_ids
            else:
                md = self.device_tables.prepare_decode_metadata(rows, positions, 1, width=self.table_width)
                dev = io.to(self.device, non_blocking=True)
                ids, pos = dev[:b], dev[b:]
            self.errors.mark("decode metadata")  # read with the step's other words, after its kernels
            next_ids = runner.forward(ids, pos, md) if runner is not None else None
            if next_ids is None:
                next_ids = self.model(input_ids_flat=ids, position_ids_flat=pos, kv_cache=self.kv_cache,
                                      attn_metadata=md, is_prefill=False).logits
            tokens = self._read_tokens(next_ids)
        for seq, token in zip(seqs, tokens):
            seq.set_decode_result(token)

    # ------------------------------------------------------------ the rest ---
    def free_seq(self, seq) -> None:
        row = self._rows.pop(seq.seq_id, None)
        if row is None:
            return
        self.block_manager.free_slot(row)
        self.device_tables.forget(row)
        self._free_rows.append(row)

    def decode_graph_stats(self) -> dict[str, int]:
        return {} if self.decode_graph_runner is None else self.decode_graph_runner.stats_dict()

    def clear_prefix_cache(self) -> None:
        self.block_manager.clear_prefix_cache()

    def release(self) -> None:
        if self.decode_graph_runner is not None:
            self.decode_graph_runner.release()
