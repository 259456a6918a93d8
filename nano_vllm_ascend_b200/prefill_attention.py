"""Causal prefill attention module (drop-in for
``nanovllm_ascend.layers.npu_prefill_attention.NpuBatchPrefillAttention``,
src/nanovllm_ascend/layers/npu_prefill_attention.py:8-113).

Two modes, chosen by ``attn_metadata.use_paged_prefill`` as in the reference:

* paged (any sequence has a cached prefix, :66-96): queries attend over the
  WHOLE paged KV of their sequence -- cached prefix + the rows appended this
  step -- through ``block_tables`` with absolute ``context_lens``;
* dense (:97-112): queries attend over the contiguous ``k``/``v`` of this step
  delimited by the cumulative ``actual_seq_lengths_kv``.

Both are bottom-right-aligned causal (the reference's ``sparse_mode=3``):
query i of a sequence with q_len Lq and kv_len Lk sees key j iff
j <= Lk - Lq + i. There is no mask tensor; the reference's 2048x2048 int8
mask (:23-29) only existed for the Ascend op.

A paged-mode ``context_lens`` longer than its block-table row raises
``RuntimeError("missing block ...")`` before the launch (block_manager.py:194-205);
a block id outside the pool is reported through the device's error word and
raised by ``device_errors`` on a following call or by
``device_errors.check_errors()``.
"""

from __future__ import annotations

import torch
from torch import nn

from . import device_errors, ops


def _cu(values: list[int], device: torch.device) -> torch.Tensor:
    return torch.tensor([0] + list(values), dtype=torch.int32).to(device)


class BatchPrefillAttention(nn.Module):
    def __init__(self, num_heads: int, num_key_value_heads: int, head_dim: int, block_size: int,
                 max_mask_len: int):
        super().__init__()
        self.num_heads = num_heads
        self.num_key_value_heads = num_key_value_heads
        self.head_dim = head_dim
        self.block_size = block_size
        self.max_mask_len = max_mask_len
        self.scale = head_dim ** -0.5

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, attn_metadata,
                key_cache: torch.Tensor | None = None, value_cache: torch.Tensor | None = None) -> torch.Tensor:
        total_tokens, num_heads, head_dim = q.shape
        if num_heads != self.num_heads or head_dim != self.head_dim:
            raise ValueError(f"query shape mismatch: got {tuple(q.shape)}")
        if k.shape[0] != total_tokens or v.shape[0] != total_tokens:
            raise ValueError(f"k/v token mismatch: q={tuple(q.shape)} k={tuple(k.shape)} v={tuple(v.shape)}")

        q_lens = []
        prev = 0
        for end in attn_metadata.actual_seq_lengths_q:
            q_lens.append(end - prev)
            prev = end
        max_prompt_len = max(q_lens, default=0)
        if max_prompt_len > self.max_mask_len:
            raise ValueError(f"prompt length {max_prompt_len} exceeds max_mask_len {self.max_mask_len}")

        query = q.to(dtype=v.dtype).contiguous()
        out = torch.empty_like(query)
        if total_tokens == 0:
            return out.view(total_tokens, self.num_heads, self.head_dim)
        device = query.device
        cache = getattr(attn_metadata, "_nvk_prefill_device", None)
        if cache is None or cache[0] != device:
            cu_q = _cu(attn_metadata.actual_seq_lengths_q, device)
            cu_kv = _cu(attn_metadata.actual_seq_lengths_kv, device)
            ctx = attn_metadata.context_lens.to(device=device, dtype=torch.int32)
            tables = attn_metadata.block_tables.to(device=device, dtype=torch.int32).contiguous()
            cache = (device, cu_q, cu_kv, ctx, tables)
            try:  # the same metadata serves every layer of the step
                attn_metadata._nvk_prefill_device = cache
            except AttributeError:
                pass
        _, cu_q, cu_kv, ctx, tables = cache
        with torch.cuda.device(device):
            errors = device_errors.state(device)
            errors.raise_if_flagged()
            if attn_metadata.use_paged_prefill:
                if key_cache is None or value_cache is None:
                    raise ValueError("paged prefill requires physical key/value cache")
                lens = attn_metadata.context_lens
                if not getattr(lens, "is_cuda", True) and lens.numel():
                    longest = int(lens.max())
                    if longest > tables.shape[1] * key_cache.shape[1]:
                        raise RuntimeError(f"missing block: context length {longest} exceeds the "
                                           f"{tables.shape[1]}-block table")
                ops.paged_prefill(out, query, key_cache, value_cache, tables, cu_q, ctx, max_prompt_len,
                                  self.scale, error_word=errors.word)
            else:
                ops.dense_prefill(out, query, k.contiguous(), v.contiguous(), cu_q, cu_kv, max_prompt_len,
                                  self.scale, error_word=errors.word)
            errors.launched()
        return out.view(total_tokens, self.num_heads, self.head_dim)
