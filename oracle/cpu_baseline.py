"""Eager PyTorch-CPU expression of the reference's paged-KV path -- TEST AND
BASELINE INFRASTRUCTURE ONLY (imported by bench.py's CPU-baseline leg and by
tests; never by the product).

This is the reference path as the reference itself would run it without an
Ascend device: ``index_copy_`` appends into the flattened layer pool
(src/nanovllm_ascend/npu/paged_kv_cache.py:57-69) and, in place of the closed
``_npu_paged_attention``/``npu_fused_infer_attention_score`` ops, a
per-sequence block-table gather followed by fp32 GQA softmax(q K^T) V, with
bottom-right causal masking for prefill. torch uses every host thread it is
given (``torch.set_num_threads``).
"""

from __future__ import annotations

import torch


def append(key_cache_layer: torch.Tensor, value_cache_layer: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
           slot_mapping: torch.Tensor) -> None:
    nb, bs, kvh, d = key_cache_layer.shape
    key_cache_layer.view(nb * bs, kvh, d).index_copy_(0, slot_mapping, key.contiguous())
    value_cache_layer.view(nb * bs, kvh, d).index_copy_(0, slot_mapping, value.contiguous())


def _gather(cache_layer: torch.Tensor, table: torch.Tensor, n: int) -> torch.Tensor:
    bs = cache_layer.shape[1]
    nblk = (n + bs - 1) // bs
    return cache_layer.index_select(0, table[:nblk].long()).reshape(nblk * bs, *cache_layer.shape[2:])[:n]


def decode(q: torch.Tensor, key_cache_layer: torch.Tensor, value_cache_layer: torch.Tensor,
           block_tables: torch.Tensor, context_lens: torch.Tensor, scale: float) -> torch.Tensor:
    """q [B, H, D] (bf16) -> [B, H, D] bf16, fp32 math."""
    b_sz, h, d = q.shape
    kvh = key_cache_layer.shape[2]
    out = torch.empty_like(q)
    for b in range(b_sz):
        n = int(context_lens[b])
        k = _gather(key_cache_layer, block_tables[b], n).float()  # [n, KVH, D]
        v = _gather(value_cache_layer, block_tables[b], n).float()
        qg = q[b].float().view(kvh, h // kvh, d)
        s = torch.einsum("gqd,ngd->gqn", qg, k) * scale
        p = torch.softmax(s, dim=-1)
        out[b] = torch.einsum("gqn,ngd->gqd", p, v).reshape(h, d).to(q.dtype)
    return out


def prefill(q: torch.Tensor, key_cache_layer: torch.Tensor, value_cache_layer: torch.Tensor,
            block_tables: torch.Tensor, cu_seqlens_q: list[int], kv_lens: list[int], scale: float) -> torch.Tensor:
    """q [Tq, H, D] -> [Tq, H, D], bottom-right causal over each sequence's paged KV."""
    tq, h, d = q.shape
    kvh = key_cache_layer.shape[2]
    out = torch.empty_like(q)
    for b in range(len(kv_lens)):
        s0, e0 = cu_seqlens_q[b], cu_seqlens_q[b + 1]
        lq, lk = e0 - s0, kv_lens[b]
        k = _gather(key_cache_layer, block_tables[b], lk).float()
        v = _gather(value_cache_layer, block_tables[b], lk).float()
        qg = q[s0:e0].float().view(lq, kvh, h // kvh, d)
        s = torch.einsum("tgqd,ngd->gqtn", qg, k) * scale
        i = torch.arange(lq)[:, None]
        j = torch.arange(lk)[None, :]
        s = s.masked_fill(~(j <= (lk - lq) + i), float("-inf"))
        p = torch.softmax(s, dim=-1)
        out[s0:e0] = torch.einsum("gqtn,ngd->tgqd", p, v).reshape(lq, h, d).to(q.dtype)
    return out
