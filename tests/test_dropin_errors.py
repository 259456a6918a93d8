"""The drop-in classes reject bad inputs with the reference's exceptions and
messages, before any device work (so these run on the CPU):
PagedKVCache.write (src/nanovllm_ascend/npu/paged_kv_cache.py:51-55),
NpuPagedAttention.forward (layers/npu_paged_attention.py:35-37) and
NpuBatchPrefillAttention.forward (layers/npu_prefill_attention.py:50-62)."""

import re
from types import SimpleNamespace

import pytest
import torch

from nano_vllm_ascend_b200 import NpuBatchPrefillAttention, NpuPagedAttention, PagedKVCache

BF16 = torch.bfloat16


def test_kv_cache_write_errors():
    kv = PagedKVCache(1, 4, 128, 8, 128, BF16, "cpu")
    bad = torch.zeros(3, 4, 128, dtype=BF16)
    with pytest.raises(ValueError, match=re.escape("kv shape mismatch: got (3, 4, 128)")):
        kv.write(0, bad, bad, torch.zeros(3, dtype=torch.long))
    k = torch.zeros(3, 8, 128, dtype=BF16)
    with pytest.raises(ValueError, match=re.escape("slot_mapping numel 2 != total_tokens 3")):
        kv.write(0, k, k, torch.zeros(2, dtype=torch.long))


def test_paged_attention_query_shape_error():
    attn = NpuPagedAttention(16, 8, 128)
    q = torch.zeros(2, 8, 128, dtype=BF16)
    kc = torch.zeros(4, 128, 8, 128, dtype=BF16)
    with pytest.raises(ValueError, match=re.escape("query shape mismatch: got (2, 8, 128)")):
        attn(q, kc, kc, torch.zeros(2, 1, dtype=torch.int32), torch.ones(2, dtype=torch.int32))


def test_prefill_attention_errors():
    attn = NpuBatchPrefillAttention(16, 8, 128, 128, max_mask_len=64)
    md = SimpleNamespace(actual_seq_lengths_q=[100], actual_seq_lengths_kv=[100], use_paged_prefill=False)
    q = torch.zeros(100, 16, 128, dtype=BF16)
    kv = torch.zeros(100, 8, 128, dtype=BF16)
    with pytest.raises(ValueError, match=re.escape("query shape mismatch: got (100, 8, 128)")):
        attn(kv, kv, kv, md)
    with pytest.raises(ValueError, match=re.escape("k/v token mismatch: q=(100, 16, 128) k=(99, 8, 128) v=(100, 8, 128)")):
        attn(q, kv[:99], kv, md)
    with pytest.raises(ValueError, match=re.escape("prompt length 100 exceeds max_mask_len 64")):
        attn(q, kv, kv, md)


def test_host_slot_outside_the_pool_raises_index_error_before_the_launch():
    # the reference's index_copy_ raises IndexError for it (paged_kv_cache.py:68-69)
    kv = PagedKVCache(1, 4, 16, 8, 128, BF16, "cpu")
    k = torch.zeros(2, 8, 128, dtype=BF16)
    with pytest.raises(IndexError, match="out of bounds for dimension 0 with size 64"):
        kv.write(0, k, k, torch.tensor([3, 64], dtype=torch.long))
    with pytest.raises(IndexError, match="index -1 is out of bounds"):
        kv.write(0, k, k, torch.tensor([-1, 2], dtype=torch.long))


def test_host_context_longer_than_its_table_raises_missing_block():
    # BlockManager._physical_slot raises RuntimeError("missing block ...") (block_manager.py:194-205)
    attn = NpuPagedAttention(16, 8, 128)
    q = torch.zeros(2, 16, 128, dtype=BF16)
    kc = torch.zeros(4, 16, 8, 128, dtype=BF16)
    with pytest.raises(RuntimeError, match="missing block: context length 33 exceeds the 2-block table"):
        attn(q, kc, kc, torch.zeros(2, 2, dtype=torch.int32), torch.tensor([5, 33], dtype=torch.int32))
