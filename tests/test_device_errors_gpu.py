"""Device-side errors surface through the drop-in classes with the
reference's exception types (device_errors):

* a device slot_mapping entry outside the pool (PagedKVCache.write, and the
  fused append of a decode graph) -> IndexError, as the reference's
  index_copy_ raises (src/nanovllm_ascend/npu/paged_kv_cache.py:68-69);
* a device context length longer than its block-table row ->
  RuntimeError("missing block ..."), as BlockManager._physical_slot raises
  (src/nanovllm_ascend/npu/block_manager.py:194-205);
* a block id outside the pool (decode and prefill) -> RuntimeError.

Each flagged call raises at check_errors(), or, without it, on a later call
once the non-blocking read has landed; the error is cleared when raised, so
the next good call runs clean and matches the oracle. Nothing here faults:
the kernels read a bad block as zeros and skip a bad slot.
"""

import numpy as np
import pytest
import torch

from nano_vllm_ascend_b200 import (BatchPrefillAttention, BlockManager, DecodeGraphRunner, PagedAttention,
                                   PagedKVCache, device_errors)
from nano_vllm_ascend_b200.device_errors import KVCacheDeviceError, check_errors
from oracle import paged_kv_oracle as orc
from tests.helpers import assert_close, bits, random_pool, seeded_tables

pytestmark = pytest.mark.gpu
D = 128
SCALE = D ** -0.5


@pytest.fixture(autouse=True)
def clean_state(cuda_device):
    try:
        check_errors(cuda_device)
    except KVCacheDeviceError:
        pass
    yield


def test_write_with_a_device_slot_outside_the_pool_raises_index_error(cuda_device):
    kv = PagedKVCache(2, 8, 128, 8, D, torch.bfloat16, cuda_device)
    kv.key_cache.zero_()
    k = torch.ones(3, 8, D, dtype=torch.bfloat16, device=cuda_device)
    kv.write(1, k, k, torch.tensor([5, 8 * 128 + 7, 9], dtype=torch.int64, device=cuda_device))
    with pytest.raises(IndexError, match="slot_mapping entry is out of bounds"):
        check_errors(cuda_device)
    # the good rows landed, the bad one was skipped; the error is cleared
    flat = kv.key_cache[1].view(-1, 8, D)
    assert bool((flat[5] == 1).all()) and bool((flat[9] == 1).all()) and int((flat != 0).sum()) == 2 * 8 * D
    check_errors(cuda_device)


def test_a_flagged_append_raises_on_a_later_call_without_check(cuda_device):
    kv = PagedKVCache(1, 8, 128, 8, D, torch.bfloat16, cuda_device)
    k = torch.ones(1, 8, D, dtype=torch.bfloat16, device=cuda_device)
    kv.write(0, k, k, torch.tensor([-3], dtype=torch.int64, device=cuda_device))
    torch.cuda.synchronize()  # the non-blocking read of the error word has landed
    with pytest.raises(IndexError):
        kv.write(0, k, k, torch.tensor([0], dtype=torch.int64, device=cuda_device))
    check_errors(cuda_device)  # raised once, then clear


def _decode_inputs(dev, ctx, seed=0, nb=None):
    nb = nb or sum((n + 127) // 128 for n in ctx) + 4
    kc, vc = random_pool(nb, 128, 8, D, dev, seed)
    tables = seeded_tables(ctx, 128, nb, seed, width=32).to(dev)
    g = torch.Generator(device=dev).manual_seed(seed + 1)
    q = torch.randn(len(ctx), 16, D, generator=g, device=dev).to(torch.bfloat16)
    return q, kc, vc, tables


def test_decode_with_a_bad_block_id_raises_then_recovers(cuda_device):
    ctx = [300, 1000, 17]
    q, kc, vc, tables = _decode_inputs(cuda_device, ctx)
    attn = PagedAttention(16, 8, D)
    bad = tables.clone()
    bad[1, 3] = kc.shape[0] + 11
    ctx_t = torch.tensor(ctx, dtype=torch.int32, device=cuda_device)
    attn(q, kc, vc, bad, ctx_t)
    with pytest.raises(RuntimeError, match="block-table entry is outside the KV pool") as info:
        check_errors(cuda_device)
    assert info.value.bits & device_errors.BAD_BLOCK_ID
    out = attn(q, kc, vc, tables, ctx_t)
    check_errors(cuda_device)
    want = orc.paged_decode(bits(q), bits(kc), bits(vc), tables.cpu().numpy(), np.array(ctx), SCALE)
    assert_close(out.float().cpu().numpy(), want, "decode after a flagged call")


def test_decode_with_a_device_context_longer_than_the_table_raises_missing_block(cuda_device):
    ctx = [300, 200]
    q, kc, vc, tables = _decode_inputs(cuda_device, ctx)
    attn = PagedAttention(16, 8, D)
    narrow = tables[:, :2].contiguous()  # 256 tokens of table for a 300-token context
    attn(q, kc, vc, narrow, torch.tensor(ctx, dtype=torch.int32, device=cuda_device))
    with pytest.raises(RuntimeError, match="missing block"):
        check_errors(cuda_device)


def test_paged_prefill_with_a_bad_block_id_raises(cuda_device):
    dev = cuda_device
    nb = 16
    bm = BlockManager(nb, 128, dev)
    md = bm.prepare_prefill_metadata([0], [200], [0], [[]])
    md.use_paged_prefill = True  # attend over the pool through the table
    md.block_tables = md.block_tables.clone()
    md.block_tables[0, 1] = nb + 2
    kv = PagedKVCache(1, nb, 128, 8, D, torch.bfloat16, dev)
    g = torch.Generator(device=dev).manual_seed(4)
    q = torch.randn(200, 16, D, generator=g, device=dev).to(torch.bfloat16)
    k = torch.randn(200, 8, D, generator=g, device=dev).to(torch.bfloat16)
    attn = BatchPrefillAttention(16, 8, D, 128, max_mask_len=4096)
    kc, vc = kv.get_physical_cache(0)
    attn(q, k, k, md, kc, vc)
    with pytest.raises(RuntimeError, match="block-table entry is outside the KV pool"):
        check_errors(dev)


class OneLayer:
    def __init__(self, q, k, v):
        self.q, self.k, self.v = q, k, v
        self.attn = PagedAttention(q.shape[1], k.shape[1], D)

    def __call__(self, input_ids_flat, position_ids_flat, kv_cache, attn_metadata, is_prefill=False):
        kv_cache.write(0, self.k, self.v, attn_metadata.slot_mapping)
        kc, vc = kv_cache.get_physical_cache(0)

        class Out:
            logits = self.attn(self.q, kc, vc, attn_metadata.block_tables, attn_metadata.context_lens)

        return Out()


def test_graph_replay_with_a_wrong_fused_append_slot_raises_on_the_next_call(cuda_device):
    dev = cuda_device
    ctx = [400, 129]
    nb = 16
    bm = BlockManager(nb, 128, dev)
    bm.prepare_prefill_metadata([0, 1], ctx, [0, 0], [[], []])
    md = bm.prepare_decode_metadata([0, 1], ctx, q_len=1)
    kv = PagedKVCache(1, nb, 128, 8, D, torch.bfloat16, dev)
    kv.key_cache.normal_()
    kv.value_cache.normal_()
    g = torch.Generator(device=dev).manual_seed(8)
    model = OneLayer(*(torch.randn(2, h, D, generator=g, device=dev).to(torch.bfloat16) for h in (16, 8, 8)))
    runner = DecodeGraphRunner(model, kv, batch_sizes=[2], max_model_len=1024, block_size=128, device=dev)
    ids = torch.zeros(2, dtype=torch.long, device=dev)
    pos = torch.tensor(ctx, dtype=torch.long, device=dev)
    try:
        assert runner.forward(ids, pos, md) is not None
        check_errors(dev)
        wrong = type(md)(block_tables=md.block_tables, context_lens=md.context_lens,
                         slot_mapping=md.slot_mapping + 1)  # not each sequence's last position
        runner.forward(ids, pos, wrong)
        torch.cuda.synchronize()
        with pytest.raises(IndexError):
            runner.forward(ids, pos, md)
        assert runner.forward(ids, pos, md) is not None
        check_errors(dev)
    finally:
        runner.release()
