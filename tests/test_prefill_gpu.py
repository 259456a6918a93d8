"""Parity of the tcgen05 prefill kernel (through the C ABI) with the fp32 oracle.

Bottom-right causal attention of each sequence's new queries over its paged KV
(cached prefix + the rows appended this step) or over contiguous K/V (dense
mode), within max-abs 2e-2 / max-rel 1e-2: config-3 shapes (768 cached + 256
new), ragged q/kv lengths (1, 127, 128, 129, ...), GQA ratios 1/2/4/8, rows that
see no key, and the reference's prefix-cache flow end to end through
BlockManager -> PagedKVCache.write -> BatchPrefillAttention.
"""

import numpy as np
import pytest
import torch

from nano_vllm_ascend_b200 import BatchPrefillAttention, BlockManager, PagedKVCache, ops
from oracle import paged_kv_oracle as orc
from tests.helpers import assert_close, bits, random_pool, seeded_tables

pytestmark = pytest.mark.gpu


def run_paged(dev, q_lens, kv_lens, h=16, kvh=8, seed=0):
    nb = sum((n + 127) // 128 for n in kv_lens) + 2
    kc, vc = random_pool(nb, 128, kvh, 128, dev, seed)
    tables = seeded_tables(kv_lens, 128, nb, seed).to(dev)
    cu = np.concatenate([[0], np.cumsum(q_lens)]).astype(np.int32)
    g = torch.Generator(device=dev).manual_seed(seed + 7)
    q = torch.randn(int(cu[-1]), h, 128, generator=g, device=dev).to(torch.bfloat16)
    out = torch.full_like(q, float("nan"))
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    ops.paged_prefill(out, q, kc, vc, tables, torch.from_numpy(cu).to(dev),
                      torch.tensor(kv_lens, dtype=torch.int32, device=dev), max(q_lens), 128 ** -0.5, err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    want = orc.paged_prefill(bits(q), bits(kc), bits(vc), tables.cpu().numpy(), cu, np.array(kv_lens), 128 ** -0.5)
    return out.float().cpu().numpy(), want


def test_prefill_config3_shape(cuda_device):
    # 4 of the 32 config-3 requests: 768 cached prefix + 256 new tokens
    got, want = run_paged(cuda_device, [256] * 4, [1024] * 4)
    assert_close(got, want, "config3")


@pytest.mark.parametrize("q_lens,prefix", [
    ([1, 77, 128, 129, 300], [0, 128, 640, 5, 1000]),
    ([255, 3, 384], [1, 0, 129]),
    ([128], [0]),
])
def test_prefill_ragged(cuda_device, q_lens, prefix):
    kv = [p + n for p, n in zip(prefix, q_lens)]
    got, want = run_paged(cuda_device, q_lens, kv, seed=len(q_lens))
    assert_close(got, want, f"ragged {q_lens}")


@pytest.mark.parametrize("h,kvh", [(8, 8), (32, 8), (64, 8), (16, 2)])
def test_prefill_gqa(cuda_device, h, kvh):
    got, want = run_paged(cuda_device, [200, 64], [700, 64], h=h, kvh=kvh, seed=h)
    assert_close(got, want, f"h={h} kvh={kvh}")


def test_prefill_rows_without_visible_keys_are_zero(cuda_device):
    # kv shorter than q: the first Lq - Lk rows see no key
    got, want = run_paged(cuda_device, [200], [150], seed=5)
    assert np.all(got[:50] == 0)
    assert_close(got, want, "kv < q")


def test_dense_prefill_matches_oracle(cuda_device):
    dev = cuda_device
    lens = [300, 1, 128, 77]
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    g = torch.Generator(device=dev).manual_seed(3)
    t = int(cu[-1])
    q = torch.randn(t, 16, 128, generator=g, device=dev).to(torch.bfloat16)
    k = torch.randn(t, 8, 128, generator=g, device=dev).to(torch.bfloat16)
    v = torch.randn(t, 8, 128, generator=g, device=dev).to(torch.bfloat16)
    out = torch.empty_like(q)
    cu_t = torch.from_numpy(cu).to(dev)
    ops.dense_prefill(out, q, k, v, cu_t, cu_t, max(lens), 128 ** -0.5)
    torch.cuda.synchronize()
    want = orc.dense_prefill(bits(q), bits(k), bits(v), cu, cu, 128 ** -0.5)
    assert_close(out.float().cpu().numpy(), want, "dense")


def test_prefix_cache_flow_through_host_classes(cuda_device):
    """Reference flow (model_runner.py:146-238): prompt 1 fills and caches
    its blocks; prompt 2 shares a 768-token prefix, hits 6 cached blocks,
    appends only its 256-token suffix and attends over prefix + suffix."""
    dev = cuda_device
    bs, kvh, h, nb = 128, 8, 16, 32
    bm = BlockManager(nb, bs, dev)
    kv = PagedKVCache(1, nb, bs, kvh, 128, torch.bfloat16, dev)
    attn = BatchPrefillAttention(h, kvh, 128, bs, max_mask_len=2048)
    g = torch.Generator().manual_seed(11)
    prefix = torch.randint(0, 1000, (768,), generator=g)
    p1 = torch.cat([prefix, torch.randint(1000, 2000, (256,), generator=g)])
    p2 = torch.cat([prefix, torch.randint(2000, 3000, (256,), generator=g)])
    gd = torch.Generator(device=dev).manual_seed(12)

    def kv_rows(n):
        return (torch.randn(n, kvh, 128, generator=gd, device=dev).to(torch.bfloat16),
                torch.randn(n, kvh, 128, generator=gd, device=dev).to(torch.bfloat16))

    # prompt 1: no hit, dense mode
    md1 = bm.prepare_prefill_metadata([0], [1024], [0], [[]])
    assert not md1.use_paged_prefill
    k1, v1 = kv_rows(1024)
    kv.write(0, k1, v1, md1.slot_mapping)
    q1 = torch.randn(1024, h, 128, generator=gd, device=dev).to(torch.bfloat16)
    kc, vc = kv.get_physical_cache(0)
    out1 = attn(q1, k1, v1, md1, kc, vc)
    bm.cache_full_blocks(slot=0, token_ids=p1, num_cached_blocks=0, num_full_blocks=8)

    # prompt 2: 6 cached prefix blocks, paged mode over prefix + new suffix
    hit = bm.find_longest_prefix_blocks(p2, max_cache_blocks=7)
    assert len(hit) == 6 and hit == md1.block_tables[0, :6].tolist()
    md2 = bm.prepare_prefill_metadata([1], [256], [768], [hit])
    assert md2.use_paged_prefill and md2.context_lens.tolist() == [1024]
    k2, v2 = kv_rows(256)
    kv.write(0, k2, v2, md2.slot_mapping)
    q2 = torch.randn(256, h, 128, generator=gd, device=dev).to(torch.bfloat16)
    out2 = attn(q2, k2, v2, md2, kc, vc)
    torch.cuda.synchronize()

    cu1 = np.array([0, 1024], np.int32)
    want1 = orc.dense_prefill(bits(q1), bits(k1), bits(v1), cu1, cu1, 128 ** -0.5)
    assert_close(out1.float().cpu().numpy(), want1, "prompt 1 (dense)")
    # oracle for prompt 2 from the explicit rows: prefix K/V of prompt 1 + suffix of prompt 2
    kfull = torch.cat([k1[:768], k2]).cpu()
    vfull = torch.cat([v1[:768], v2]).cpu()
    want2 = orc.dense_prefill(bits(q2), bits(kfull), bits(vfull), np.array([0, 256], np.int32),
                              np.array([0, 1024], np.int32), 128 ** -0.5)
    assert_close(out2.float().cpu().numpy(), want2, "prompt 2 (paged, prefix hit)")
    # and the paged oracle over the pool agrees
    want2p = orc.paged_prefill(bits(q2), bits(kc), bits(vc), md2.block_tables.cpu().numpy(),
                               np.array([0, 256]), np.array([1024]), 128 ** -0.5)
    assert_close(out2.float().cpu().numpy(), want2p, "prompt 2 vs paged oracle")
