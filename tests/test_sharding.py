"""Multi-GPU partitioning host logic, run as two gloo ranks on the CPU.

* sequence sharding: the ranks' slices cover the batch exactly once, and each
  rank's independent BlockManager produces the same per-sequence tables as a
  single manager would for that slice;
* KV-head sharding: each rank computes attention for its KV heads with the
  oracle, the outputs are all-gathered (gather_head_shards) and must equal the
  single-process result over all heads, in query-head order.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from nano_vllm_ascend_b200.sharding import gather_head_shards, kv_head_shard, sequence_shard, token_balanced_shard
from oracle import paged_kv_oracle as orc


def test_token_balanced_shard_partitions_and_balances():
    g = torch.Generator().manual_seed(0)
    for n, w in ((256, 8), (256, 2), (7, 3), (3, 4), (0, 2)):
        lens = torch.randint(2048, 6145, (n,), generator=g).tolist()
        parts = [token_balanced_shard(lens, w, r) for r in range(w)]
        assert sorted(i for p in parts for i in p) == list(range(n))
        assert all(p == sorted(p) for p in parts)
        totals = [sum(lens[i] for i in p) for p in parts]
        if n:
            assert max(totals) - min(totals) <= max(lens)
        assert parts == [token_balanced_shard(lens, w, r) for r in range(w)]  # deterministic
    lens = torch.randint(2048, 6145, (256,), generator=torch.Generator().manual_seed(0)).tolist()
    totals = [sum(lens[i] for i in token_balanced_shard(lens, 8, r)) for r in range(8)]
    assert max(totals) / min(totals) < 1.01  # the contiguous split of the same batch is ~10 % apart
    with pytest.raises(ValueError):
        token_balanced_shard([1, 2], 2, 2)


def test_sequence_shard_partitions_exactly():
    for n in (0, 1, 7, 256, 257):
        for w in (1, 2, 3, 4, 8):
            got = [i for r in range(w) for i in sequence_shard(n, w, r)]
            assert got == list(range(n))
            sizes = [len(sequence_shard(n, w, r)) for r in range(w)]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        sequence_shard(4, 2, 2)


def test_kv_head_shard_ranges():
    assert kv_head_shard(32, 8, 8, 3) == (range(3, 4), range(12, 16))
    assert kv_head_shard(32, 8, 2, 1) == (range(4, 8), range(16, 32))
    with pytest.raises(ValueError):
        kv_head_shard(32, 8, 3, 0)


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(0)
        b, h, kvh, d, nb, bs = 3, 32, 8, 128, 12, 16
        q = torch.randn(b, h, d, generator=g)
        kc = torch.randn(nb, bs, kvh, d, generator=g)
        vc = torch.randn(nb, bs, kvh, d, generator=g)
        tables = torch.tensor([[0, 1, 2], [3, 4, 0], [5, 0, 0]])
        ctx = np.array([40, 20, 7])
        kv_range, q_range = kv_head_shard(h, kvh, world, rank)
        local = orc.paged_decode(q[:, q_range.start:q_range.stop].numpy(),
                                 kc[:, :, kv_range.start:kv_range.stop].numpy(),
                                 vc[:, :, kv_range.start:kv_range.stop].numpy(), tables.numpy(), ctx, 0.1)
        full = gather_head_shards(torch.from_numpy(local))
        want = orc.paged_decode(q.numpy(), kc.numpy(), vc.numpy(), tables.numpy(), ctx, 0.1)
        ok_heads = bool(np.allclose(full.numpy(), want, atol=1e-5))

        # sequence sharding with independent managers
        from nano_vllm_ascend_b200 import BlockManager

        lens = [37, 128, 255, 513, 4, 90, 700]
        mine = sequence_shard(len(lens), world, rank)
        bm = BlockManager(num_blocks=64, block_size=128, device="cpu")
        md = bm.prepare_prefill_metadata(list(mine), [lens[i] for i in mine], [0] * len(mine),
                                         [[] for _ in mine])
        counts = torch.tensor([len(mine)])
        dist.all_reduce(counts)
        result_q.put((rank, ok_heads, int(counts.item()), md.context_lens.tolist()))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_gather_heads_and_shard_sequences():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    results.sort()
    assert all(ok for _, ok, _, _ in results)
    assert all(c == 7 for _, _, c, _ in results)
    assert results[0][3] + results[1][3] == [37, 128, 255, 513, 4, 90, 700]
