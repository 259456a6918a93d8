"""The per-rank workloads bench.py times (CPU only).

* weak scaling (configs 2 and 3 replicas): every rank decodes the same
  per-GPU context lengths, so per-GPU work is fixed as the GPU count grows;
  one rank's lengths are those of the single-GPU run;
* strong scaling (config 4): the ranks' sequences partition the one batch
  exactly, and their KV token totals differ by at most one sequence's length.
"""

import pytest

import bench


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_weak_scaling_ranks_share_the_single_gpu_lengths(world):
    wl = bench.WORKLOADS["decode_c2"]
    single = bench.rank_contexts(wl, 1, 0)
    assert len(single) == wl.batch and all(wl.ctx_lo <= c <= wl.ctx_hi for c in single)
    for rank in range(world):
        assert bench.rank_contexts(wl, world, rank) == single


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_strong_scaling_ranks_partition_the_batch_by_tokens(world):
    wl = bench.WORKLOADS["decode_c4"]
    whole = bench.rank_contexts(wl, 1, 0)
    parts = [bench.rank_contexts(wl, world, r) for r in range(world)]
    assert sorted(c for p in parts for c in p) == sorted(whole)
    totals = [sum(p) for p in parts]
    assert max(totals) - min(totals) <= max(whole)
    cfg = bench.decode_config(wl, world)
    assert cfg["global_batch"] == wl.batch
