"""BlockManager parity with the reference (CPU only).

The first three tests restate the reference's own unit tests
(tests/test_block_manager.py:6-54 in Pla-Yer/nano_vllm_ascend); the rest
replay scenarios whose outputs were recorded from the reference's
BlockManager by tests/golden/make_golden.py and require bit-identical block
tables, context lengths, slot mappings, prefix lookups, free-queue order,
reference counts and errors.
"""

import json
from pathlib import Path

import pytest
import torch

from nano_vllm_ascend_b200.block_manager import BlockManager
from tests.golden.make_golden import _md, config1, run_script, unit_scenarios

GOLDEN = json.loads((Path(__file__).parent / "golden" / "block_manager_golden.json").read_text())


def test_prefill_metadata_cumulative_lengths_and_slots():
    manager = BlockManager(num_blocks=8, block_size=4, device="cpu")
    md = manager.prepare_prefill_metadata(slots=[0, 1, 2], seq_lens=[3, 5, 2], start_positions=[0, 0, 0],
                                          prefix_block_ids=[[], [], []])
    assert md.actual_seq_lengths_q == [3, 8, 10]
    assert md.actual_seq_lengths_kv == [3, 8, 10]
    assert md.context_lens.tolist() == [3, 5, 2]
    assert md.slot_mapping.tolist() == [0, 1, 2, 4, 5, 6, 7, 8, 12, 13]


def test_decode_metadata_for_active_slots_and_positions():
    manager = BlockManager(num_blocks=8, block_size=4, device="cpu")
    manager.prepare_prefill_metadata(slots=[0, 1, 2], seq_lens=[3, 5, 2], start_positions=[0, 0, 0],
                                     prefix_block_ids=[[], [], []])
    md = manager.prepare_decode_metadata(slots=[1, 2], start_positions=[5, 2], q_len=1)
    assert md.context_lens.tolist() == [6, 3]
    assert md.slot_mapping.tolist() == [9, 14]


def test_prefix_cache_reuses_full_blocks():
    manager = BlockManager(num_blocks=8, block_size=4, device="cpu")
    token_ids = torch.tensor([10, 11, 12, 13, 20, 21], dtype=torch.long)
    manager.prepare_prefill_metadata(slots=[0], seq_lens=[6], start_positions=[0], prefix_block_ids=[[]])
    manager.cache_full_blocks(slot=0, token_ids=token_ids)
    manager.free_slot(0)
    assert manager.find_longest_prefix_blocks(token_ids, max_cache_blocks=1) == [0]


def test_unit_scenarios_match_reference_golden():
    assert unit_scenarios(BlockManager) == GOLDEN["unit"]


def test_config1_tables_and_slots_match_reference_golden():
    got = config1(BlockManager)
    assert got == GOLDEN["config1"]
    # dtype/device contract of the metadata (block_manager.py:207-250)
    assert got["decode"]["block_tables_dtype"] == "torch.int32"
    assert got["decode"]["context_lens_device"] == "cpu"
    assert got["decode"]["slot_mapping_dtype"] == "torch.int64"


def test_random_script_matches_reference_golden():
    sc = GOLDEN["script"]
    got = run_script(BlockManager, sc["ops"], sc["num_blocks"], sc["block_size"])
    assert len(got) == len(sc["results"])
    for i, (g, r) in enumerate(zip(got, sc["results"])):
        assert g == r, f"step {i} ({sc['ops'][i]['op']}) differs"
    # the script must actually exercise prefix hits and errors
    assert any(r.get("cached") for r in sc["results"] if r["op"] == "admit")
    assert any("error" in r for r in sc["results"])


def test_errors_match_reference_types():
    bm = BlockManager(num_blocks=2, block_size=4, device="cpu")
    with pytest.raises(RuntimeError, match="out of free blocks"):
        bm.prepare_prefill_metadata(slots=[0], seq_lens=[9], start_positions=[0], prefix_block_ids=[[]])
    bm = BlockManager(num_blocks=2, block_size=4, device="cpu")
    bm._init_slot(5, 0, [])
    with pytest.raises(RuntimeError, match="missing block: slot=5, logical_pos=0"):
        bm.get_slot_mapping([5], [0], [1])
    with pytest.raises(ValueError, match="length mismatch"):
        bm.prepare_decode_metadata(slots=[5], start_positions=[0, 1], q_len=1)
    with pytest.raises(RuntimeError, match="underflow"):
        bm._release_block(1)
    with pytest.raises(RuntimeError, match="active sequences"):
        bm.clear_prefix_cache()


def test_chain_keys_are_garbage_collected_with_their_blocks():
    bm = BlockManager(num_blocks=4, block_size=2, device="cpu")
    toks = torch.tensor([1, 2, 3, 4, 5], dtype=torch.long)
    bm.prepare_prefill_metadata(slots=[0], seq_lens=[5], start_positions=[0], prefix_block_ids=[[]])
    bm.cache_full_blocks(slot=0, token_ids=toks)
    assert len(bm._keys) == 2 and bm.num_cached_keys() == 2
    bm.free_slot(0)
    # reuse every physical block: their keys are forgotten and, with no
    # holder and no child left, dropped from the intern table
    bm.prepare_prefill_metadata(slots=[1], seq_lens=[8], start_positions=[0], prefix_block_ids=[[]])
    assert bm.num_cached_keys() == 0 and len(bm._keys) == 0


def test_free_queue_setter_permutes_allocation_order():
    bm = BlockManager(num_blocks=4, block_size=2, device="cpu")
    bm.free_block_ids = [3, 1, 0, 2]
    md = bm.prepare_prefill_metadata(slots=[0], seq_lens=[5], start_positions=[0], prefix_block_ids=[[]])
    assert md.block_tables.tolist() == [[3, 1, 0]]
    assert bm.free_block_ids == [2]
    assert _md(md)["slot_mapping"] == [6, 7, 2, 3, 0]


@pytest.mark.parametrize("seed", [1, 2, 3, 4, 5])
def test_native_prefix_index_matches_python_side_by_side(seed):
    """The C++ prefix index (nvk_prefix_*) and the Python one give identical
    observable behaviour on seeded scripts with shared prefixes, decode steps,
    frees, block reuse and cache clears."""
    from functools import partial

    from tests.golden.make_golden import random_script

    ops = random_script(seed, num_blocks=48, block_size=4, steps=250)
    native = run_script(partial(BlockManager, native_prefix=True), ops, 48, 4)
    python = run_script(partial(BlockManager, native_prefix=False), ops, 48, 4)
    assert native == python
    assert any(r.get("cached") for r in native if r["op"] == "admit")


def test_native_prefix_index_keys_track_block_reuse():
    for native in (True, False):
        bm = BlockManager(num_blocks=6, block_size=2, device="cpu", native_prefix=native)
        a = torch.tensor([1, 2, 3, 4, 5, 6, 7], dtype=torch.long)
        bm.prepare_prefill_metadata(slots=[0], seq_lens=[7], start_positions=[0], prefix_block_ids=[[]])
        bm.cache_full_blocks(slot=0, token_ids=a)
        assert bm.num_cached_keys() == 3 and len(bm._keys) == 3
        bm.free_slot(0)
        assert bm.find_longest_prefix_blocks(a, max_cache_blocks=3) == [0, 1, 2]
        # a second prompt sharing two blocks
        b = torch.tensor([1, 2, 3, 4, 9, 9], dtype=torch.long)
        hit = bm.find_longest_prefix_blocks(b, max_cache_blocks=2)
        assert hit == [0, 1]
        bm.prepare_prefill_metadata(slots=[1], seq_lens=[2], start_positions=[4], prefix_block_ids=[hit])
        bm.cache_full_blocks(slot=1, token_ids=b, num_cached_blocks=2)
        assert bm.num_cached_keys() == 4
        bm.free_slot(1)
        bm.clear_prefix_cache()
        assert bm.num_cached_keys() == 0 and len(bm._keys) == 0
        assert all(blk.block_hash is None for blk in bm.blocks)
