"""Device-built decode metadata (nvk_decode_metadata via DeviceBlockTables)
is bit-identical to BlockManager.prepare_decode_metadata over a seeded script
of prefills with prefix hits, decode steps crossing block boundaries (q_len 1
and 3), frees and slot reuse, with two managers driven by the same
operations."""

import random

import numpy as np
import pytest
import torch

from nano_vllm_ascend_b200 import BlockManager
from nano_vllm_ascend_b200.device_metadata import DeviceBlockTables

pytestmark = pytest.mark.gpu


def test_device_decode_metadata_bit_exact_over_a_seeded_script(cuda_device):
    rnd = random.Random(7)
    bs, nb = 16, 4000
    host_bm, dev_bm = BlockManager(nb, bs, "cpu"), BlockManager(nb, bs, cuda_device)
    perm = list(range(nb))
    rnd.shuffle(perm)
    host_bm.free_block_ids = perm
    dev_bm.free_block_ids = perm
    dt = DeviceBlockTables(dev_bm, max_slots=64, max_blocks_per_seq=256, device=cuda_device)
    pos: dict[int, int] = {}
    for step in range(300):
        op = rnd.random()
        free_slots = [s for s in range(64) if s not in pos]
        if (op < 0.15 or not pos) and free_slots:  # prefill a new sequence (sometimes over a prefix)
            slot = rnd.choice(free_slots)
            n = rnd.randint(1, 300)
            prefix = []
            if pos and rnd.random() < 0.3:
                donor = rnd.choice(list(pos))
                prefix = host_bm.block_tables[donor][: rnd.randint(0, len(host_bm.block_tables[donor]))]
                n = max(n, len(prefix) * bs + 1)
            start = len(prefix) * bs
            for bm in (host_bm, dev_bm):
                bm.prepare_prefill_metadata([slot], [n - start], [start], [list(prefix)])
            pos[slot] = n
        elif op < 0.22 and len(pos) > 1:  # finish a sequence
            slot = rnd.choice(list(pos))
            for bm in (host_bm, dev_bm):
                bm.free_slot(slot)
            del pos[slot]
        else:  # one decode step of a random subset
            q_len = 3 if rnd.random() < 0.2 else 1
            slots = rnd.sample(list(pos), rnd.randint(1, len(pos)))
            starts = [pos[s] for s in slots]
            want = host_bm.prepare_decode_metadata(slots, starts, q_len)
            got = dt.prepare_decode_metadata(slots, starts, q_len)
            torch.cuda.synchronize()
            assert np.array_equal(got.block_tables.cpu().numpy(), want.block_tables.cpu().numpy()), step
            assert np.array_equal(got.context_lens.cpu().numpy(), want.context_lens.numpy()), step
            assert np.array_equal(got.slot_mapping.cpu().numpy(), want.slot_mapping.cpu().numpy()), step
            for s in slots:
                pos[s] += q_len
    assert int(dt.error_word.item()) == 0


def test_device_decode_metadata_padded_width(cuda_device):
    bm = BlockManager(64, 16, cuda_device)
    bm.prepare_prefill_metadata([0, 1], [40, 5], [0, 0], [[], []])
    dt = DeviceBlockTables(bm, 4, 32, cuda_device)
    md = dt.prepare_decode_metadata([0, 1], [40, 5], 1, width=32)
    t = md.block_tables.cpu()
    assert t.shape == (2, 32) and int(t[0, 3:].abs().sum()) == 0 and int(t[1, 1:].abs().sum()) == 0
    assert t[0, :3].tolist() == bm.block_tables[0] and t[1, :1].tolist() == bm.block_tables[1]


def test_device_decode_metadata_back_to_back_steps_without_sync(cuda_device):
    """Twelve steps queued with no synchronisation in between (more than the
    pinned staging buffers, so each is reused while earlier copies may be in
    flight); every step's tensors still hold that step's metadata."""
    bs = 16
    host_bm, dev_bm = BlockManager(512, bs, "cpu"), BlockManager(512, bs, cuda_device)
    ctx = [5, 17, 31, 16, 1, 47, 64, 3]
    slots = list(range(len(ctx)))
    for bm in (host_bm, dev_bm):
        bm.prepare_prefill_metadata(slots, ctx, [0] * len(ctx), [[] for _ in slots])
    dt = DeviceBlockTables(dev_bm, 16, 64, cuda_device)
    wants, gots = [], []
    for step in range(12):
        starts = [c + step for c in ctx]
        wants.append(host_bm.prepare_decode_metadata(slots, starts, 1))
        gots.append(dt.prepare_decode_metadata(slots, starts, 1, width=16))
    torch.cuda.synchronize()
    for step, (want, got) in enumerate(zip(wants, gots)):
        w = want.block_tables.cpu()
        assert torch.equal(got.block_tables.cpu()[:, : w.shape[1]], w), step
        assert int(got.block_tables.cpu()[:, w.shape[1]:].abs().sum()) == 0, step
        assert torch.equal(got.context_lens.cpu(), want.context_lens.cpu()), step
        assert torch.equal(got.slot_mapping.cpu(), want.slot_mapping.cpu()), step


def test_device_decode_metadata_rejected_step_then_recovers(cuda_device):
    """A slot outside the mirror raises ValueError before any device work; the
    steps after it still match the host path (whole tables are re-sent)."""
    bs = 16
    host_bm, dev_bm = BlockManager(64, bs, "cpu"), BlockManager(64, bs, cuda_device)
    for bm in (host_bm, dev_bm):
        bm.prepare_prefill_metadata([0, 1, 5], [40, 5, 3], [0, 0, 0], [[], [], []])
    dt = DeviceBlockTables(dev_bm, 4, 32, cuda_device)
    dt.prepare_decode_metadata([0, 1], [40, 5], 1)
    host_bm.prepare_decode_metadata([0, 1], [40, 5], 1)
    with pytest.raises(ValueError, match="outside the device mirror"):
        dt.prepare_decode_metadata([0, 5], [41, 3], 1)
    host_bm.prepare_decode_metadata([0, 5], [41, 3], 1)  # the same allocator bookkeeping
    want = host_bm.prepare_decode_metadata([1, 0], [6, 48], 1)
    got = dt.prepare_decode_metadata([1, 0], [6, 48], 1)
    torch.cuda.synchronize()
    assert torch.equal(got.block_tables.cpu(), want.block_tables.cpu())
    assert torch.equal(got.context_lens.cpu(), want.context_lens.cpu())
    assert torch.equal(got.slot_mapping.cpu(), want.slot_mapping.cpu())
    assert int(dt.error_word.item()) == 0


def test_device_decode_metadata_slot_named_twice(cuda_device):
    """A batch that names a sequence slot twice (with new table entries to
    send) gives both rows the host path's values: the slot's final length and
    whole table (BlockManager.prepare_decode_metadata runs every row's
    ensure_blocks and seq_lens update before building any tensor)."""
    bs = 16
    host_bm, dev_bm = BlockManager(64, bs, "cpu"), BlockManager(64, bs, cuda_device)
    for bm in (host_bm, dev_bm):
        bm.prepare_prefill_metadata([0, 1], [31, 5], [0, 0], [[], []])
    dt = DeviceBlockTables(dev_bm, 4, 32, cuda_device)
    for starts in ([31, 32, 5], [47, 48, 6]):  # the first step sends whole tables, the second a new block
        want = host_bm.prepare_decode_metadata([0, 0, 1], starts, 1)
        got = dt.prepare_decode_metadata([0, 0, 1], starts, 1)
        torch.cuda.synchronize()
        assert torch.equal(got.block_tables.cpu(), want.block_tables.cpu())
        assert torch.equal(got.context_lens.cpu(), want.context_lens.cpu())
        assert torch.equal(got.slot_mapping.cpu(), want.slot_mapping.cpu())
    assert int(dt.error_word.item()) == 0


def test_device_decode_metadata_rewinds_and_repeats_over_a_seeded_script(cuda_device):
    """The seeded script again, now also with rows decoded behind their
    sequence's length (the host path then reports seq_lens, not start + q_len)
    and slots named twice in a batch."""
    rnd = random.Random(11)
    bs, nb = 16, 4000
    host_bm, dev_bm = BlockManager(nb, bs, "cpu"), BlockManager(nb, bs, cuda_device)
    perm = list(range(nb))
    rnd.shuffle(perm)
    host_bm.free_block_ids = perm
    dev_bm.free_block_ids = perm
    dt = DeviceBlockTables(dev_bm, max_slots=32, max_blocks_per_seq=128, device=cuda_device)
    pos: dict[int, int] = {}
    for step in range(200):
        free_slots = [s for s in range(32) if s not in pos]
        if (rnd.random() < 0.15 or not pos) and free_slots:
            slot = rnd.choice(free_slots)
            n = rnd.randint(1, 200)
            for bm in (host_bm, dev_bm):
                bm.prepare_prefill_metadata([slot], [n], [0], [[]])
            pos[slot] = n
            continue
        q_len = 2 if rnd.random() < 0.2 else 1
        slots = rnd.sample(list(pos), rnd.randint(1, len(pos)))
        starts = [pos[s] for s in slots]
        if rnd.random() < 0.3:
            j = rnd.randrange(len(slots))
            slots.append(slots[j])
            starts.append(starts[j] + q_len)
        if rnd.random() < 0.3:
            j = rnd.randrange(len(slots))
            starts[j] = max(0, starts[j] - rnd.randint(1, 40))
        want = host_bm.prepare_decode_metadata(slots, starts, q_len)
        got = dt.prepare_decode_metadata(slots, starts, q_len)
        torch.cuda.synchronize()
        assert np.array_equal(got.block_tables.cpu().numpy(), want.block_tables.cpu().numpy()), step
        assert np.array_equal(got.context_lens.cpu().numpy(), want.context_lens.numpy()), step
        assert np.array_equal(got.slot_mapping.cpu().numpy(), want.slot_mapping.cpu().numpy()), step
        for s, st in zip(slots, starts):
            pos[s] = max(pos[s], st + q_len)
    assert int(dt.error_word.item()) == 0
