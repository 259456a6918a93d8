"""Host side of DeviceBlockTables on the CPU: the allocator bookkeeping, the
update lists, the staged input layout and the per-row lengths, checked
against BlockManager.prepare_decode_metadata (the reference's host path,
src/nanovllm_ascend/npu/block_manager.py:304-328) over seeded scripts with
rewinds and repeated slots. The device entry point is replaced by a
stand-in that reads the staged arrays through their raw pointers and
follows the contract that include/nvk_paged_kv.h states for
nvk_decode_metadata; the GPU tests run the real kernel."""

import ctypes
import random
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from nano_vllm_ascend_b200 import BlockManager
from nano_vllm_ascend_b200 import device_metadata as dm


def _view(ptr: int, n: int, dtype) -> np.ndarray:
    if n == 0:
        return np.zeros(0, dtype)
    ctype = np.ctypeslib.as_ctypes_type(dtype)
    return np.ctypeslib.as_array(ctypes.cast(ptr, ctypes.POINTER(ctype)), (n,))


def _stand_in(mirror, stride, rows, slots, starts, row_ctx, row_blocks, batch, q_len, bs, offsets, idx, blk,
              tables, out_stride, width, ctx_out, slot_out, err, stream):
    """nvk_decode_metadata as its header describes it, on host memory."""
    s = _view(slots, batch, np.int32)
    st = _view(starts, batch, np.int64)
    off = _view(offsets, batch + 1, np.int32)
    m = int(off[-1]) if batch else 0
    ui, ub = _view(idx, m, np.int32), _view(blk, m, np.int32)
    rc, rb = _view(row_ctx, batch, np.int32), _view(row_blocks, batch, np.int32)
    mir = _view(mirror, rows * stride, np.int32).reshape(rows, stride)
    tab = _view(tables, batch * out_stride, np.int32).reshape(batch, out_stride)
    cl, sm = _view(ctx_out, batch, np.int32), _view(slot_out, batch * q_len, np.int64)
    for b in range(batch):
        row, start = int(s[b]), int(st[b])
        end, ctx, nblk = start + q_len, int(rc[b]), int(rb[b])
        assert 0 <= row < rows and ctx >= end and nblk * bs >= end and nblk <= min(stride, width)
        for u in range(off[b], off[b + 1]):
            mir[row, ui[u]] = ub[u]
        tab[b, :width] = 0
        tab[b, :nblk] = mir[row, :nblk]
        cl[b] = ctx
        for t in range(q_len):
            p = start + t
            sm[b * q_len + t] = int(mir[row, p // bs]) * bs + p % bs
    return 0


@pytest.fixture
def host_tables(monkeypatch):
    """DeviceBlockTables on CPU tensors with the stand-in entry point."""
    lib = SimpleNamespace(nvk_decode_metadata=_stand_in)
    monkeypatch.setattr(dm, "_lib", SimpleNamespace(load=lambda: lib, check=lambda name, rc: None))
    monkeypatch.setattr(torch.cuda, "Event", lambda: SimpleNamespace(synchronize=lambda: None,
                                                                     record=lambda stream=None: None))
    monkeypatch.setattr(torch.cuda, "current_stream", lambda device=None: SimpleNamespace(cuda_stream=0))
    empty = torch.empty
    monkeypatch.setattr(torch, "empty", lambda *a, pin_memory=False, **k: empty(*a, **k))
    return lambda bm, rows, cols: dm.DeviceBlockTables(bm, rows, cols, "cpu")


def _check(got, want, step):
    assert got.block_tables.dtype == torch.int32 and got.slot_mapping.dtype == torch.int64
    assert np.array_equal(got.block_tables.numpy(), want.block_tables.numpy()), step
    assert np.array_equal(got.context_lens.numpy(), want.context_lens.numpy()), step
    assert np.array_equal(got.slot_mapping.numpy(), want.slot_mapping.numpy()), step


def test_seeded_script_with_prefixes_rewinds_and_repeated_slots(host_tables):
    rnd = random.Random(5)
    bs, nb = 16, 4000
    host_bm, dev_bm = BlockManager(nb, bs, "cpu"), BlockManager(nb, bs, "cpu")
    perm = list(range(nb))
    rnd.shuffle(perm)
    host_bm.free_block_ids = perm
    dev_bm.free_block_ids = perm
    dt = host_tables(dev_bm, 64, 256)
    pos: dict[int, int] = {}
    for step in range(300):
        op = rnd.random()
        free_slots = [s for s in range(64) if s not in pos]
        if (op < 0.15 or not pos) and free_slots:  # prefill, sometimes over a prefix of another sequence
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
        elif op < 0.22 and len(pos) > 1:  # a sequence finishes; its slot may be reused
            slot = rnd.choice(list(pos))
            for bm in (host_bm, dev_bm):
                bm.free_slot(slot)
            del pos[slot]
        else:
            q_len = 3 if rnd.random() < 0.2 else 1
            slots = rnd.sample(list(pos), rnd.randint(1, len(pos)))
            starts = [pos[s] for s in slots]
            if rnd.random() < 0.15:  # a slot named twice
                j = rnd.randrange(len(slots))
                slots.append(slots[j])
                starts.append(starts[j] + q_len)
            if rnd.random() < 0.15:  # a row decoded behind its sequence's length
                j = rnd.randrange(len(slots))
                starts[j] = max(0, starts[j] - rnd.randint(1, 40))
            want = host_bm.prepare_decode_metadata(slots, starts, q_len)
            _check(dt.prepare_decode_metadata(slots, starts, q_len), want, step)
            for s, st in zip(slots, starts):
                pos[s] = max(pos[s], st + q_len)


def test_only_new_entries_cross_after_the_first_step(host_tables):
    bs = 16
    bm = BlockManager(64, bs, "cpu")
    bm.prepare_prefill_metadata([0, 1], [40, 5], [0, 0], [[], []])
    dt = host_tables(bm, 4, 32)
    sent = []
    inner = dm._lib.load().nvk_decode_metadata

    def spy(*args):
        batch, offsets = args[7], args[10]
        sent.append(int(_view(offsets, batch + 1, np.int32)[-1]))
        return inner(*args)

    dt._fn = spy
    dt.prepare_decode_metadata([0, 1], [40, 5], 1)   # whole tables: 3 + 1 entries
    dt.prepare_decode_metadata([0, 1], [41, 6], 1)   # nothing new
    dt.prepare_decode_metadata([0, 1], [48, 16], 1)  # one new block for each
    assert sent == [4, 0, 2]


def test_rejected_step_leaves_the_record_and_later_steps_match(host_tables):
    bs = 16
    host_bm, dev_bm = BlockManager(64, bs, "cpu"), BlockManager(64, bs, "cpu")
    for bm in (host_bm, dev_bm):
        bm.prepare_prefill_metadata([0, 1, 5], [40, 5, 3], [0, 0, 0], [[], [], []])
    dt = host_tables(dev_bm, 4, 32)
    _check(dt.prepare_decode_metadata([0, 1], [40, 5], 1), host_bm.prepare_decode_metadata([0, 1], [40, 5], 1), 0)
    record = dict(dt._synced)
    with pytest.raises(ValueError, match="outside the device mirror"):
        dt.prepare_decode_metadata([0, 5], [47, 3], 1)
    assert dt._synced == record
    host_bm.prepare_decode_metadata([0, 5], [47, 3], 1)  # the same allocator bookkeeping
    _check(dt.prepare_decode_metadata([1, 0], [6, 48], 1), host_bm.prepare_decode_metadata([1, 0], [6, 48], 1), 1)
