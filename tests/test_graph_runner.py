"""DecodeGraphRunner host logic on CPU with a stand-in graph backend.

Covers the reference runner's observable contract (its tests,
tests/test_decode_graph.py:129-173 in Pla-Yer/nano_vllm_ascend, and
acl_graph.py:58-73, 184-219, 253-267): capture once then replay, the stats
keys, a failing capture disabling only its own batch size with the
"[decode_graph] disable" line, unsupported sizes falling back, static block
tables padded to ceil(max_model_len / block_size) with a zero tail, and
copy_block_tables' width check. Plus this runner's own design: attention
layers draw the slot's workspace through graph_workspace() (a model with no
attention call fails its capture), and metadata already living in the slot's
static buffers is not copied again.
"""

import pytest
import torch

from nano_vllm_ascend_b200 import PagedKVCacheMetadata
from nano_vllm_ascend_b200.cuda_graph import (CudaGraphBackend, DecodeGraphRunner, copy_block_tables,
                                              graph_workspace, recording_slot)


class FakeGraph:
    def __init__(self):
        self.replays = 0


class FakeBackend(CudaGraphBackend):
    def __init__(self):
        self.in_capture = False

    def new_graph(self):
        return FakeGraph()

    def capture(self, graph):
        backend = self

        class Ctx:
            def __enter__(self):
                backend.in_capture = True
                return graph

            def __exit__(self, *exc):
                backend.in_capture = False
                return False

        return Ctx()

    def replay(self, graph):
        graph.replays += 1

    def synchronize(self):
        pass

    def capturing(self):
        return self.in_capture


class FakeAttention:
    def workspace_bytes(self, batch):
        return 64 * batch


class FakeModel:
    def __init__(self, attention_calls=1):
        self.calls = 0
        self.attn = FakeAttention()
        self.attention_calls = attention_calls
        self.workspaces = []

    def __call__(self, input_ids_flat, position_ids_flat, kv_cache, attn_metadata, is_prefill):
        self.calls += 1
        for _ in range(self.attention_calls):
            self.workspaces.append(graph_workspace(self.attn, input_ids_flat.numel()))

        class Out:
            logits = torch.full((input_ids_flat.numel(), 4), 99.0)

        return Out()


def runner_for(model, **kw):
    return DecodeGraphRunner(model=model, kv_cache=object(), device="cpu", backend=FakeBackend(), **kw)


def metadata(batch=1, width=2):
    return PagedKVCacheMetadata(block_tables=torch.arange(batch * width, dtype=torch.int32).view(batch, width),
                                context_lens=torch.full((batch,), 5, dtype=torch.int32),
                                slot_mapping=torch.arange(batch, dtype=torch.int64))


def test_captures_once_then_replays():
    model = FakeModel()
    runner = runner_for(model, batch_sizes=[1])
    first = runner.forward(torch.tensor([1]), torch.tensor([2]), metadata())
    second = runner.forward(torch.tensor([3]), torch.tensor([4]), metadata())
    assert torch.equal(first, second) and float(first[0, 0]) == 99.0
    # one eager warm-up + one capture, then replays only
    assert model.calls == 2
    assert runner.stats_dict() == {"captures": 1, "replays": 2, "updates": 2, "fallbacks": 0, "capture_failures": 0}
    slot = runner.slot(1)
    assert slot.graph.replays == 2
    assert slot.input_ids.tolist() == [3] and slot.position_ids.tolist() == [4]


def test_every_attention_call_of_a_slot_shares_its_workspace():
    model = FakeModel(attention_calls=3)
    runner = runner_for(model, batch_sizes=[2])
    runner.forward(torch.tensor([1, 2]), torch.tensor([3, 4]), metadata(batch=2))
    ws = runner.slot(2).workspace
    assert ws is not None and ws.numel() == 128
    assert len(model.workspaces) == 6 and all(w is ws for w in model.workspaces)
    assert graph_workspace(FakeAttention(), 2) is None  # outside warm-up and capture
    assert recording_slot() is None


def test_failing_capture_disables_only_that_batch_size(capsys):
    class FailingModel:
        def __call__(self, **kwargs):
            raise RuntimeError("capture failed")

    runner = runner_for(FailingModel(), batch_sizes=[1, 2])
    assert runner.forward(torch.tensor([1]), torch.tensor([2]), metadata()) is None
    assert 1 in runner.disabled_batch_sizes
    assert runner.supports(2) and not runner.supports(1)
    assert runner.stats_dict()["capture_failures"] == 1
    assert runner.stats_dict()["fallbacks"] == 1
    assert "[decode_graph] disable batch_size=1" in capsys.readouterr().out
    assert recording_slot() is None  # the failed recording was closed


def test_unsupported_batch_size_falls_back():
    runner = runner_for(FakeModel(), batch_sizes=[4])
    assert runner.forward(torch.tensor([1]), torch.tensor([2]), metadata()) is None
    assert runner.stats_dict()["fallbacks"] == 1 and runner.stats_dict()["captures"] == 0


def test_model_without_attention_calls_is_a_capture_failure():
    runner = runner_for(FakeModel(attention_calls=0), batch_sizes=[1])
    assert runner.forward(torch.tensor([1]), torch.tensor([2]), metadata()) is None
    assert runner.stats_dict()["capture_failures"] == 1


def test_workspace_growth_during_capture_is_refused(capsys):
    class GrowingAttention(FakeAttention):
        def __init__(self):
            self.n = 0

        def workspace_bytes(self, batch):
            self.n += 1
            return 64 * self.n  # larger in the capture than in the warm-up

    model = FakeModel()
    model.attn = GrowingAttention()
    runner = runner_for(model, batch_sizes=[1])
    assert runner.forward(torch.tensor([1]), torch.tensor([2]), metadata()) is None
    assert "sized by the warm-up" in capsys.readouterr().out


def test_static_block_tables_are_padded_to_max_model_len():
    runner = runner_for(FakeModel(), batch_sizes=[2], max_model_len=1000, block_size=128)
    runner.forward(torch.tensor([1, 2]), torch.tensor([3, 4]), metadata(batch=2, width=3))
    slot = runner.slot(2)
    assert slot.block_tables.shape == (2, 8)  # ceil(1000 / 128)
    assert slot.block_tables[:, :3].tolist() == [[0, 1, 2], [3, 4, 5]]
    assert int(slot.block_tables[:, 3:].abs().sum()) == 0
    # a later, narrower table zero-fills the tail
    runner.forward(torch.tensor([1, 2]), torch.tensor([3, 4]), metadata(batch=2, width=1))
    assert slot.block_tables.tolist() == [[0] + [0] * 7, [1] + [0] * 7]
    with pytest.raises(RuntimeError, match="smaller than runtime width"):
        runner.forward(torch.tensor([1, 2]), torch.tensor([3, 4]), metadata(batch=2, width=9))


def test_metadata_in_the_static_buffers_is_not_copied_again():
    runner = runner_for(FakeModel(), batch_sizes=[2], max_model_len=512, block_size=128)
    runner.forward(torch.tensor([1, 2]), torch.tensor([3, 4]), metadata(batch=2, width=2))
    slot = runner.slot(2)
    md = slot.metadata(metadata(batch=2))
    slot.block_tables.copy_(torch.tensor([[7, 8, 9, 1], [6, 5, 4, 3]], dtype=torch.int32))
    slot.context_lens.copy_(torch.tensor([400, 300], dtype=torch.int32))
    runner.forward(torch.tensor([1, 2]), torch.tensor([3, 4]), md)  # what a device-side builder wrote stays
    assert slot.block_tables.tolist() == [[7, 8, 9, 1], [6, 5, 4, 3]]
    assert slot.context_lens.tolist() == [400, 300]


def test_host_context_lens_reach_the_static_buffer():
    runner = runner_for(FakeModel(), batch_sizes=[2])
    md = metadata(batch=2)
    md.context_lens = torch.tensor([11, 12], dtype=torch.int32)
    runner.forward(torch.tensor([1, 2]), torch.tensor([3, 4]), md)
    assert runner.slot(2).context_lens.tolist() == [11, 12]


def test_copy_block_tables_rejects_wider_source():
    target = torch.ones(2, 4, dtype=torch.int32)
    with pytest.raises(RuntimeError, match="smaller than runtime width"):
        copy_block_tables(target, torch.zeros(2, 5, dtype=torch.int32))
    copy_block_tables(target, torch.full((2, 1), 3, dtype=torch.int32))
    assert target.tolist() == [[3, 0, 0, 0], [3, 0, 0, 0]]
