"""DecodeGraphRunner host logic on CPU with a fake graph backend.

Restates the reference's graph-runner tests (tests/test_decode_graph.py:129-173
in Pla-Yer/nano_vllm_ascend): capture once then replay, stats keys, and a
failing capture disabling only its own batch size; plus the static block-table
contract of acl_graph.py:208-219, :253-267.
"""

import pytest
import torch

from nano_vllm_ascend_b200 import PagedKVCacheMetadata
from nano_vllm_ascend_b200.cuda_graph import (DecodeGraphRunner, PagedAttentionGraphTask, copy_block_tables,
                                              record_paged_attention_task)


class FakeGraph:
    def __init__(self):
        self.replays = 0


class FakeGraphContext:
    def __init__(self, graph):
        self.graph = graph

    def __enter__(self):
        return self.graph

    def __exit__(self, *exc):
        return False


class FakeRunner(DecodeGraphRunner):
    def _new_graph(self):
        return FakeGraph()

    def _graph_context(self, graph):
        return FakeGraphContext(graph)

    def _synchronize(self):
        pass

    def _replay(self, graph):
        graph.replays += 1


class FakeModel:
    def __init__(self):
        self.calls = 0
        self.seen_block_tables = []

    def __call__(self, input_ids_flat, position_ids_flat, kv_cache, attn_metadata, is_prefill):
        self.calls += 1
        self.seen_block_tables.append(attn_metadata.block_tables)
        record_paged_attention_task(PagedAttentionGraphTask(
            query=torch.zeros(1), key_cache=None, value_cache=None, num_kv_heads=1, num_heads=1, scale=1.0,
            block_tables=attn_metadata.block_tables, context_lens=attn_metadata.context_lens,
            output=torch.zeros(1), workspace=None))

        class Out:
            logits = torch.full((input_ids_flat.numel(), 4), 99.0)

        return Out()


def metadata(batch=1, width=2):
    return PagedKVCacheMetadata(block_tables=torch.arange(batch * width, dtype=torch.int32).view(batch, width),
                                context_lens=torch.full((batch,), 5, dtype=torch.int32),
                                slot_mapping=torch.arange(batch, dtype=torch.int64))


def test_captures_once_then_replays():
    model = FakeModel()
    runner = FakeRunner(model=model, kv_cache=object(), batch_sizes=[1], device="cpu")
    first = runner.forward(torch.tensor([1]), torch.tensor([2]), metadata())
    second = runner.forward(torch.tensor([3]), torch.tensor([4]), metadata())
    assert torch.equal(first, second) and float(first[0, 0]) == 99.0
    # one eager warm-up + one capture, then replays only
    assert model.calls == 2
    stats = runner.stats_dict()
    assert stats == {"captures": 1, "replays": 2, "updates": 2, "fallbacks": 0, "capture_failures": 0}
    entry = runner.entries[1]
    assert entry.graph.replays == 2
    assert entry.input_ids.tolist() == [3] and entry.position_ids.tolist() == [4]


def test_failing_capture_disables_only_that_batch_size(capsys):
    class FailingModel:
        def __call__(self, **kwargs):
            raise RuntimeError("capture failed")

    runner = FakeRunner(model=FailingModel(), kv_cache=object(), batch_sizes=[1, 2], device="cpu")
    assert runner.forward(torch.tensor([1]), torch.tensor([2]), metadata()) is None
    assert 1 in runner.disabled_batch_sizes
    assert runner.supports(2) and not runner.supports(1)
    assert runner.stats_dict()["capture_failures"] == 1
    assert runner.stats_dict()["fallbacks"] == 1
    assert "[decode_graph] disable batch_size=1" in capsys.readouterr().out


def test_unsupported_batch_size_falls_back():
    runner = FakeRunner(model=FakeModel(), kv_cache=object(), batch_sizes=[4], device="cpu")
    assert runner.forward(torch.tensor([1]), torch.tensor([2]), metadata()) is None
    assert runner.stats_dict()["fallbacks"] == 1 and runner.stats_dict()["captures"] == 0


def test_model_without_attention_tasks_is_a_capture_failure():
    class NoAttention:
        def __call__(self, input_ids_flat, **kwargs):
            class Out:
                logits = torch.zeros(1)

            return Out()

    runner = FakeRunner(model=NoAttention(), kv_cache=object(), batch_sizes=[1], device="cpu")
    assert runner.forward(torch.tensor([1]), torch.tensor([2]), metadata()) is None
    assert runner.stats_dict()["capture_failures"] == 1


def test_static_block_tables_are_padded_to_max_model_len():
    model = FakeModel()
    runner = FakeRunner(model=model, kv_cache=object(), batch_sizes=[2], max_model_len=1000, block_size=128,
                        device="cpu")
    runner.forward(torch.tensor([1, 2]), torch.tensor([3, 4]), metadata(batch=2, width=3))
    entry = runner.entries[2]
    assert entry.block_tables.shape == (2, 8)  # ceil(1000 / 128)
    assert entry.block_tables[:, :3].tolist() == [[0, 1, 2], [3, 4, 5]]
    assert int(entry.block_tables[:, 3:].abs().sum()) == 0
    # a later, narrower table zero-fills the tail
    runner.forward(torch.tensor([1, 2]), torch.tensor([3, 4]), metadata(batch=2, width=1))
    assert entry.block_tables.tolist() == [[0] + [0] * 7, [1] + [0] * 7]


def test_copy_block_tables_rejects_wider_source():
    target = torch.zeros(2, 2, dtype=torch.int32)
    with pytest.raises(RuntimeError, match="smaller than runtime width"):
        copy_block_tables(target, torch.zeros(2, 3, dtype=torch.int32))


def test_record_outside_capture_raises():
    with pytest.raises(RuntimeError, match="outside graph capture"):
        record_paged_attention_task(None)
