"""Host logic of the fused decode append, on CPU (the kernels are replaced by
recorders): PagedKVCache.deferred_appends() holds each layer's rows back
instead of launching the append, PagedAttention takes them (take_deferred)
by the layer's key view -- owned by (cache, layer), so two caches never
mix -- rows nobody took are appended when the block exits and the exit
raises, a second write of a layer lands the first, and DecodeGraphRunner runs
the model inside the block only when fuse_appends is on."""

import pytest
import torch

import nano_vllm_ascend_b200.paged_kv_cache as pkc
from nano_vllm_ascend_b200 import PagedKVCacheMetadata
from nano_vllm_ascend_b200.cuda_graph import DecodeGraphRunner, graph_workspace
from tests.test_graph_runner import FakeAttention, FakeBackend


class NoErrors:
    word = None

    def raise_if_flagged(self):
        pass

    def launched(self, *names):
        pass


def make_cache(monkeypatch, layers=3):
    calls = []
    monkeypatch.setattr(pkc.ops, "kv_append",
                        lambda kc, vc, k, v, slots, error_word=None: calls.append((kc.data_ptr(), k, slots)))
    monkeypatch.setattr(pkc.torch.cuda, "device", lambda *_: __import__("contextlib").nullcontext())
    monkeypatch.setattr(pkc.device_errors, "state", lambda *_: NoErrors())
    cache = pkc.PagedKVCache(layers, 4, 16, 2, 8, torch.bfloat16, "cpu")
    return cache, calls


def rows(n=3, seed=0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(n, 2, 8, generator=g).to(torch.bfloat16), torch.randn(n, 2, 8, generator=g).to(torch.bfloat16),
            torch.arange(n, dtype=torch.int64))


def test_write_appends_at_once_outside_the_block(monkeypatch):
    cache, calls = make_cache(monkeypatch)
    k, v, s = rows()
    cache.write(1, k, v, s)
    assert len(calls) == 1 and calls[0][0] == cache.key_cache[1].data_ptr()
    assert pkc.take_deferred(cache.key_cache[1]) is None


def test_deferred_rows_are_taken_by_layer_view(monkeypatch):
    cache, calls = make_cache(monkeypatch)
    k, v, s = rows()
    with cache.deferred_appends():
        cache.write(0, k, v, s)
        cache.write(2, k, v, s)
        assert calls == []
        got = pkc.take_deferred(cache.key_cache[2])
        assert got is not None and torch.equal(got[0], k) and torch.equal(got[2], s)
        assert pkc.take_deferred(cache.key_cache[2]) is None  # taken once
        assert torch.equal(pkc.take_deferred(cache.key_cache[0])[0], k)
    assert calls == []
    assert pkc.take_deferred(cache.key_cache[0]) is None  # outside the block nothing is deferred


def test_rows_no_attention_took_are_appended_and_the_exit_raises(monkeypatch):
    cache, calls = make_cache(monkeypatch)
    k, v, s = rows()
    with pytest.raises(RuntimeError, match=r"layer\(s\) \[0\] was not consumed"):
        with cache.deferred_appends():
            cache.write(0, k, v, s)
    assert [c[0] for c in calls] == [cache.key_cache[0].data_ptr()]
    assert not pkc._DEFERRING


def test_two_caches_keep_their_own_rows(monkeypatch):
    a, _ = make_cache(monkeypatch)
    b, _ = make_cache(monkeypatch)
    ka, va, sa = rows(seed=3)
    kb, vb, sb = rows(seed=4)
    with a.deferred_appends(), b.deferred_appends():
        a.write(1, ka, va, sa)
        b.write(1, kb, vb, sb)
        assert torch.equal(pkc.take_deferred(b.key_cache[1])[0], kb)
        assert torch.equal(pkc.take_deferred(a.key_cache[1])[0], ka)
        # a view that is not one whole layer of a pool owns nothing
        assert pkc.take_deferred(a.key_cache[1, 1:]) is None


def test_second_write_of_a_layer_lands_the_first(monkeypatch):
    cache, calls = make_cache(monkeypatch)
    k1, v1, s1 = rows(seed=1)
    k2, v2, s2 = rows(seed=2)
    with cache.deferred_appends():
        cache.write(1, k1, v1, s1)
        cache.write(1, k2, v2, s2)
        assert len(calls) == 1 and torch.equal(calls[0][1], k1)
        got = pkc.take_deferred(cache.key_cache[1])
        assert torch.equal(got[0], k2)
    assert len(calls) == 1


def test_nested_blocks_flush_only_at_the_outermost(monkeypatch):
    cache, calls = make_cache(monkeypatch)
    k, v, s = rows()
    with cache.deferred_appends():
        with cache.deferred_appends():
            cache.write(0, k, v, s)
        assert calls == []
        assert pkc.take_deferred(cache.key_cache[0]) is not None
    assert calls == []


class DeferringCache:
    def __init__(self):
        self.entered = 0

    def deferred_appends(self):
        cache = self

        class Ctx:
            def __enter__(self):
                cache.entered += 1

            def __exit__(self, *exc):
                return False

        return Ctx()


class Model:
    def __call__(self, input_ids_flat, position_ids_flat, kv_cache, attn_metadata, is_prefill):
        graph_workspace(FakeAttention(), input_ids_flat.numel())

        class Out:
            logits = torch.zeros(2)

        return Out()


def metadata():
    return PagedKVCacheMetadata(block_tables=torch.zeros(2, 3, dtype=torch.int32),
                                context_lens=torch.tensor([3, 5], dtype=torch.int32),
                                slot_mapping=torch.tensor([2, 4], dtype=torch.int64))


def test_graph_runner_defers_appends_only_when_fusing():
    for fuse, expected in ((True, 2), (False, 0)):  # warm-up run + capture
        cache = DeferringCache()
        runner = DecodeGraphRunner(Model(), cache, batch_sizes=[2], device="cpu", fuse_appends=fuse,
                                   backend=FakeBackend())
        ids = torch.zeros(2, dtype=torch.long)
        assert runner.forward(ids, ids, metadata()) is not None
        assert cache.entered == expected
