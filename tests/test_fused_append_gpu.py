"""Decode with this step's KV append fused into the attention kernel
(nvk_paged_decode_append), and the CUDA-graph decode runner that uses it.

* the pool after the call is bit-identical to the oracle's append, and the
  outputs match the fp32 oracle of append-then-decode, over GQA ratios, block
  sizes, persistent grids (pairs split across CTAs, so the CTA owning a pair's
  last tile is not the one that starts it), strided new rows (a slice of a
  fused QKV output) and zero-length contexts;
* a slot that is not the sequence's last position is skipped and flagged;
* DecodeGraphRunner on real CUDA graphs: the fused (default) and unfused
  runners leave bit-identical pools and outputs, equal to the oracle, over
  repeated replays with new inputs.
"""

from types import SimpleNamespace

import numpy as np
import pytest
import torch

from nano_vllm_ascend_b200 import BlockManager, DecodeGraphRunner, PagedAttention, PagedKVCache, ops
from oracle import paged_kv_oracle as orc
from tests.helpers import assert_close, bits, random_pool, seeded_tables

pytestmark = pytest.mark.gpu

D = 128
SCALE = D ** -0.5


def last_slots(tables: torch.Tensor, ctx: list[int], bs: int, nb: int) -> torch.Tensor:
    """Each sequence's last context position; a sequence without context gets a
    row of its own in a block no sequence uses (distinct slots, as a decode step has)."""
    used = {int(x) for b, n in enumerate(ctx) for x in tables[b, : (n + bs - 1) // bs]}
    spare = iter(sorted(set(range(nb)) - used))
    return torch.tensor([int(tables[b, (n - 1) // bs]) * bs + (n - 1) % bs if n > 0 else next(spare) * bs
                         for b, n in enumerate(ctx)], dtype=torch.int64)


def run_fused(dev, ctx, h=16, kvh=8, bs=128, num_ctas=0, seed=0, strided=False, bad=None):
    nb = sum((n + bs - 1) // bs for n in ctx) + 4
    kc, vc = random_pool(nb, bs, kvh, D, dev, seed)
    tables = seeded_tables(ctx, bs, nb, seed)
    slots = last_slots(tables, ctx, bs, nb)
    if bad is not None:
        slots[bad] = (slots[bad] + 1) % (nb * bs)  # not the sequence's last position
    g = torch.Generator(device=dev).manual_seed(seed + 7)
    b = len(ctx)
    q = torch.randn(b, h, D, generator=g, device=dev).to(torch.bfloat16)
    if strided:  # K and V as column slices of a fused [B, h + 2*kvh, D] projection output
        qkv = torch.randn(b, h + 2 * kvh, D, generator=g, device=dev).to(torch.bfloat16)
        k_new, v_new = qkv[:, h:h + kvh], qkv[:, h + kvh:]
        assert not k_new.is_contiguous()
    else:
        k_new = torch.randn(b, kvh, D, generator=g, device=dev).to(torch.bfloat16)
        v_new = torch.randn(b, kvh, D, generator=g, device=dev).to(torch.bfloat16)
    kc_host, vc_host = bits(kc).copy(), bits(vc).copy()
    ws = torch.zeros(ops.decode_workspace_bytes(b, h, kvh, D, num_ctas), dtype=torch.uint8, device=dev)
    out = torch.full_like(q, float("nan"))
    ctx_t = torch.tensor(ctx, dtype=torch.int32, device=dev)
    ops.paged_decode(out, q, kc, vc, tables.to(dev), ctx_t, SCALE, ws, num_ctas, new_key=k_new, new_value=v_new,
                     slot_mapping=slots.to(dev))
    torch.cuda.synchronize()
    keep = [i for i in range(b) if i != bad]
    orc.kv_append(kc_host, vc_host, bits(k_new)[keep], bits(v_new)[keep], slots.numpy()[keep])
    want = orc.paged_decode(bits(q), kc_host, vc_host, tables.numpy(), np.array(ctx), SCALE)
    return out, kc, vc, kc_host, vc_host, want, ws


@pytest.mark.parametrize("h,kvh,bs", [(16, 8, 128), (32, 8, 128), (8, 8, 16), (16, 2, 64), (64, 8, 256)])
def test_fused_append_matches_append_then_decode(cuda_device, h, kvh, bs):
    ctx = [1, bs - 1, bs, bs + 1, 3 * bs + 5, 700, 2304]
    out, kc, vc, kc_want, vc_want, want, ws = run_fused(cuda_device, ctx, h, kvh, bs, seed=h + kvh + bs)
    assert ops.decode_error_word(ws) == 0
    assert np.array_equal(bits(kc), kc_want) and np.array_equal(bits(vc), vc_want), "pool differs from the append"
    assert_close(out.float().cpu().numpy(), want, f"h={h} kvh={kvh} bs={bs}")


@pytest.mark.parametrize("num_ctas", [1, 5, 148, 600])
def test_fused_append_split_pairs(cuda_device, num_ctas):
    ctx = [5000, 3, 2304, 129, 4097, 640]
    out, kc, vc, kc_want, vc_want, want, ws = run_fused(cuda_device, ctx, num_ctas=num_ctas, seed=num_ctas)
    assert ops.decode_error_word(ws) == 0
    assert np.array_equal(bits(kc), kc_want) and np.array_equal(bits(vc), vc_want)
    assert_close(out.float().cpu().numpy(), want, f"num_ctas={num_ctas}")


def test_fused_append_strided_rows_and_zero_context(cuda_device):
    ctx = [0, 77, 1025, 0, 128]
    out, kc, vc, kc_want, vc_want, want, ws = run_fused(cuda_device, ctx, seed=9, strided=True)
    assert ops.decode_error_word(ws) == 0
    assert np.array_equal(bits(kc), kc_want) and np.array_equal(bits(vc), vc_want)
    got = out.float().cpu().numpy()
    assert not got[0].any() and not got[3].any()
    assert_close(got, want, "strided / zero ctx")


def test_fused_append_wrong_slot_is_skipped_and_flagged(cuda_device):
    ctx = [300, 129, 900]
    out, kc, vc, kc_want, vc_want, want, ws = run_fused(cuda_device, ctx, seed=5, bad=1)
    assert ops.decode_error_word(ws) & 4
    assert np.array_equal(bits(kc), kc_want) and np.array_equal(bits(vc), vc_want), "only the bad row is skipped"
    assert_close(out.float().cpu().numpy()[[0, 2]], want[[0, 2]], "other sequences")


# ------------------------------------------------------- graph runner ----
class TinyDecoder:
    """Qwen3Attention's hot-path order per layer (append, then attention) on static q/k/v."""

    def __init__(self, layers, batch, heads, kvh, device, seed):
        g = torch.Generator(device=device).manual_seed(seed)
        self.q = torch.randn(layers, batch, heads, D, generator=g, device=device).to(torch.bfloat16)
        self.k = torch.randn(layers, batch, kvh, D, generator=g, device=device).to(torch.bfloat16)
        self.v = torch.randn(layers, batch, kvh, D, generator=g, device=device).to(torch.bfloat16)
        self.attn = PagedAttention(heads, kvh, D)
        self.layers = layers

    def __call__(self, input_ids_flat, position_ids_flat, kv_cache, attn_metadata, is_prefill=False):
        n = input_ids_flat.shape[0]  # the first n sequences (views: fixed addresses for each graph)
        outs = []
        for layer in range(self.layers):
            kv_cache.write(layer, self.k[layer][:n], self.v[layer][:n], attn_metadata.slot_mapping)
            kc, vc = kv_cache.get_physical_cache(layer)
            outs.append(self.attn(self.q[layer][:n], kc, vc, attn_metadata.block_tables, attn_metadata.context_lens))
        return SimpleNamespace(logits=torch.stack(outs))


def build_runner(dev, fuse, ctx, layers=3, heads=16, kvh=8, nb=96):
    bm = BlockManager(nb, 128, dev)
    bm.free_block_ids = torch.randperm(nb, generator=torch.Generator().manual_seed(1)).tolist()
    seqs = list(range(len(ctx)))
    bm.prepare_prefill_metadata(seqs, ctx, [0] * len(ctx), [[] for _ in seqs])
    md = bm.prepare_decode_metadata(seqs, ctx, q_len=1)
    kv = PagedKVCache(layers, nb, 128, kvh, D, torch.bfloat16, dev)
    g = torch.Generator(device=dev).manual_seed(2)
    kv.key_cache.copy_(torch.randn(kv.key_cache.shape, generator=g, device=dev).to(torch.bfloat16))
    kv.value_cache.copy_(torch.randn(kv.value_cache.shape, generator=g, device=dev).to(torch.bfloat16))
    model = TinyDecoder(layers, len(ctx), heads, kvh, dev, seed=3)
    runner = DecodeGraphRunner(model, kv, batch_sizes=[len(ctx)], max_model_len=4096, block_size=128, device=dev,
                               fuse_appends=fuse)
    return bm, md, kv, model, runner


def test_graph_runner_fused_appends_on_real_graphs(cuda_device):
    ctx = [255, 1, 1500, 130]
    results = {}
    for fuse in (True, False):
        bm, md, kv, model, runner = build_runner(cuda_device, fuse, ctx)
        pool0 = (bits(kv.key_cache).copy(), bits(kv.value_cache).copy())
        ids = torch.zeros(len(ctx), dtype=torch.long, device=cuda_device)
        pos = torch.tensor(ctx, dtype=torch.long, device=cuda_device)
        outs = []
        for it in range(2):
            if it == 1:  # new inputs between replays
                model.q.normal_(generator=torch.Generator(device=cuda_device).manual_seed(9))
            logits = runner.forward(ids, pos, md)
            assert logits is not None
            torch.cuda.synchronize()
            outs.append(logits.clone())
        assert runner.stats_dict()["captures"] == 1 and runner.stats_dict()["replays"] == 2
        results[fuse] = (outs, bits(kv.key_cache).copy(), bits(kv.value_cache).copy())
        # oracle: this step's rows appended, then attention per layer
        kc, vc = pool0
        ctx_after = md.context_lens.numpy()
        slots = md.slot_mapping.cpu().numpy()
        tables = md.block_tables.cpu().numpy()
        for layer in range(model.layers):
            orc.kv_append(kc[layer], vc[layer], bits(model.k[layer]), bits(model.v[layer]), slots)
            want = orc.paged_decode(bits(model.q[layer]), kc[layer], vc[layer], tables, ctx_after, SCALE)
            assert_close(outs[1][layer].float().cpu().numpy(), want, f"fuse={fuse} layer {layer}")
        assert np.array_equal(results[fuse][1], kc) and np.array_equal(results[fuse][2], vc)
        runner.release()
    (o_f, k_f, v_f), (o_u, k_u, v_u) = results[True], results[False]
    assert np.array_equal(k_f, k_u) and np.array_equal(v_f, v_u)
    for a, b in zip(o_f, o_u):
        assert torch.equal(a, b), "fused and unfused graphs must produce identical outputs"


def test_graph_runner_capture_sizes(cuda_device):
    """One runner serving the reference's capture sizes 1, 2, 4, 8, 16, 32
    (acl_graph.py:110-250): a graph per exact batch size, captured on first
    use, every replay equal to the oracle for its sequences."""
    dev = cuda_device
    sizes = [1, 2, 4, 8, 16, 32]
    ctx = torch.randint(1, 900, (32,), generator=torch.Generator().manual_seed(21)).tolist()
    layers, nb = 2, sum((c + 128) // 128 for c in ctx) + 8
    bm = BlockManager(nb, 128, dev)
    bm.free_block_ids = torch.randperm(nb, generator=torch.Generator().manual_seed(22)).tolist()
    seqs = list(range(32))
    bm.prepare_prefill_metadata(seqs, ctx, [0] * 32, [[] for _ in seqs])
    kv = PagedKVCache(layers, nb, 128, 8, D, torch.bfloat16, dev)
    g = torch.Generator(device=dev).manual_seed(23)
    kv.key_cache.copy_(torch.randn(kv.key_cache.shape, generator=g, device=dev).to(torch.bfloat16))
    kv.value_cache.copy_(torch.randn(kv.value_cache.shape, generator=g, device=dev).to(torch.bfloat16))
    pool0 = (bits(kv.key_cache).copy(), bits(kv.value_cache).copy())
    model = TinyDecoder(layers, 32, 16, 8, dev, seed=24)
    runner = DecodeGraphRunner(model, kv, batch_sizes=sizes, max_model_len=4096, block_size=128, device=dev)
    try:
        for bs in sizes:
            md = bm.prepare_decode_metadata(seqs[:bs], ctx[:bs], q_len=1)
            ids = torch.zeros(bs, dtype=torch.long, device=dev)
            pos = torch.tensor(ctx[:bs], dtype=torch.long, device=dev)
            logits = runner.forward(ids, pos, md)
            assert logits is not None, f"batch size {bs} fell back"
            torch.cuda.synchronize()
            kc, vc = pool0[0].copy(), pool0[1].copy()
            slots = md.slot_mapping.cpu().numpy()
            for layer in range(layers):
                orc.kv_append(kc[layer], vc[layer], bits(model.k[layer][:bs]), bits(model.v[layer][:bs]), slots)
                want = orc.paged_decode(bits(model.q[layer][:bs]), kc[layer], vc[layer], md.block_tables.cpu().numpy(),
                                        md.context_lens.numpy(), SCALE)
                assert_close(logits[layer].float().cpu().numpy(), want, f"bs={bs} layer {layer}")
        stats = runner.stats_dict()
        assert stats["captures"] == len(sizes) and stats["replays"] == len(sizes) and stats["fallbacks"] == 0
    finally:
        runner.release()


def test_graph_runner_host_context_lens_overwritten_after_forward(cuda_device):
    """context_lens from the host (pinned, as a serving loop may keep it):
    forward() queues its copy without blocking the host, and the caller may
    overwrite its tensor as soon as forward() returns. A spin kernel queued
    first keeps the copy from running before the overwrite."""
    dev = cuda_device
    ctx = [700, 3, 1200, 129]
    bm, md, kv, model, runner = build_runner(dev, True, ctx, layers=2)
    pool0 = (bits(kv.key_cache).copy(), bits(kv.value_cache).copy())
    want_ctx = md.context_lens.clone()
    host_ctx = md.context_lens.to(torch.int32).pin_memory()
    step_md = type(md)(block_tables=md.block_tables, context_lens=host_ctx, slot_mapping=md.slot_mapping)
    ids = torch.zeros(len(ctx), dtype=torch.long, device=dev)
    pos = torch.tensor(ctx, dtype=torch.long, device=dev)
    try:
        assert runner.forward(ids, pos, step_md) is not None  # capture + first replay
        torch.cuda.synchronize()
        torch.cuda._sleep(20_000_000)
        logits = runner.forward(ids, pos, step_md)
        host_ctx.fill_(1)
        torch.cuda.synchronize()
        kc, vc = pool0[0].copy(), pool0[1].copy()
        slots = md.slot_mapping.cpu().numpy()
        for layer in range(2):
            orc.kv_append(kc[layer], vc[layer], bits(model.k[layer]), bits(model.v[layer]), slots)
            want = orc.paged_decode(bits(model.q[layer]), kc[layer], vc[layer], md.block_tables.cpu().numpy(),
                                    want_ctx.numpy(), SCALE)
            assert_close(logits[layer].float().cpu().numpy(), want, f"layer {layer}")
    finally:
        runner.release()
