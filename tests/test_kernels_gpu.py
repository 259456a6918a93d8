"""Parity of the CUDA kernels (through the C ABI) with the CPU oracle.

* append: bit-exact vs the reference's own PagedKVCache.write (golden digests)
  and vs the oracle on strided / ragged inputs;
* decode: within max-abs 2e-2 / max-rel 1e-2 of the fp32 oracle over GQA
  ratios 1/2/4/8, block sizes 16..256, ragged and edge context lengths
  (0, 1, block-1, block, block+1, long), persistent grids from 1 CTA to more
  CTAs than tiles (pairs split across CTAs and merged), repeated calls on one
  workspace, and CUDA-graph replay with new inputs.
"""

import hashlib
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from nano_vllm_ascend_b200 import ops
from oracle import paged_kv_oracle as orc
from tests.golden.make_golden import append_inputs
from tests.helpers import assert_close, bits, random_pool, seeded_tables

pytestmark = pytest.mark.gpu

APPEND = json.loads((Path(__file__).parent / "golden" / "append_golden.json").read_text())


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


# ----------------------------------------------------------------- append ---
@pytest.mark.parametrize("case", sorted(APPEND))
def test_append_bit_exact_vs_reference_golden(cuda_device, case):
    g = APPEND[case]
    nb, bs, kvh, d = g["shape"]
    k, v = append_inputs(len(g["slots"]), kvh, d, g["seed"])
    kc = torch.zeros(nb, bs, kvh, d, dtype=torch.bfloat16, device=cuda_device)
    vc = torch.zeros_like(kc)
    slots = torch.tensor(g["slots"], dtype=torch.int64, device=cuda_device)
    ops.kv_append(kc, vc, k.to(cuda_device), v.to(cuda_device), slots)
    torch.cuda.synchronize()
    assert sha(bits(kc)) == g["sha_pool_key"]
    assert sha(bits(vc)) == g["sha_pool_value"]


@pytest.mark.parametrize("tokens", [1, 7, 32, 8192])
def test_append_strided_rows_vs_oracle(cuda_device, tokens):
    nb, bs, kvh, d = 96, 128, 8, 128
    gen = torch.Generator(device=cuda_device).manual_seed(tokens)
    # K and V as slices of a fused [T, (16 + 8 + 8) * 128] projection output
    qkv = torch.randn(tokens, 32, d, generator=gen, device=cuda_device).to(torch.bfloat16)
    k, v = qkv[:, 16:24], qkv[:, 24:32]
    assert tokens == 1 or not k.is_contiguous()
    perm = torch.randperm(nb * bs, device=cuda_device)[:tokens]
    kc = torch.zeros(nb, bs, kvh, d, dtype=torch.bfloat16, device=cuda_device)
    vc = torch.zeros_like(kc)
    ops.kv_append(kc, vc, k, v, perm)
    torch.cuda.synchronize()
    kc_ref = np.zeros((nb, bs, kvh, d), np.uint16)
    vc_ref = np.zeros_like(kc_ref)
    orc.kv_append(kc_ref, vc_ref, bits(k), bits(v), perm.cpu().numpy())
    assert np.array_equal(bits(kc), kc_ref)
    assert np.array_equal(bits(vc), vc_ref)


def test_append_out_of_range_slot_is_skipped_and_flagged(cuda_device):
    kc = torch.zeros(2, 16, 8, 128, dtype=torch.bfloat16, device=cuda_device)
    vc = torch.zeros_like(kc)
    k = torch.ones(3, 8, 128, dtype=torch.bfloat16, device=cuda_device)
    slots = torch.tensor([5, 32, -1], dtype=torch.int64, device=cuda_device)
    err = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    ops.kv_append(kc, vc, k, k, slots, error_word=err)
    torch.cuda.synchronize()
    assert int(err.item()) & 4
    flat = kc.view(-1, 8, 128)
    assert bool((flat[5] == 1).all()) and int((flat != 0).sum()) == 8 * 128


@pytest.mark.parametrize("tokens,kvh", [(1024, 8), (5000, 8), (3000, 4), (2048, 1)])
def test_append_bulk_path_vs_oracle_with_bad_slots(cuda_device, tokens, kvh):
    # >= 1024 rows take the TMA bulk-copy kernel; a few slots are out of range
    nb, bs, d = (tokens + 127) // 128 + 8, 128, 128
    gen = torch.Generator(device=cuda_device).manual_seed(tokens + kvh)
    k = torch.randn(tokens, kvh, d, generator=gen, device=cuda_device).to(torch.bfloat16)
    v = torch.randn(tokens, kvh, d, generator=gen, device=cuda_device).to(torch.bfloat16)
    slots = torch.randperm(nb * bs, device=cuda_device)[:tokens]
    bad = torch.tensor([3, tokens // 2, tokens - 1], device=cuda_device)
    slots[bad] = torch.tensor([-5, nb * bs, nb * bs + 99], device=cuda_device)
    kc = torch.zeros(nb, bs, kvh, d, dtype=torch.bfloat16, device=cuda_device)
    vc = torch.zeros_like(kc)
    err = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    ops.kv_append(kc, vc, k, v, slots, error_word=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 4
    keep = torch.ones(tokens, dtype=torch.bool, device=cuda_device)
    keep[bad] = False
    kc_ref = np.zeros((nb, bs, kvh, d), dtype=np.uint16)
    vc_ref = np.zeros_like(kc_ref)
    orc.kv_append(kc_ref, vc_ref, bits(k[keep]), bits(v[keep]), slots[keep].cpu().numpy())
    assert np.array_equal(bits(kc), kc_ref)
    assert np.array_equal(bits(vc), vc_ref)


# ----------------------------------------------------------------- decode ---
def run_decode(cuda_device, ctx, h=16, kvh=8, bs=128, nb=None, seed=0, num_ctas=0, width=None, q_scale=1.0):
    need = sum((n + bs - 1) // bs for n in ctx)
    nb = nb or max(need + 3, 4)
    kc, vc = random_pool(nb, bs, kvh, 128, cuda_device, seed)
    tables = seeded_tables(ctx, bs, nb, seed, width).to(cuda_device)
    g = torch.Generator(device=cuda_device).manual_seed(seed + 1)
    q = (torch.randn(len(ctx), h, 128, generator=g, device=cuda_device) * q_scale).to(torch.bfloat16)
    ctx_t = torch.tensor(ctx, dtype=torch.int32, device=cuda_device)
    scale = 128 ** -0.5
    ws = torch.zeros(ops.decode_workspace_bytes(len(ctx), h, kvh, 128, num_ctas), dtype=torch.uint8,
                     device=cuda_device)
    out = torch.full_like(q, float("nan"))
    ops.paged_decode(out, q, kc, vc, tables, ctx_t, scale, ws, num_ctas)
    torch.cuda.synchronize()
    assert ops.decode_error_word(ws) == 0
    want = orc.paged_decode(bits(q), bits(kc), bits(vc), tables.cpu().numpy(), np.array(ctx), scale)
    got = out.float().cpu().numpy()
    return got, want, ws


def test_decode_config1(cuda_device):
    got, want, _ = run_decode(cuda_device, [38, 129, 256, 514], nb=64)
    assert_close(got, want, "config1")


@pytest.mark.parametrize("h,kvh", [(8, 8), (16, 8), (32, 8), (64, 8), (16, 2)])
def test_decode_gqa_ratios(cuda_device, h, kvh):
    got, want, _ = run_decode(cuda_device, [1, 77, 128, 300, 1025], h=h, kvh=kvh, seed=h + kvh)
    assert_close(got, want, f"h={h} kvh={kvh}")


@pytest.mark.parametrize("bs", [16, 32, 64, 128, 256])
def test_decode_block_sizes(cuda_device, bs):
    ctx = [1, bs - 1, bs, bs + 1, 3 * bs + 5, 700]
    got, want, _ = run_decode(cuda_device, ctx, bs=bs, seed=bs)
    assert_close(got, want, f"bs={bs}")


@pytest.mark.parametrize("num_ctas", [1, 3, 7, 148, 1000])
def test_decode_persistent_grid_sizes(cuda_device, num_ctas):
    # 1 CTA walks everything; 1000 CTAs is more CTAs than tiles (empty ranges,
    # pairs split over many CTAs and merged by the last to finish)
    ctx = [5000, 1, 2304, 129, 4097]
    got, want, _ = run_decode(cuda_device, ctx, seed=num_ctas, num_ctas=num_ctas)
    assert_close(got, want, f"num_ctas={num_ctas}")


def test_decode_single_long_sequence_split_over_all_sms(cuda_device):
    got, want, _ = run_decode(cuda_device, [30000], h=32, kvh=8, seed=17)
    assert_close(got, want, "one long sequence")


def test_decode_large_batch_above_one_launch_chunk(cuda_device):
    # more sequences than one launch's schedule holds (1024): chunked launches
    rng = np.random.default_rng(5)
    ctx = rng.integers(0, 65, size=1100).tolist()
    got, want, _ = run_decode(cuda_device, ctx, bs=16, seed=23)
    assert_close(got, want, "1100 sequences")


def test_decode_zero_context_gives_zeros(cuda_device):
    got, want, _ = run_decode(cuda_device, [0, 5, 0])
    assert np.all(got[0] == 0) and np.all(got[2] == 0)
    assert_close(got, want, "zero ctx")


def test_decode_peaked_softmax_rescaling(cuda_device):
    # large q makes logits span far more than 2^8 so the lazy rescale fires
    got, want, _ = run_decode(cuda_device, [2000, 900, 333], q_scale=12.0, seed=3)
    assert_close(got, want, "peaked")


def test_decode_workspace_reuse_across_calls(cuda_device):
    ctx = [3000, 10, 1500, 700]
    got1, want1, ws = run_decode(cuda_device, ctx, seed=21, num_ctas=6)
    tickets = ws[256:256 + 4 * 8 * 32 * 4].view(torch.int32)  # one 128-byte line per (sequence, kv head)
    assert int(tickets.abs().sum()) == 0, "arrival tickets must return to zero"
    assert_close(got1, want1, "first")
    got2, want2, _ = run_decode(cuda_device, ctx, seed=22, num_ctas=6)
    assert_close(got2, want2, "second")


def test_eager_shared_workspace_survives_a_batch_size_change(cuda_device):
    """PagedAttention's per-device workspace serving a batch of 2, then 3, then
    2 again: each call's tickets lie where the call before it left partial
    results, which the workspace helper clears when the shape changes."""
    from nano_vllm_ascend_b200 import PagedAttention, check_errors

    attn = PagedAttention(16, 8, 128)
    for seed, ctx in ((31, [300, 200]), (32, [700, 130, 2000]), (33, [50, 4000])):
        nb = sum((n + 127) // 128 for n in ctx) + 3
        kc, vc = random_pool(nb, 128, 8, 128, cuda_device, seed)
        tables = seeded_tables(ctx, 128, nb, seed).to(cuda_device)
        g = torch.Generator(device=cuda_device).manual_seed(seed + 1)
        q = torch.randn(len(ctx), 16, 128, generator=g, device=cuda_device).to(torch.bfloat16)
        out = attn(q, kc, vc, tables, torch.tensor(ctx, dtype=torch.int32, device=cuda_device))
        check_errors(cuda_device)
        want = orc.paged_decode(bits(q), bits(kc), bits(vc), tables.cpu().numpy(), np.array(ctx), 128 ** -0.5)
        assert_close(out.float().cpu().numpy(), want, f"eager decode of batch {len(ctx)}")


def test_decode_wide_padded_table(cuda_device):
    # graph-style static table: much wider than any context
    got, want, _ = run_decode(cuda_device, [130, 9], width=64, seed=4)
    assert_close(got, want, "wide table")


def test_decode_under_cuda_graph_replay(cuda_device):
    bs, kvh, h, nb = 128, 8, 16, 80
    kc, vc = random_pool(nb, bs, kvh, 128, cuda_device, 31)
    width = 16
    ws = torch.zeros(ops.decode_workspace_bytes(4, h, kvh, 128), dtype=torch.uint8, device=cuda_device)
    q = torch.zeros(4, h, 128, dtype=torch.bfloat16, device=cuda_device)
    tables = torch.zeros(4, width, dtype=torch.int32, device=cuda_device)
    ctx = torch.ones(4, dtype=torch.int32, device=cuda_device)
    out = torch.empty_like(q)
    ops.paged_decode(out, q, kc, vc, tables, ctx, 128 ** -0.5, ws)  # warm-up
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        ops.paged_decode(out, q, kc, vc, tables, ctx, 128 ** -0.5, ws)
    for seed, lens in ((1, [100, 2000, 1, 640]), (2, [1999, 5, 1024, 129])):
        g = torch.Generator(device=cuda_device).manual_seed(seed)
        q.copy_(torch.randn(4, h, 128, generator=g, device=cuda_device).to(torch.bfloat16))
        tables.copy_(seeded_tables(lens, bs, nb, seed, width))
        ctx.copy_(torch.tensor(lens, dtype=torch.int32))
        graph.replay()
        torch.cuda.synchronize()
        want = orc.paged_decode(bits(q), bits(kc), bits(vc), tables.cpu().numpy(), np.array(lens), 128 ** -0.5)
        assert_close(out.float().cpu().numpy(), want, f"graph replay {seed}")
