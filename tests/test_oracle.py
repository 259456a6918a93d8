"""Pins the CPU oracle (CPU only).

* append and slot mapping: bit-exact against the reference's own
  PagedKVCache.write / BlockManager outputs recorded in tests/golden/;
* attention: the numpy restatement agrees with the independent eager
  torch-CPU expression of the reference path (oracle/cpu_baseline.py) --
  the reference's attention op is closed, so no golden vector exists for it.
"""

import hashlib
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import cpu_baseline
from oracle import paged_kv_oracle as orc
from tests.golden.make_golden import append_inputs

GOLDEN_DIR = Path(__file__).parent / "golden"
APPEND = json.loads((GOLDEN_DIR / "append_golden.json").read_text())
BM = json.loads((GOLDEN_DIR / "block_manager_golden.json").read_text())


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.mark.parametrize("case", sorted(APPEND))
def test_oracle_append_matches_reference_golden(case):
    g = APPEND[case]
    nb, bs, kvh, d = g["shape"]
    k, v = append_inputs(len(g["slots"]), kvh, d, g["seed"])
    assert sha(bits(k)) == g["sha_key_in"] and sha(bits(v)) == g["sha_value_in"], "seeded inputs changed"
    kc = np.zeros((nb, bs, kvh, d), dtype=np.uint16)
    vc = np.zeros_like(kc)
    slots = np.asarray(g["slots"], dtype=np.int64)
    orc.kv_append(kc, vc, bits(k), bits(v), slots)
    assert sha(kc.reshape(-1, kvh, d)[slots]) == g["sha_rows_key"]
    assert sha(vc.reshape(-1, kvh, d)[slots]) == g["sha_rows_value"]
    assert sha(kc) == g["sha_pool_key"] and sha(vc) == g["sha_pool_value"]


def test_oracle_slot_mapping_matches_reference_golden():
    c1 = BM["config1"]
    tables = [[b for b in row] for row in c1["decode"]["block_tables"]]
    lens = [len([1 for _ in range((n + 127) // 128)]) for n in c1["decode"]["context_lens"]]
    tables = [row[:n] for row, n in zip(tables, lens)]
    got = orc.slot_mapping(tables, c1["ctx"], [1] * 4, 128)
    assert got.tolist() == c1["decode"]["slot_mapping"]
    got = orc.slot_mapping(tables, [0] * 4, c1["ctx"], 128)
    assert got.tolist() == c1["prefill"]["slot_mapping"]
    unit = BM["unit"]["prefill"]
    tables = [row[: (n + 3) // 4] for row, n in zip(unit["block_tables"], unit["context_lens"])]
    assert orc.slot_mapping(tables, [0, 0, 0], [3, 5, 2], 4).tolist() == unit["slot_mapping"]
    with pytest.raises(RuntimeError):
        orc.slot_mapping([[0]], [4], [1], 4)


def test_bf16_round_trip_is_exact_and_rne():
    x = torch.randn(4096, generator=torch.Generator().manual_seed(3)) * 10
    ref = bits(x.to(torch.bfloat16))
    assert np.array_equal(orc.f32_to_bf16_bits(x.numpy()), ref)
    assert np.array_equal(orc.f32_to_bf16_bits(orc.bf16_bits_to_f32(ref)), ref)


def _c1_inputs(seed=0, kvh=8, h=16, ctx=(38, 129, 256, 514), nb=64, bs=128):
    g = torch.Generator().manual_seed(seed)
    kc = torch.randn(nb, bs, kvh, 128, generator=g).to(torch.bfloat16)
    vc = torch.randn(nb, bs, kvh, 128, generator=g).to(torch.bfloat16)
    q = torch.randn(len(ctx), h, 128, generator=g).to(torch.bfloat16)
    perm = torch.randperm(nb, generator=g)
    width = max((n + bs - 1) // bs for n in ctx)
    tables = torch.zeros(len(ctx), width, dtype=torch.int32)
    used = 0
    for i, n in enumerate(ctx):
        m = (n + bs - 1) // bs
        tables[i, :m] = perm[used : used + m].to(torch.int32)
        used += m
    return q, kc, vc, tables, torch.tensor(ctx, dtype=torch.int32)


@pytest.mark.parametrize("h,kvh", [(16, 8), (32, 8), (8, 8)])
def test_oracle_decode_agrees_with_torch_cpu_path(h, kvh):
    q, kc, vc, tables, ctx = _c1_inputs(h=h, kvh=kvh)
    scale = 128 ** -0.5
    want = cpu_baseline.decode(q, kc, vc, tables, ctx, scale).float().numpy()
    got = orc.paged_decode(bits(q), bits(kc), bits(vc), tables.numpy(), ctx.numpy(), scale)
    # cpu_baseline rounds its output to bf16
    np.testing.assert_allclose(got, want, atol=2e-2, rtol=1e-2)
    assert np.abs(got - want).max() < 1e-2


def test_oracle_prefill_agrees_with_torch_cpu_path():
    g = torch.Generator().manual_seed(5)
    nb, bs, kvh, h = 16, 128, 8, 16
    kc = torch.randn(nb, bs, kvh, 128, generator=g).to(torch.bfloat16)
    vc = torch.randn(nb, bs, kvh, 128, generator=g).to(torch.bfloat16)
    kv_lens = [300, 129, 64]
    q_lens = [44, 129, 1]  # prefix-cached, fresh, single-token suffix
    cu = [0]
    for n in q_lens:
        cu.append(cu[-1] + n)
    q = torch.randn(cu[-1], h, 128, generator=g).to(torch.bfloat16)
    perm = torch.randperm(nb, generator=g).to(torch.int32)
    tables = torch.zeros(3, 3, dtype=torch.int32)
    tables[0, :3] = perm[0:3]
    tables[1, :2] = perm[3:5]
    tables[2, :1] = perm[5:6]
    scale = 128 ** -0.5
    want = cpu_baseline.prefill(q, kc, vc, tables, cu, kv_lens, scale).float().numpy()
    got = orc.paged_prefill(bits(q), bits(kc), bits(vc), tables.numpy(), np.array(cu), np.array(kv_lens), scale)
    np.testing.assert_allclose(got, want, atol=2e-2, rtol=1e-2)


def test_oracle_dense_prefill_equals_paged_prefill_on_same_rows():
    g = torch.Generator().manual_seed(9)
    lens = [130, 7]
    cu = np.array([0, 130, 137])
    k = torch.randn(137, 2, 128, generator=g)
    v = torch.randn(137, 2, 128, generator=g)
    q = torch.randn(137, 4, 128, generator=g)
    dense = orc.dense_prefill(q.numpy(), k.numpy(), v.numpy(), cu, cu, 0.1)
    # lay the same rows into a paged pool (block size 128)
    kc = np.zeros((4, 128, 2, 128), np.float32)
    vc = np.zeros_like(kc)
    tables = np.array([[2, 0], [3, 0]])
    orc.kv_append(kc, vc, k.numpy()[:130], v.numpy()[:130], np.r_[np.arange(256, 384), 0, 1])
    orc.kv_append(kc, vc, k.numpy()[130:], v.numpy()[130:], np.arange(384, 391))
    paged = orc.paged_prefill(q.numpy(), kc, vc, tables, cu, np.array(lens), 0.1)
    np.testing.assert_allclose(dense, paged, rtol=1e-5, atol=1e-6)


def test_oracle_empty_and_fully_masked_rows_are_zero():
    q = np.ones((2, 2, 128), np.float32)
    kc = np.ones((1, 16, 1, 128), np.float32)
    out = orc.paged_decode(q, kc, kc, np.array([[0], [0]]), np.array([0, 3]), 0.1)
    assert np.all(out[0] == 0) and np.allclose(out[1], 1.0)


def test_norm_rope_oracle_matches_torch_cpu_restatement():
    """The numpy restatement of qwen3.py:83-96 against an independent torch-CPU
    expression of the same ops (float32 norm, bf16 output, bf16 cos/sin)."""
    import torch

    g = torch.Generator().manual_seed(0)
    t, h, kvh, d = 9, 4, 2, 128
    q = (torch.randn(t, h, d, generator=g) * 2).to(torch.bfloat16)
    k = (torch.randn(t, kvh, d, generator=g) * 2).to(torch.bfloat16)
    v = torch.randn(t, kvh, d, generator=g).to(torch.bfloat16)
    wq = (1 + 0.1 * torch.randn(d, generator=g)).to(torch.bfloat16)
    wk = (1 + 0.1 * torch.randn(d, generator=g)).to(torch.bfloat16)
    inv = 1.0 / (1e6 ** (torch.arange(0, d, 2, dtype=torch.float32) / d))
    emb = torch.cat([torch.outer(torch.arange(64, dtype=torch.float32), inv)] * 2, dim=-1)
    cos, sin = emb.cos(), emb.sin()
    pos = torch.randint(0, 64, (t,), generator=g)
    slots = torch.randperm(4 * 16, generator=g)[:t]

    def norm(x, w):
        xf = x.float()
        y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()
        return y.to(torch.bfloat16).float()

    def rope(y):
        c = cos[pos].to(torch.bfloat16).float()[:, None]
        s = sin[pos].to(torch.bfloat16).float()[:, None]
        rot = torch.cat([-y[..., d // 2:], y[..., : d // 2]], dim=-1)
        return (y * c + rot * s).to(torch.bfloat16)

    q_t, k_t = rope(norm(q, wq)), rope(norm(k, wk))
    bits = lambda x: x.contiguous().view(torch.int16).numpy().view(np.uint16)
    kc = np.zeros((4, 16, kvh, d), dtype=np.uint16)
    vc = np.zeros_like(kc)
    q_o = orc.qk_norm_rope_append(bits(q), bits(k), bits(v), bits(wq), bits(wk), 1e-6, cos.numpy(), sin.numpy(),
                                  pos.numpy(), kc, vc, slots.numpy())
    kflat = kc.reshape(-1, kvh, d)
    for got, want in ((q_o, bits(q_t)), (kflat[slots.numpy()], bits(k_t))):
        diff = np.abs(got.astype(np.int32) - want.astype(np.int32))
        assert (diff == 0).mean() > 0.99 and diff.max() <= 1
    assert np.array_equal(vc.reshape(-1, kvh, d)[slots.numpy()], bits(v))
