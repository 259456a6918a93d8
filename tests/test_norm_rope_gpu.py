"""Fused q/k RMSNorm + rotary embedding + KV append (nvk_qk_norm_rope_append)
against the oracle restatement of qwen3.py:83-96: v rows bit-exact in the
pool, rotated q and k over 99 % bit-identical and all within one bf16 unit in
the last place of the value plus one of the row's largest entry (fp32
reduction order and rsqrt differ from numpy's, so the norm's bf16 output can
round the other way; a rotation that cancels to ~0 keeps only that absolute
accuracy); strided rows
(slices of a fused QKV output), decode- and prefill-sized token counts, a
bad slot skipped and flagged."""

import numpy as np
import pytest
import torch

from nano_vllm_ascend_b200 import ops
from oracle import paged_kv_oracle as orc
from tests.helpers import bits

pytestmark = pytest.mark.gpu


def rope_tables(max_pos, d=128, theta=1e6):
    inv = 1.0 / (theta ** (torch.arange(0, d, 2, dtype=torch.float32) / d))
    freqs = torch.outer(torch.arange(max_pos, dtype=torch.float32), inv)
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos(), emb.sin()


def ulp_diff(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    ai, bi = a.astype(np.int32), b.astype(np.int32)
    ai = np.where(ai & 0x8000, 0x8000 - ai, ai)  # sign-magnitude -> ordered integers
    bi = np.where(bi & 0x8000, 0x8000 - bi, bi)
    return np.abs(ai - bi)


@pytest.mark.parametrize("tokens,h,kvh", [(1, 16, 8), (32, 16, 8), (777, 32, 8), (8192, 16, 8)])
def test_norm_rope_append_vs_oracle(cuda_device, tokens, h, kvh):
    dev = cuda_device
    g = torch.Generator(device=dev).manual_seed(tokens + h)
    qkv = (torch.randn(tokens, h + 2 * kvh, 128, generator=g, device=dev) * 3).to(torch.bfloat16)
    q, k, v = qkv[:, :h], qkv[:, h:h + kvh], qkv[:, h + kvh:]
    wq = (1 + 0.1 * torch.randn(128, generator=g, device=dev)).to(torch.bfloat16)
    wk = (1 + 0.1 * torch.randn(128, generator=g, device=dev)).to(torch.bfloat16)
    max_pos = 40960
    cos, sin = rope_tables(max_pos)
    positions = torch.randint(0, max_pos, (tokens,), generator=torch.Generator().manual_seed(3))
    nb = (tokens + 127) // 128 + 3
    slots = torch.randperm(nb * 128, generator=torch.Generator().manual_seed(4))[:tokens]
    kc = torch.zeros(nb, 128, kvh, 128, dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    q_out = ops.qk_norm_rope_append(q, k, v, wq, wk, 1e-6, cos.to(dev), sin.to(dev), positions.to(dev), kc, vc,
                                    slots.to(dev), error_word=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    kc_ref = np.zeros((nb, 128, kvh, 128), dtype=np.uint16)
    vc_ref = np.zeros_like(kc_ref)
    q_ref = orc.qk_norm_rope_append(bits(q), bits(k), bits(v), bits(wq), bits(wk), 1e-6, cos.numpy(), sin.numpy(),
                                    positions.numpy(), kc_ref, vc_ref, slots.numpy())
    assert np.array_equal(bits(vc), vc_ref), "v rows must be copied bit for bit"
    for name, got, want in (("q", bits(q_out), q_ref), ("k pool", bits(kc), kc_ref)):
        d = ulp_diff(got, want)
        assert (d == 0).mean() > 0.99, f"{name}: only {(d == 0).mean():.4f} bit-identical"
        # One bf16 ulp of the value plus one of the row's largest entry: the
        # norm's bf16 output can round the other way near a tie, and a rotation
        # that cancels to ~0 then keeps only that absolute accuracy.
        g32, w32 = orc.bf16_bits_to_f32(got), orc.bf16_bits_to_f32(want)
        row_max = np.abs(w32).max(axis=-1, keepdims=True)
        bad = np.abs(g32 - w32) > (np.abs(w32) + row_max) * 2.0 ** -8
        assert not bad.any(), f"{name}: {int(bad.sum())} values outside 1 ulp of value + row max"


def test_norm_rope_append_bad_slot(cuda_device):
    dev = cuda_device
    q = torch.randn(3, 16, 128, device=dev).to(torch.bfloat16)
    k = torch.randn(3, 8, 128, device=dev).to(torch.bfloat16)
    cos, sin = rope_tables(64)
    kc = torch.zeros(2, 128, 8, 128, dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    w = torch.ones(128, dtype=torch.bfloat16, device=dev)
    ops.qk_norm_rope_append(q, k, k, w, w, 1e-6, cos.to(dev), sin.to(dev), torch.tensor([1, 2, 3], device=dev),
                            kc, vc, torch.tensor([5, 256, -1], device=dev), error_word=err)
    torch.cuda.synchronize()
    assert int(err.item()) & 4
    flat = vc.view(-1, 8, 128)
    assert torch.equal(flat[5], k[0]) and int((vc != 0).sum()) == 8 * 128


def _prefill_inputs(dev, tokens, h, kvh, row_pad, seed):
    """q, k, v as slices of one fused QKV buffer whose token stride is
    (h + 2 kvh) * 128 + row_pad elements (row_pad = 2 makes the rows 4-byte
    but not 16-byte aligned)."""
    g = torch.Generator(device=dev).manual_seed(seed)
    width = (h + 2 * kvh) * 128
    buf = torch.zeros(tokens, width + row_pad, dtype=torch.bfloat16, device=dev)
    buf[:, :width] = (torch.randn(tokens, width, generator=g, device=dev) * 3).to(torch.bfloat16)
    qkv = buf[:, :width].view(tokens, h + 2 * kvh, 128)
    return qkv[:, :h], qkv[:, h:h + kvh], qkv[:, h + kvh:]


def test_norm_rope_append_row_padding_bit_identical(cuda_device):
    """A prefill-sized launch (one warp per token) over fused-QKV slices whose
    token stride is padded to break 16-byte row alignment gives the same bits
    as the aligned layout (q out, k and v pool rows)."""
    dev = cuda_device
    tokens, h, kvh = 4096, 16, 8
    cos, sin = rope_tables(40960)
    cos, sin = cos.to(dev), sin.to(dev)
    positions = torch.randint(0, 40960, (tokens,), generator=torch.Generator().manual_seed(8)).to(dev)
    nb = tokens // 128 + 2
    slots = torch.randperm(nb * 128, generator=torch.Generator().manual_seed(9))[:tokens].to(dev)
    w = (1 + 0.1 * torch.randn(2, 128, generator=torch.Generator().manual_seed(10))).to(torch.bfloat16).to(dev)
    outs = []
    for pad in (0, 2):
        q, k, v = _prefill_inputs(dev, tokens, h, kvh, pad, seed=11)
        assert (q.stride(0) % 8 == 0) == (pad == 0)
        kc = torch.zeros(nb, 128, kvh, 128, dtype=torch.bfloat16, device=dev)
        vc = torch.zeros_like(kc)
        err = torch.zeros(1, dtype=torch.int32, device=dev)
        q_out = ops.qk_norm_rope_append(q, k, v, w[0], w[1], 1e-6, cos, sin, positions, kc, vc, slots,
                                        error_word=err)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        outs.append((q_out, kc, vc))
    for a, b in zip(outs[0], outs[1]):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))


def test_norm_rope_append_prefill_bad_slots(cuda_device):
    """Prefill-sized launch: tokens whose slot is negative or past the pool
    are flagged and their k/v rows skipped; every other token lands as the
    oracle says."""
    dev = cuda_device
    tokens, h, kvh = 4096, 16, 8
    q, k, v = _prefill_inputs(dev, tokens, h, kvh, 0, seed=12)
    cos, sin = rope_tables(4096)
    positions = torch.randint(0, 4096, (tokens,), generator=torch.Generator().manual_seed(13))
    nb = tokens // 128 + 2
    slots = torch.randperm(nb * 128, generator=torch.Generator().manual_seed(14))[:tokens]
    bad = [7, 2000, 4095]
    slots[bad[0]], slots[bad[1]], slots[bad[2]] = -1, nb * 128, -5
    w = torch.ones(128, dtype=torch.bfloat16, device=dev)
    kc = torch.zeros(nb, 128, kvh, 128, dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    q_out = ops.qk_norm_rope_append(q, k, v, w, w, 1e-6, cos.to(dev), sin.to(dev), positions.to(dev), kc, vc,
                                    slots.to(dev), error_word=err)
    torch.cuda.synchronize()
    assert int(err.item()) & 4
    good = np.setdiff1d(np.arange(tokens), bad)
    kc_ref = np.zeros((nb, 128, kvh, 128), dtype=np.uint16)
    vc_ref = np.zeros_like(kc_ref)
    q_ref = orc.qk_norm_rope_append(bits(q)[good], bits(k)[good], bits(v)[good], bits(w), bits(w), 1e-6,
                                    cos.numpy(), sin.numpy(), positions.numpy()[good], kc_ref, vc_ref,
                                    slots.numpy()[good])
    assert np.array_equal(bits(vc), vc_ref)
    for got, want in ((bits(q_out)[good], q_ref), (bits(kc), kc_ref)):
        d = ulp_diff(got, want)
        assert (d == 0).mean() > 0.99
        g32, w32 = orc.bf16_bits_to_f32(got), orc.bf16_bits_to_f32(want)
        row_max = np.abs(w32).max(axis=-1, keepdims=True)
        assert not (np.abs(g32 - w32) > (np.abs(w32) + row_max) * 2.0 ** -8).any()
