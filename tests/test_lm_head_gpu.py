"""LM head + greedy argmax on the device (nvk_lm_head_argmax) against the
oracle (bf16 logits of hidden @ W.T, first index of the maximum): every row
picks the oracle's token or, where the oracle's top logits tie within one
bf16 unit (f32 summation order differs), a token whose logit is that maximum;
planted clear winners are picked exactly; the workspace is left zeroed for
the next call; vocabularies not a multiple of the 128-row tile."""

import numpy as np
import pytest
import torch

from nano_vllm_ascend_b200 import ops
from oracle import paged_kv_oracle as orc
from tests.helpers import bits

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("batch,vocab,hsize", [(1, 151936, 1024), (32, 151936, 1024), (5, 1000, 1024),
                                               (100, 20000, 4096), (17, 333, 128)])
def test_lm_head_argmax_vs_oracle(cuda_device, batch, vocab, hsize):
    dev = cuda_device
    g = torch.Generator(device=dev).manual_seed(batch + vocab)
    hidden = torch.randn(batch, hsize, generator=g, device=dev).to(torch.bfloat16)
    weight = (torch.randn(vocab, hsize, generator=g, device=dev) * 0.05).to(torch.bfloat16)
    # plant a clear winner for every other row
    winners = torch.randint(0, vocab, (batch,), generator=torch.Generator().manual_seed(1))
    for b in range(0, batch, 2):
        weight[winners[b]] = (hidden[b].float() * 0.5).to(torch.bfloat16)
    ws = torch.zeros(ops.lm_head_argmax_workspace_bytes(batch), dtype=torch.uint8, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    got = None
    for _ in range(2):  # the second call checks the workspace was left clean
        got = ops.lm_head_argmax(hidden, weight, ws, error_word=err).cpu().numpy()
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert int(ws.abs().sum()) == 0, "workspace must be zero after a call"
    logits = orc.lm_head_logits(bits(hidden), bits(weight))
    want = orc.greedy_tokens(logits)
    rows = np.arange(batch)
    top = logits[rows, want]
    picked = logits[rows, got]
    ulp = np.abs(top) * 2.0 ** -8
    assert np.all(top - picked <= ulp), "a picked token's logit is below the maximum by more than one bf16 ulp"
    assert (got == want).mean() >= 0.9
    for b in range(0, batch, 2):
        assert got[b] == winners[b], f"row {b}: planted winner {int(winners[b])}, got {got[b]}"


@pytest.mark.parametrize("vocab,num_ctas", [(4099, 7), (4099, 0), (151936, 137), (151936, 0), (333, 5)])
def test_lm_head_argmax_range_edges(cuda_device, vocab, num_ctas):
    """CTA c covers 128-row tiles [T*c/C, T*(c+1)/C) of the vocabulary (the
    last tile partly past its end): planted winners on the first and last rows
    of every CTA's range, next to tile edges inside it and on the last vocab
    row are each picked exactly."""
    dev = cuda_device
    hsize = 1024
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    tiles = -(-vocab // 128)
    ctas = min(num_ctas or sms, tiles)
    edges = set()
    for c in range(ctas):
        lo, hi = tiles * c // ctas * 128, min(tiles * (c + 1) // ctas * 128, vocab)
        edges.update((lo, hi - 1, lo + 127, lo + 128, hi - 129))
    rows = sorted(r for r in edges if 0 <= r < vocab)
    rows = sorted(set(rows[:: max(1, len(rows) // 120)][:120] + [vocab - 1]))
    batch = len(rows)
    g = torch.Generator(device=dev).manual_seed(vocab + ctas)
    hidden = torch.randn(batch, hsize, generator=g, device=dev).to(torch.bfloat16)
    weight = (torch.randn(vocab, hsize, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    for b, r in enumerate(rows):
        weight[r] = (hidden[b].float() * 0.5).to(torch.bfloat16)
    ws = torch.zeros(ops.lm_head_argmax_workspace_bytes(batch), dtype=torch.uint8, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    got = ops.lm_head_argmax(hidden, weight, ws, num_ctas=num_ctas, error_word=err).cpu().numpy()
    torch.cuda.synchronize()
    assert int(err.item()) == 0 and int(ws.abs().sum()) == 0
    assert got.tolist() == rows
