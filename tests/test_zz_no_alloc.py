"""The allocation-free decode entry point (nvk_paged_decode_noalloc).

It serves callers that cannot allocate device memory where they run
attention -- a plugin enqueue inside a framework that owns every device
buffer, a cgo/JNI/N-API binding with no device allocator, a serving thread
that must not take cudaMalloc's implicit synchronisation -- by keeping the
split-K scratch in a fixed array of the library's device memory.

Checks, through the C ABI: two calls in a row (the second reuses the array
the first left behind, with a different split count and different inputs)
each match the workspace entry point nvk_paged_decode within the attention
tolerance of the other tests; a shape whose scratch need exceeds the array is
refused on the host with NVK_ERR_UNSUPPORTED. This file sorts last so that a
stop-at-first-failure run has already run every other test.
"""

import ctypes
import pytest
import torch

from nano_vllm_ascend_b200 import _lib, ops
from tests.helpers import assert_close, random_pool, seeded_tables

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 16 << 20


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _inputs(device, ctx, seed, h=16, kvh=8, bs=128):
    need = sum((n + bs - 1) // bs for n in ctx)
    nb = need + 4
    kc, vc = random_pool(nb, bs, kvh, 128, device, seed)
    tables = seeded_tables(ctx, bs, nb, seed, width=24).to(device)
    g = torch.Generator(device=device).manual_seed(seed + 100)
    q = torch.randn(len(ctx), h, 128, generator=g, device=device).to(torch.bfloat16)
    ctx_t = torch.tensor(ctx, dtype=torch.int32, device=device)
    return q, kc, vc, tables, ctx_t


def _noalloc(lib, out, q, kc, vc, tables, ctx_t, num_ctas):
    b, h, d = q.shape
    nb, bs, kvh, _ = kc.shape
    stream = ctypes.c_void_p(torch.cuda.current_stream(q.device).cuda_stream)
    return lib.nvk_paged_decode_noalloc(_p(out), _p(q), _p(kc), _p(vc), nb, bs, _p(tables), tables.stride(0),
                                        tables.shape[1], _p(ctx_t), b, h, kvh, d, 128 ** -0.5, num_ctas, stream)


def test_noalloc_decode_matches_workspace_decode_on_two_calls(cuda_device):
    lib = _lib.load()
    # the second call uses a different grid, so a different set of partial slots
    cases = [([2900, 17, 1300, 640, 129, 1], 0, 0), ([600, 3000, 5, 2048], 1, 5)]
    prepared = []
    for ctx, seed, num_ctas in cases:
        q, kc, vc, tables, ctx_t = _inputs(cuda_device, ctx, seed)
        ws = torch.zeros(ops.decode_workspace_bytes(len(ctx), 16, 8, 128, num_ctas), dtype=torch.uint8,
                         device=cuda_device)
        want = torch.empty_like(q)
        ops.paged_decode(want, q, kc, vc, tables, ctx_t, 128 ** -0.5, ws, num_ctas)
        torch.cuda.synchronize()
        assert ops.decode_error_word(ws) == 0
        prepared.append((q, kc, vc, tables, ctx_t, num_ctas, want))
    # two calls in a row on one stream: the second reuses the scratch the first left behind
    outs = []
    for q, kc, vc, tables, ctx_t, num_ctas, _ in prepared:
        got = torch.full_like(q, float("nan"))
        rc = _noalloc(lib, got, q, kc, vc, tables, ctx_t, num_ctas)
        assert rc == _lib.NVK_OK, lib.nvk_last_error()
        outs.append(got)
    torch.cuda.synchronize()
    for i, (got, prep) in enumerate(zip(outs, prepared)):
        want = prep[-1]
        assert not torch.isnan(got.float()).any()
        assert_close(got.float().cpu().numpy(), want.float().cpu().numpy(), f"noalloc call {i + 1} vs workspace")


def test_noalloc_decode_refuses_shapes_beyond_its_scratch(cuda_device):
    lib = _lib.load()
    # one arrival ticket per (sequence, KV head): 1M sequences x 8 heads x 4 B > 16 MiB
    need = ops.decode_workspace_bytes(1 << 20, 16, 8, 128)
    assert need > SCRATCH_BYTES
    n = ctypes.c_void_p(0)
    rc = lib.nvk_paged_decode_noalloc(n, n, n, n, 8, 128, n, 64, 64, n, 1 << 20, 16, 8, 128, 0.1, 0,
                                      ctypes.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream))
    assert rc == _lib.NVK_ERR_UNSUPPORTED
    assert b"static scratch" in lib.nvk_last_error()
