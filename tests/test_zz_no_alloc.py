"""The allocation-free decode entry point (nvk_paged_decode_noalloc).

It serves callers that cannot allocate device memory where they run
attention -- a plugin enqueue inside a framework that owns every device
buffer, a cgo/JNI/N-API binding with no device allocator, a serving thread
that must not take cudaMalloc's implicit synchronisation -- by keeping the
split-K scratch in a fixed array of the library's device memory.

Checks, through the C ABI:
* two calls in a row (the second reuses the array the first left behind, with
  a different split count and different inputs) each match the workspace
  entry point nvk_paged_decode within the attention tolerance of the other
  tests, and the fp32 oracle;
* the calls leave the device's free memory unchanged (nothing is allocated);
* a call with a block id outside the pool reports bit 2 through
  nvk_paged_decode_noalloc_error, and the good call after it (which starts
  from the scratch the bad one left) reports 0 and matches nvk_paged_decode;
* a shape whose scratch need exceeds the array is refused on the host with
  NVK_ERR_UNSUPPORTED, after the ordinary argument checks.
This file sorts last so that a stop-at-first-failure run has already run
every other test.
"""

import ctypes

import numpy as np
import pytest
import torch

from nano_vllm_ascend_b200 import _lib, ops
from oracle import paged_kv_oracle as orc
from tests.helpers import assert_close, bits, random_pool, seeded_tables

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 16 << 20
SCALE = 128 ** -0.5


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _stream(device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


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
    return lib.nvk_paged_decode_noalloc(_p(out), _p(q), _p(kc), _p(vc), nb, bs, _p(tables), tables.stride(0),
                                        tables.shape[1], _p(ctx_t), b, h, kvh, d, SCALE, num_ctas,
                                        _stream(q.device))


def _noalloc_error(lib, device) -> int:
    word = ctypes.c_int(-1)
    rc = lib.nvk_paged_decode_noalloc_error(ctypes.byref(word), _stream(device))
    assert rc == _lib.NVK_OK, lib.nvk_last_error()
    return word.value


def _workspace_decode(q, kc, vc, tables, ctx_t, num_ctas):
    ws = torch.zeros(ops.decode_workspace_bytes(q.shape[0], q.shape[1], kc.shape[2], 128, num_ctas),
                     dtype=torch.uint8, device=q.device)
    want = torch.empty_like(q)
    ops.paged_decode(want, q, kc, vc, tables, ctx_t, SCALE, ws, num_ctas)
    torch.cuda.synchronize()
    return want, ops.decode_error_word(ws)


def test_noalloc_decode_matches_workspace_decode_on_two_calls(cuda_device):
    lib = _lib.load()
    # the second call uses a different grid, so a different set of partial slots
    cases = [([2900, 17, 1300, 640, 129, 1], 0, 0), ([600, 3000, 5, 2048], 1, 5)]
    prepared = []
    for ctx, seed, num_ctas in cases:
        q, kc, vc, tables, ctx_t = _inputs(cuda_device, ctx, seed)
        want, err = _workspace_decode(q, kc, vc, tables, ctx_t, num_ctas)
        assert err == 0
        prepared.append((q, kc, vc, tables, ctx_t, num_ctas, want))
    outs = [torch.full_like(p[0], float("nan")) for p in prepared]
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info(cuda_device)[0]
    # two calls in a row on one stream: the second reuses the scratch the first left behind
    for got, (q, kc, vc, tables, ctx_t, num_ctas, _) in zip(outs, prepared):
        rc = _noalloc(lib, got, q, kc, vc, tables, ctx_t, num_ctas)
        assert rc == _lib.NVK_OK, lib.nvk_last_error()
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info(cuda_device)[0] == free_before, "the no-alloc calls changed free device memory"
    assert _noalloc_error(lib, cuda_device) == 0
    for i, (got, prep) in enumerate(zip(outs, prepared)):
        q, kc, vc, tables, ctx_t, _, want = prep
        assert not torch.isnan(got.float()).any()
        assert_close(got.float().cpu().numpy(), want.float().cpu().numpy(), f"noalloc call {i + 1} vs workspace")
        ref = orc.paged_decode(bits(q), bits(kc), bits(vc), tables.cpu().numpy(), ctx_t.cpu().numpy(), SCALE)
        assert_close(got.float().cpu().numpy(), ref, f"noalloc call {i + 1} vs oracle")


def test_noalloc_decode_reports_a_bad_block_id_then_recovers(cuda_device):
    lib = _lib.load()
    ctx = [700, 130, 2048]
    q, kc, vc, tables, ctx_t = _inputs(cuda_device, ctx, 7)
    bad_tables = tables.clone()
    bad_tables[1, 1] = kc.shape[0] + 3  # outside the pool: zero-filled and flagged, never read
    got = torch.empty_like(q)
    assert _noalloc(lib, got, q, kc, vc, bad_tables, ctx_t, 0) == _lib.NVK_OK, lib.nvk_last_error()
    assert _noalloc_error(lib, cuda_device) & 2, "bad block id not reported"
    # the next call starts from the scratch the flagged call left behind
    got = torch.full_like(q, float("nan"))
    assert _noalloc(lib, got, q, kc, vc, tables, ctx_t, 0) == _lib.NVK_OK, lib.nvk_last_error()
    assert _noalloc_error(lib, cuda_device) == 0
    want, err = _workspace_decode(q, kc, vc, tables, ctx_t, 0)
    assert err == 0
    assert_close(got.float().cpu().numpy(), want.float().cpu().numpy(), "call after a flagged call")


def test_noalloc_decode_refuses_shapes_beyond_its_scratch(cuda_device):
    lib = _lib.load()
    # one arrival ticket per (sequence, KV head): 1M sequences x 8 heads x 128 B > 16 MiB
    batch = 1 << 20
    need = ops.decode_workspace_bytes(batch, 16, 8, 128)
    assert need > SCRATCH_BYTES
    q = torch.empty(1, 16, 128, dtype=torch.bfloat16, device=cuda_device)
    kc = torch.empty(8, 128, 8, 128, dtype=torch.bfloat16, device=cuda_device)
    tables = torch.zeros(1, 64, dtype=torch.int32, device=cuda_device)
    ctx_t = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    # the pointers are never dereferenced: the size check refuses the call before any launch
    rc = lib.nvk_paged_decode_noalloc(_p(q), _p(q), _p(kc), _p(kc), 8, 128, _p(tables), 64, 64, _p(ctx_t), batch,
                                      16, 8, 128, SCALE, 0, _stream(cuda_device))
    assert rc == _lib.NVK_ERR_UNSUPPORTED
    assert b"static scratch" in lib.nvk_last_error()
