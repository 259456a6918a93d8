"""KV-head-sharded decode with the output all-gather inside the kernel
(nvk_paged_decode_gather, nano_vllm_ascend_b200.peer_gather).

* one rank: the gather path stores this rank's heads into a head range of a
  wider output and signals itself; repeated calls cycle slots and epochs; the
  rows of other heads are never written;
* two ranks on two GPUs (skipped with fewer GPUs): each rank holds half the KV
  heads of the same synthetic pool; after every call each rank's gathered
  output equals the fp32 oracle over ALL heads;
* a peer that never posts its epoch (a flag nothing sets): the bounded wait
  runs out, the call reports error bit 16 and the GPU stays usable.
"""

import ctypes
import os
import socket
import time

import numpy as np
import pytest
import torch

from nano_vllm_ascend_b200 import _lib, ops
from nano_vllm_ascend_b200.peer_gather import PeerGather
from oracle import paged_kv_oracle as orc
from tests.helpers import assert_close, bits, seeded_tables

pytestmark = pytest.mark.gpu

H, KVH, D, BS = 32, 8, 128, 128
SCALE = D ** -0.5


def full_problem(ctx, seed):
    """Pool, tables and queries of all heads, generated on the host (identical on every rank)."""
    nb = sum((n + BS - 1) // BS for n in ctx) + 5
    g = torch.Generator().manual_seed(seed)
    kc = torch.randn(nb, BS, KVH, D, generator=g).to(torch.bfloat16)
    vc = torch.randn(nb, BS, KVH, D, generator=g).to(torch.bfloat16)
    q = torch.randn(len(ctx), H, D, generator=g).to(torch.bfloat16)
    tables = seeded_tables(ctx, BS, nb, seed)
    want = orc.paged_decode(bits(q), bits(kc), bits(vc), tables.numpy(), np.array(ctx), SCALE)
    return kc, vc, q, tables, want


def shard(kc, vc, q, kv_lo, kv_hi, device):
    qpk = H // KVH
    return (kc[:, :, kv_lo:kv_hi].contiguous().to(device), vc[:, :, kv_lo:kv_hi].contiguous().to(device),
            q[:, kv_lo * qpk: kv_hi * qpk].contiguous().to(device))


def test_gather_single_rank_head_range(cuda_device):
    ctx = [1, 130, 700, 2000, 37]
    kc, vc, q, tables, want = full_problem(ctx, seed=3)
    kc_l, vc_l, q_l = shard(kc, vc, q, 2, 4, cuda_device)  # KV heads 2-3 -> query heads 8-15
    tables = tables.to(cuda_device)
    ctx_t = torch.tensor(ctx, dtype=torch.int32, device=cuda_device)
    ws = torch.zeros(ops.decode_workspace_bytes(len(ctx), 8, 2, D), dtype=torch.uint8, device=cuda_device)
    pg = PeerGather(len(ctx), H, D, slots=2, device=cuda_device)
    try:
        for call in range(3):
            out = pg.decode(q_l, kc_l, vc_l, tables, ctx_t, SCALE, ws, head_offset=8)
            torch.cuda.synchronize()
            assert ops.decode_error_word(ws) == 0
            got = out.float().cpu().numpy()
            assert_close(got[:, 8:16], want[:, 8:16], f"call {call}")
            assert not got[:, :8].any() and not got[:, 16:].any(), "rows of other heads were written"
        sig = pg._buffer[:256].view(torch.int32).cpu()
        assert int(sig[0]) == 3 and int(sig[8]) == 3, "epoch flag / counter after three calls"
        assert int(ws[64:68].view(torch.int32).item()) == 0, "CTA counter returns to zero"
    finally:
        pg.close()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _two_rank_worker(rank: int, port: int, world: int) -> None:
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        ctx = [5, 128, 129, 900, 3000, 64, 2500, 17]
        kc, vc, q, tables, want = full_problem(ctx, seed=11)
        per = KVH // world
        kc_l, vc_l, q_l = shard(kc, vc, q, rank * per, (rank + 1) * per, dev)
        tables = tables.to(dev)
        ctx_t = torch.tensor(ctx, dtype=torch.int32, device=dev)
        hl = q_l.shape[1]
        ws = torch.zeros(ops.decode_workspace_bytes(len(ctx), hl, per, D), dtype=torch.uint8, device=dev)
        pg = PeerGather(len(ctx), H, D, slots=2, device=dev)
        try:
            for call in range(4):
                out = pg.decode(q_l, kc_l, vc_l, tables, ctx_t, SCALE, ws, head_offset=rank * hl)
                torch.cuda.synchronize(dev)
                assert ops.decode_error_word(ws) == 0, f"rank {rank} error word"
                assert_close(out.float().cpu().numpy(), want, f"rank {rank} call {call}")
                dist.barrier()
        finally:
            pg.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_gather_two_ranks_two_gpus():
    import torch.multiprocessing as mp

    mp.spawn(_two_rank_worker, args=(_free_port(), 2), nprocs=2, join=True)


def test_gather_epoch_wait_runs_out_and_reports(cuda_device):
    """world = 2 in one process, both "ranks'" output and signal areas local:
    rank 1 never posts its epoch, so the last CTA's wait (bounded at 1 s)
    gives up, sets bit 16 of the error word and returns. This rank's rows
    still reached both output buffers, and a following launch works."""
    dev = cuda_device
    ctx = [100, 300, 1]
    kc, vc, q, tables, want = full_problem(ctx, seed=5)
    kc_d, vc_d, q_d, tables_d = kc.to(dev), vc.to(dev), q.to(dev), tables.to(dev)
    ctx_t = torch.tensor(ctx, dtype=torch.int32, device=dev)
    b = len(ctx)
    ws = torch.zeros(ops.decode_workspace_bytes(b, H, KVH, D), dtype=torch.uint8, device=dev)
    bufs = [torch.zeros(_lib.PEER_SIGNAL_BYTES + b * H * D * 2, dtype=torch.uint8, device=dev) for _ in range(2)]
    pad = [0] * (_lib.MAX_PEERS - 2)
    outs = (ctypes.c_void_p * _lib.MAX_PEERS)(*([t.data_ptr() + _lib.PEER_SIGNAL_BYTES for t in bufs] + pad))
    sigs = (ctypes.c_void_p * _lib.MAX_PEERS)(*([t.data_ptr() for t in bufs] + pad))
    stream = torch.cuda.current_stream(dev).cuda_stream
    torch.cuda.synchronize()
    t0 = time.time()
    _lib.call("nvk_paged_decode_gather", q_d.data_ptr(), kc_d.data_ptr(), vc_d.data_ptr(), kc_d.shape[0], BS,
              tables_d.data_ptr(), tables_d.stride(0), tables_d.shape[1], ctx_t.data_ptr(), b, H, KVH, D, SCALE, 0,
              ws.data_ptr(), ws.numel(), outs, sigs, 2, 0, H, 0, None, None, 0, 0, None, stream)
    torch.cuda.synchronize()
    elapsed = time.time() - t0
    assert ops.decode_error_word(ws) & 16, "the epoch wait must report its timeout"
    assert 0.5 < elapsed < 20.0
    for t in bufs:
        got = t[_lib.PEER_SIGNAL_BYTES:].view(torch.bfloat16).view(b, H, D).float().cpu().numpy()
        assert_close(got, want, "rows stored before the wait")
    out = torch.empty_like(q_d)
    ws2 = torch.zeros_like(ws)
    ops.paged_decode(out, q_d, kc_d, vc_d, tables_d, ctx_t, SCALE, ws2)
    torch.cuda.synchronize()
    assert ops.decode_error_word(ws2) == 0
    assert_close(out.float().cpu().numpy(), want, "launch after the timeout")
