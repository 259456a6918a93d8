#!/usr/bin/env python
"""Benchmark of the B200 paged-KV hot path.

    python bench.py [--gpus N] [--steps K] [--warmup W]
                    [--workload decode_c2|decode_c4|decode_c5|prefill_c3|kernels]
                    [--impl ours|reference]

Without --workload (what the driver runs) one JSON line is printed whose
headline is config 2 (decode_c2) and whose ``sub_results`` carry the other
configs measured in the same run, one after another on the same GPUs:
prefill_c3, decode_c4 and step_c2 at N = 1; decode_c4, step_c2 and decode_c5
at N > 1. Every
workload first measures, then checks a sampled slice of its own output on the
box against an fp32 torch-CPU reference (``parity``), so each number is
backed by a parity verdict of the same run. --workload X prints X alone.

A decode "step" is one decode step of the configured batch through every
layer: per layer, the KV append of this step's token and paged GQA decode
attention over the whole context, replayed as ONE CUDA graph captured by
DecodeGraphRunner at the batch size. The runner defers each layer's
PagedKVCache.write so that the decode kernel performs the append itself
(nvk_paged_decode_append): one launch per layer.

Workloads (seeded synthetic inputs with the configs' shapes; no model weights):
  decode_c2 (headline): 28 layers, 32 sequences, context ~ U[256, 2304], 16
      query / 8 KV heads, head_dim 128, block 128, pool = 80% of free HBM,
      block tables drawn without replacement from a seeded permutation of the
      pool. At N > 1 every rank runs its own such batch on its own pool
      (sequence-sharded replicas, no collective): weak scaling.
  decode_c4: 256 sequences, context ~ U[2048, 6144], split evenly across
      ranks by sequence (strong scaling).
  prefill_c3: config[2]: 32 requests sharing a hash-hit 768-token prefix
      (6 cached blocks in the real BlockManager) prefill their 256 new tokens
      each: per layer the 8192-row append and prefix-aware causal attention
      over 1024 keys; value = attention TF/s of the step.
  decode_c5: Qwen3-8B KV shapes (36 layers, 32 query / 8 KV heads), 128
      sequences at context 8192, KV-head sharded over N in {2, 4, 8} GPUs
      (the pool does not fit one GPU). Per layer: append of this rank's KV
      heads, then decode attention over them whose output rows go straight
      into every rank's gathered [128, 32, 128] output (in-kernel all-gather
      over NVLink, --gather kernel) or, as the baseline, decode followed by an
      NCCL all_gather_into_tensor and a permuting copy (--gather nccl).
  step_c2: config 2 through StepRunner (the reference's ModelRunner step
      drivers): a Qwen3-0.6B-shaped model with seeded random weights, 32
      sequences prefilled to context ~U[256, 2304], then greedy decode steps
      from one CUDA graph (device metadata, 28 layers of fused q/k norm + RoPE
      + append, paged decode, cuBLAS projections and MLP, LM head + argmax)
      with the next tokens read back every step; value = decode tok/s.
  kernels: the path's other kernels timed one by one under CUDA graphs on
      config-sized inputs (prefill-sized append, decode- and prefill-sized
      q/k norm + RoPE + append, device decode metadata, LM head + greedy
      argmax over the 151,936-token vocabulary), with bytes moved and the
      fraction of the measured HBM copy bandwidth.

Printed per workload: value = KV bytes read by decode attention per step,
summed over ranks, / max-over-ranks step time (GB/s) for decode, attention
TF/s for prefill; the dominant kernel's roofline (timed alone with CUDA events
on its stream, one launch per layer captured in a CUDA graph, cycling layers
so that every launch reads HBM); appends over four rotating source sets
(block-contiguous and scattered slots); an end-to-end figure through the
public API with pinned host inputs and a device->host read of the outputs;
SM clocks sampled by nvidia-smi during the measurement; per-rank step times
and clocks at N > 1; the CPU baseline (eager torch-CPU expression of the
reference path on a bounded sample, rank 0 at N = 1).

--impl reference times that CPU path alone on the host cores (rank 0 only):
whole decode steps (every layer of the workload on the same one-layer host
pool), with the same ``config`` as this arm.
"""

from __future__ import annotations

import argparse
import gc
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from dataclasses import dataclass
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
KVH, HEAD_DIM, BLOCK = 8, 128, 128
ATOL, RTOL = 2e-2, 1e-2  # attention tolerance vs fp32 (bf16 outputs)


@dataclass
class Workload:
    name: str
    layers: int
    batch: int
    heads: int
    kv_heads: int
    ctx_lo: int
    ctx_hi: int
    scaling: str  # "weak": batch per rank; "strong": batch split across ranks
    util: float = 0.8
    describe: str = ""


WORKLOADS = {
    "decode_c2": Workload("decode_c2", 28, 32, 16, 8, 256, 2304, "weak",
                          describe="config[1]: Qwen3-0.6B decode step, 32 seqs, ctx~U[256,2304], CUDA graph bs 32"),
    "decode_c4": Workload("decode_c4", 28, 256, 16, 8, 2048, 6144, "strong",
                          describe="config[3]: Qwen3-0.6B decode step, 256 seqs, ctx~U[2048,6144], sequence-sharded"),
    "decode_c5": Workload("decode_c5", 36, 128, 32, 8, 8192, 8192, "strong",
                          describe="config[4]: Qwen3-8B KV cache, 128 seqs at ctx 8192, KV-head sharded, "
                                   "outputs all-gathered"),
    "kernels": Workload("kernels", 28, 32, 16, 8, 256, 2304, "weak",
                        describe="the hot path's other kernels on config-2/3-sized inputs"),
    # prefill: ctx_lo = cached prefix tokens, ctx_hi = new tokens per request
    "prefill_c3": Workload("prefill_c3", 28, 32, 16, 8, 768, 256, "weak",
                           describe="config[2]: Qwen3-0.6B prefix-cache prefill, 32 requests x (768 cached + 256 new)"),
}


# --------------------------------------------------------------- helpers ----
def peaks(key: str = "hbm_gbs") -> tuple[float, str]:
    """Roofline denominators: measured copy bandwidth (GB/s) or bf16 GEMM
    TFLOP/s from MEASURED_PEAKS.json, else this pool's earlier measurement."""
    fallback = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())[key]), "measured"
        except Exception:
            pass
    return fallback[key], "fallback"


def profiled_value(workload: str, kernel: str, key: str) -> float | None:
    """A figure from a committed ncu summary: the line '<key>: N' in
    profiles/<kernel>_<workload>.txt."""
    p = ROOT / "profiles" / f"{kernel}_{workload}.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith(key + ":"):
            try:
                return float(line.split(":", 1)[1].split()[0].replace(",", ""))
            except ValueError:
                return None
    return None


def profiled_traffic(workload: str, kernel: str = "paged_decode") -> float | None:
    """Per-launch DRAM bytes of a kernel from its committed ncu summary."""
    return profiled_value(workload, kernel, "traffic_bytes_per_launch")


class ClockSampler:
    """nvidia-smi clock/throttle sampling in the background (every 200 ms)."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(prefix="clocks", suffix=".csv")
            os.close(fd)
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=self.fh, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.fh.close()

    def summary(self) -> dict:
        rows = []
        if self.path and os.path.exists(self.path):
            for line in open(self.path):
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
            os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None

        sm = [num(r[1]) for r in rows if num(r[1]) is not None]
        smax = [num(r[2]) for r in rows if num(r[2]) is not None]
        power = [num(r[3]) for r in rows if num(r[3]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        loaded = [s for s, p in zip(sm, power) if p is not None and p > 200] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": reasons, "samples": len(rows), "power_w_max": max(power) if power else None}


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and args.impl == "ours":
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    elif args.impl == "ours":
        torch.cuda.set_device(local)
    return world, rank, local


def barrier_sync(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    torch.cuda.synchronize()


def _reduce(x: float, world: int, op: str) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op={"max": dist.ReduceOp.MAX, "sum": dist.ReduceOp.SUM, "min": dist.ReduceOp.MIN}[op])
    return float(t.item())


def max_over_ranks(x: float, world: int) -> float:
    return _reduce(x, world, "max")


def sum_over_ranks(x: float, world: int) -> float:
    return _reduce(x, world, "sum")


def all_ranks(obj, world: int) -> list:
    if world == 1:
        return [obj]
    import torch.distributed as dist

    out = [None] * world
    dist.all_gather_object(out, obj)
    return out


def free_device_memory() -> None:
    gc.collect()
    torch.cuda.synchronize()
    torch.cuda.empty_cache()


# ----------------------------------------------------------------- setup ----
def rank_contexts(wl: Workload, world: int, rank: int) -> list[int]:
    """Context lengths (before this step's token) of this rank's sequences."""
    from nano_vllm_ascend_b200.sharding import token_balanced_shard

    if wl.scaling == "strong":
        # one batch split across the ranks by context length (equal KV bytes per rank)
        g = torch.Generator().manual_seed(0)
        ctx = torch.randint(wl.ctx_lo, wl.ctx_hi + 1, (wl.batch,), generator=g).tolist()
        return [ctx[i] for i in token_balanced_shard(ctx, world, rank)]
    # weak scaling: every rank decodes the same per-GPU workload (its own K/V
    # values and block tables, the same context lengths)
    g = torch.Generator().manual_seed(1000)
    return torch.randint(wl.ctx_lo, wl.ctx_hi + 1, (wl.batch,), generator=g).tolist()


def decode_config(wl: Workload, world: int) -> dict:
    """The workload as both arms name it (``config`` of the JSON line)."""
    batch_per_gpu = wl.batch if wl.scaling == "weak" else -(-wl.batch // world)
    global_batch = wl.batch * world if wl.scaling == "weak" else wl.batch
    ctx_after = [c + 1 for r in range(world) for c in rank_contexts(wl, world, r)]
    return {
        "workload": wl.describe,
        "layers": wl.layers,
        "batch_per_gpu": batch_per_gpu,
        "global_batch": global_batch,
        "seq_len": [wl.ctx_lo, wl.ctx_hi],
        "heads": [wl.heads, wl.kv_heads, HEAD_DIM],
        "block_size": BLOCK,
        "parallelism": f"sequence-sharded x{world}, independent pools, no collective",
        "cache": "inputs larger than L2: every step reads %.2f GB of KV"
                 % (kv_bytes_per_layer(ctx_after, wl.kv_heads) * wl.layers / 1e9),
    }


class AttentionOnlyDecoder:
    """Stands in for Qwen3ForCausalLM inside the decode graph: per layer, the
    reference's Qwen3Attention hot-path order (qwen3.py:91-117) -- append this
    step's K/V, then paged attention -- on static per-layer q/k/v buffers."""

    def __init__(self, layers: int, batch: int, heads: int, kv_heads: int, device, seed: int = 7):
        from nano_vllm_ascend_b200 import PagedAttention

        g = torch.Generator(device=device).manual_seed(seed)
        self.q = torch.randn(layers, batch, heads, HEAD_DIM, generator=g, device=device).to(torch.bfloat16)
        self.k = torch.randn(layers, batch, kv_heads, HEAD_DIM, generator=g, device=device).to(torch.bfloat16)
        self.v = torch.randn(layers, batch, kv_heads, HEAD_DIM, generator=g, device=device).to(torch.bfloat16)
        self.attn = PagedAttention(heads, kv_heads, HEAD_DIM)
        self.layers = layers

    def __call__(self, input_ids_flat, position_ids_flat, kv_cache, attn_metadata, is_prefill=False):
        outs = []
        for layer in range(self.layers):
            kv_cache.write(layer, self.k[layer], self.v[layer], attn_metadata.slot_mapping)
            kc, vc = kv_cache.get_physical_cache(layer)
            outs.append(self.attn(self.q[layer], kc, vc, attn_metadata.block_tables, attn_metadata.context_lens))

        class Out:
            logits = torch.stack(outs)

        return Out()


def build(wl: Workload, world: int, rank: int, device, pool_blocks: int = 0):
    from nano_vllm_ascend_b200 import BlockManager, PagedKVCache
    from nano_vllm_ascend_b200.pool import num_blocks_from_memory

    ctx = rank_contexts(wl, world, rank)
    b = len(ctx)
    num_blocks = num_blocks_from_memory(wl.util, wl.layers, BLOCK, wl.kv_heads, HEAD_DIM, torch.bfloat16, device)
    if pool_blocks > 0:
        num_blocks = min(num_blocks, pool_blocks)
    bm = BlockManager(num_blocks, BLOCK, device)
    g = torch.Generator().manual_seed(42 + rank)
    bm.free_block_ids = torch.randperm(num_blocks, generator=g).tolist()
    slots = list(range(b))
    bm.prepare_prefill_metadata(slots, ctx, [0] * b, [[] for _ in slots])
    md = bm.prepare_decode_metadata(slots, ctx, q_len=1)
    kv = PagedKVCache(wl.layers, num_blocks, BLOCK, wl.kv_heads, HEAD_DIM, torch.bfloat16, device)
    used = torch.unique(torch.cat([torch.tensor(bm.block_tables[s], dtype=torch.int64) for s in slots])).to(device)
    gen = torch.Generator(device=device).manual_seed(5 + rank)
    for layer in range(wl.layers):
        shape = (used.numel(), BLOCK, wl.kv_heads, HEAD_DIM)
        kv.key_cache[layer].index_copy_(0, used, torch.randn(shape, generator=gen, device=device, dtype=torch.bfloat16))
        kv.value_cache[layer].index_copy_(0, used,
                                          torch.randn(shape, generator=gen, device=device, dtype=torch.bfloat16))
    model = AttentionOnlyDecoder(wl.layers, b, wl.heads, wl.kv_heads, device, seed=11 + rank)
    return ctx, bm, md, kv, model, num_blocks


def kv_bytes_per_layer(ctx_after: list[int], kv_heads: int) -> int:
    return sum(ctx_after) * kv_heads * HEAD_DIM * 2 * 2


# ---------------------------------------------------------------- parity ----
def _gather_rows(cache_layer: torch.Tensor, table_row: torch.Tensor, n: int) -> torch.Tensor:
    """First n token rows [n, KVH, D] of one sequence, as fp32 on the host."""
    nblk = -(-n // BLOCK)
    rows = cache_layer.index_select(0, table_row[:nblk].to(torch.int64))
    return rows.reshape(nblk * BLOCK, *cache_layer.shape[2:])[:n].float().cpu()


def _attend_fp32(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float, causal_lq: int = 0):
    """q [Tq, H, D], k/v [Tk, KVH, D] fp32 -> [Tq, H, D]; bottom-right causal
    when causal_lq > 0 (query i sees key j <= Tk - Tq + i)."""
    tq, h, d = q.shape
    tk, kvh, _ = k.shape
    qg = q.view(tq, kvh, h // kvh, d)
    s = torch.einsum("tgqd,ngd->gqtn", qg, k) * scale
    if causal_lq:
        i = torch.arange(tq)[:, None]
        j = torch.arange(tk)[None, :]
        s = s.masked_fill(~(j <= (tk - tq) + i), float("-inf"))
    p = torch.softmax(s, dim=-1)
    return torch.einsum("gqtn,ngd->tgqd", p, v).reshape(tq, h, d)


def _compare(got: torch.Tensor, want: torch.Tensor) -> tuple[bool, float]:
    err = (got - want).abs()
    ok = bool((err <= ATOL + RTOL * want.abs()).all()) and not bool(torch.isnan(got).any())
    return ok, float(err.max()) if err.numel() else 0.0


def decode_parity(out: torch.Tensor, q: torch.Tensor, kc: torch.Tensor, vc: torch.Tensor, tables: torch.Tensor,
                  ctx_after: list[int], layer: int, sample: list[int]) -> dict:
    """A few sequences of one layer's decode output vs an fp32 torch-CPU
    gather + softmax of the same pool rows."""
    ok, worst = True, 0.0
    for b in sample:
        n = ctx_after[b]
        k = _gather_rows(kc, tables[b], n)
        v = _gather_rows(vc, tables[b], n)
        want = _attend_fp32(q[b:b + 1].float().cpu(), k, v, HEAD_DIM ** -0.5)[0]
        good, err = _compare(out[b].float().cpu(), want)
        ok, worst = ok and good, max(worst, err)
    return {"parity_ok": ok, "max_abs_err": worst, "layer": layer, "sequences_checked": len(sample),
            "tolerance": f"|err| <= {ATOL} + {RTOL}*|ref| vs fp32 torch-CPU gather+softmax"}


def spread(n: int, k: int = 4) -> list[int]:
    return sorted({round(i * (n - 1) / max(k - 1, 1)) for i in range(k)}) if n else []


# --------------------------------------------------------------- measure ----
def graph_time(fns, launches: int, device, reps: int = 3) -> float:
    """Average device time (s) of one call over `launches` calls captured in one
    CUDA graph; call i is fns[i % len(fns)] (fns are the same kernel on
    rotating input/output sets, so that L2 does not hold a launch's data from
    the previous one)."""
    fns = fns if isinstance(fns, (list, tuple)) else [fns]
    stream = torch.cuda.Stream(device)
    with torch.cuda.stream(stream):
        for fn in fns:
            fn()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for i in range(launches):
                fns[i % len(fns)]()
        for _ in range(2):
            graph.replay()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(reps):
            graph.replay()
        end.record(stream)
        end.synchronize()
    del graph
    return start.elapsed_time(end) / 1e3 / (reps * launches)


def time_decode_kernel(wl, md, kv, model, device, launches: int, seconds: float = 0.8) -> float:
    """Average duration (s) of one nvk_paged_decode launch, cycling layers so
    that every launch reads a different slice of HBM (each larger than L2
    for the configs timed here)."""
    from nano_vllm_ascend_b200 import ops

    b = model.q.shape[1]
    tables = md.block_tables.to(device)
    ctx = md.context_lens.to(device=device, dtype=torch.int32)
    ws = torch.zeros(ops.decode_workspace_bytes(b, wl.heads, wl.kv_heads, HEAD_DIM), dtype=torch.uint8,
                     device=device)
    out = torch.empty_like(model.q[0])
    scale = HEAD_DIM ** -0.5

    def launch(i):
        layer = i % wl.layers
        kc, vc = kv.get_physical_cache(layer)
        ops.paged_decode(out, model.q[layer], kc, vc, tables, ctx, scale, ws)

    # Captured in a CUDA graph (one launch per layer, cycling), so that the
    # host's per-call cost does not gate the queue; PDL still overlaps each
    # launch's prologue with its predecessor's tail inside the graph.
    for i in range(5):
        launch(i)
    torch.cuda.synchronize()
    cap = torch.cuda.Stream(device)
    with torch.cuda.stream(cap):
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=cap):
            for i in range(launches):
                launch(i)
        graph.replay()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        # first pass sizes the replay count so that it lasts about `seconds` (clock sampling)
        reps = 1
        for rep in range(2):
            start.record(cap)
            for _ in range(reps):
                graph.replay()
            end.record(cap)
            end.synchronize()
            per = start.elapsed_time(end) / 1e3 / (reps * launches)
            if rep == 0:
                reps = max(1, int(seconds / max(per * launches, 1e-7)))
    del graph
    if ops.decode_error_word(ws) != 0:
        raise RuntimeError(f"decode kernel error word {ops.decode_error_word(ws)}")
    return per


def time_appends(kv, bm, device, rows: int = 8192, launches: int = 56) -> dict:
    """Prefill-sized appends (rows tokens, K+V) into free pool slots, timed
    under a CUDA graph over four rotating source sets (4 x 33.5 MB of rows,
    more than L2, so every launch reads its rows from HBM), each set into its
    own layer and slots:
      contiguous -- a set's rows fill whole free blocks in order (a prefill's layout);
      scattered  -- a set's rows go to distinct random free slots across the pool."""
    from nano_vllm_ascend_b200 import ops

    sets, nblk = 4, -(-rows // BLOCK)
    free = torch.tensor(bm.free_block_ids, dtype=torch.int64)
    if free.numel() < sets * nblk:
        return {"skipped": f"needs {sets * nblk} free pool blocks, {free.numel()} free (small profiling pool)"}
    g = torch.Generator(device=device).manual_seed(3)
    gc_ = torch.Generator().manual_seed(4)
    src = [(torch.randn(rows, kv.num_kv_heads, HEAD_DIM, generator=g, device=device).to(torch.bfloat16),
            torch.randn(rows, kv.num_kv_heads, HEAD_DIM, generator=g, device=device).to(torch.bfloat16))
           for _ in range(sets)]
    offs = torch.arange(BLOCK, dtype=torch.int64)
    contiguous = [(free[r * nblk:(r + 1) * nblk, None] * BLOCK + offs).reshape(-1)[:rows].to(device)
                  for r in range(sets)]
    scattered = []
    for r in range(sets):
        pick = torch.randperm(free.numel() * BLOCK, generator=gc_)[:rows]
        scattered.append((free[pick // BLOCK] * BLOCK + pick % BLOCK).to(device))
    byts = rows * kv.num_kv_heads * HEAD_DIM * 2 * 2 * 2 + rows * 8
    peak, _ = peaks()
    out = {"rows": rows, "bytes": byts, "source_sets": sets}
    for name, slot_sets in (("contiguous", contiguous), ("scattered", scattered)):
        fns = [lambda r=r, sl=sl: ops.kv_append(kv.key_cache[r % kv.num_layers], kv.value_cache[r % kv.num_layers],
                                                src[r][0], src[r][1], sl) for r, sl in enumerate(slot_sets)]
        t = graph_time(fns, launches, device)
        out[name] = {"us": t * 1e6, "gbs": byts / t / 1e9, "frac": byts / t / 1e9 / peak}
    return out


def measure_decode(args, wl: Workload, world: int, rank: int, local: int, with_cpu: bool) -> dict:
    """One decode workload (config 2 or 4) on this rank: the JSON line's fields."""
    from nano_vllm_ascend_b200 import DecodeGraphRunner, check_errors

    device = torch.device("cuda", local)
    ctx, bm, md, kv, model, num_blocks = build(wl, world, rank, device, args.pool_blocks)
    b = len(ctx)
    ctx_after = [n + 1 for n in ctx]
    bytes_layer = kv_bytes_per_layer(ctx_after, wl.kv_heads)
    bytes_step = bytes_layer * wl.layers

    runner = DecodeGraphRunner(model, kv, batch_sizes=[b], max_model_len=wl.ctx_hi + 64, block_size=BLOCK,
                               device=device)
    input_ids = torch.zeros(b, dtype=torch.long, device=device)
    positions = torch.tensor(ctx, dtype=torch.long, device=device)
    if runner.forward(input_ids, positions, md) is None:
        raise RuntimeError("decode graph capture failed")
    slot = runner.slot(b)
    torch.cuda.synchronize()

    with ClockSampler(local) as clocks:
        # dominant kernel alone (roofline)
        t_dec = time_decode_kernel(wl, md, kv, model, device, launches=max(56, 4 * wl.layers),
                                   seconds=0.0 if args.quick else 0.8)
        appends = time_appends(kv, bm, device, launches=8 if args.quick else 56)
        # the step: W warm-up replays, then exactly K timed replays
        for _ in range(args.warmup):
            slot.graph.replay()
        barrier_sync(world)
        stream = torch.cuda.current_stream(device)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(args.steps):
            slot.graph.replay()
        end.record(stream)
        barrier_sync(world)
        t_step = start.elapsed_time(end) / 1e3 / args.steps

        # end to end through the public API: pinned host inputs -> device,
        # runner.forward (metadata refresh + replay), outputs -> host
        h_q = model.q.cpu().pin_memory()
        h_k = model.k.cpu().pin_memory()
        h_v = model.v.cpu().pin_memory()
        h_out = torch.empty(slot.logits.shape, dtype=slot.logits.dtype).pin_memory()
        h_tables = md.block_tables.cpu().pin_memory()
        h_slots = md.slot_mapping.cpu().pin_memory()
        h_ctx = md.context_lens.pin_memory()
        h_pos = positions.cpu().pin_memory()
        h_ids = input_ids.cpu().pin_memory()

        def e2e_step():
            model.q.copy_(h_q, non_blocking=True)
            model.k.copy_(h_k, non_blocking=True)
            model.v.copy_(h_v, non_blocking=True)
            step_md = type(md)(block_tables=h_tables.to(device, non_blocking=True), context_lens=h_ctx,
                               slot_mapping=h_slots.to(device, non_blocking=True))
            logits = runner.forward(h_ids.to(device, non_blocking=True), h_pos.to(device, non_blocking=True),
                                    step_md)
            h_out.copy_(logits, non_blocking=True)

        for _ in range(args.warmup):
            e2e_step()
        barrier_sync(world)
        e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e_start.record(stream)
        for _ in range(args.steps):
            e2e_step()
        e_end.record(stream)
        barrier_sync(world)
        t_e2e = e_start.elapsed_time(e_end) / 1e3 / args.steps
    clk = clocks.summary()
    check_errors(device)  # every device error word of the run is clear

    # parity of the step's own output: the last layer of the last replay
    layer = wl.layers - 1
    kc, vc = kv.get_physical_cache(layer)
    parity = decode_parity(slot.logits[layer], model.q[layer], kc, vc, md.block_tables.to(device), ctx_after, layer,
                           spread(b))
    parity["parity_ok"] = _reduce(1.0 if parity["parity_ok"] else 0.0, world, "min") > 0.5
    parity["max_abs_err"] = max_over_ranks(parity["max_abs_err"], world)

    h2d = sum(t.numel() * t.element_size() for t in (h_q, h_k, h_v, h_tables, h_slots, h_ctx, h_pos, h_ids))
    d2h = h_out.numel() * h_out.element_size()
    per_rank = all_ranks({"rank": rank, "ms_per_step": t_step * 1e3, "sm_mhz": clk.get("sm_mhz"),
                          "us_per_decode_launch": t_dec * 1e6, "reasons": clk.get("reasons")}, world)
    t_step_max = max_over_ranks(t_step, world)
    t_e2e_max = max_over_ranks(t_e2e, world)
    t_dec_max = max_over_ranks(t_dec, world)
    bytes_all = sum_over_ranks(float(bytes_step), world)
    seqs_all = sum_over_ranks(float(b), world)
    peak, peak_kind = peaks()
    dec_bytes_launch = bytes_layer + b * wl.heads * HEAD_DIM * 2 * 2 + md.block_tables.numel() * 4 + b * 4
    achieved = dec_bytes_launch / t_dec_max / 1e9
    traffic = profiled_traffic(wl.name) if world == 1 else None
    runner.release()
    line = {
        "metric": "paged decode-attn KV GB/s",
        "value": bytes_all / t_step_max / 1e9,
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": t_step_max * 1e3,
        "higher_is_better": True,
        "scaling": wl.scaling,
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic: seeded N(0,1) q/K/V, seeded context lengths and block tables (no weights)",
        "config": decode_config(wl, world),
        "setup": {"pool_blocks": num_blocks, "decode_grid": "persistent, one CTA per SM",
                  "append": "fused into the decode kernel" if runner.fuse_appends else "separate kernel"},
        "tok_per_s": seqs_all / t_step_max,
        "hbm_frac_of_step": (bytes_all / t_step_max / 1e9) / (peak * world),
        "parity": parity,
        "append": appends,
        "roofline": {"kernel": "paged_decode_kernel", "bound": "hbm", "achieved": achieved, "peak": peak,
                     "peak_kind": peak_kind, "unit": "GB/s", "frac": achieved / peak,
                     "frac_of_nominal_8tbs": achieved / 8000.0, "traffic": traffic,
                     "algorithmic_bytes_per_launch": dec_bytes_launch, "us_per_launch": t_dec_max * 1e6},
        "e2e": {"value": bytes_all / t_e2e_max / 1e9, "unit": "GB/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": t_e2e_max * 1e3},
        "clocks": clk,
        "gpu_launches": args.steps * wl.layers * (1 if runner.fuse_appends else 2),
        "cpu_baseline": None,
    }
    if world > 1:
        line["per_rank"] = per_rank
    if with_cpu and rank == 0:
        line["cpu_baseline"] = cpu_baseline_decode(wl, ctx, seconds=args.cpu_seconds, threads=os.cpu_count() or 1)
    return line


# ---------------------------------------------------------- model step ----
def _step_reference_logits(model, tokens: torch.Tensor) -> torch.Tensor:
    """fp32-attention torch recompute of one sequence through the step's model
    (same weights and dense ops): logits of its last position."""
    import torch.nn.functional as F

    from nano_vllm_ascend_b200.step_runner import _rms_norm

    s = model.shape
    ids = tokens.to(model.device)
    n = ids.numel()
    pos = torch.arange(n, device=model.device)
    c = model.cos[pos].to(torch.bfloat16).float()[:, None]
    sn = model.sin[pos].to(torch.bfloat16).float()[:, None]

    def norm_rope(x, w):
        xf = x.float()
        y = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + s.rms_norm_eps) * w.float()).to(torch.bfloat16)
        y = y.float()
        half = y.shape[-1] // 2
        return (y * c + torch.cat([-y[..., half:], y[..., :half]], dim=-1) * sn).to(torch.bfloat16)

    g = s.num_heads // s.num_kv_heads
    causal = torch.ones(n, n, dtype=torch.bool, device=model.device).tril()
    x = model.embed[ids]
    for layer in model.layers:
        h = _rms_norm(x, layer.in_norm, s.rms_norm_eps)
        qkv = F.linear(h, layer.qkv).view(n, -1, s.head_dim)
        q = norm_rope(qkv[:, :s.num_heads], layer.q_norm)
        k = norm_rope(qkv[:, s.num_heads:s.num_heads + s.num_kv_heads], layer.k_norm)
        v = qkv[:, s.num_heads + s.num_kv_heads:]
        sc = torch.einsum("tkgd,nkd->kgtn", q.float().view(n, s.num_kv_heads, g, -1), k.float()) * s.head_dim ** -0.5
        p = torch.softmax(sc.masked_fill(~causal, float("-inf")), dim=-1)
        x = x + F.linear(torch.einsum("kgtn,nkd->tkgd", p, v.float()).reshape(n, -1).to(torch.bfloat16), layer.o)
        h = _rms_norm(x, layer.post_norm, s.rms_norm_eps)
        gate, up = F.linear(h, layer.gate_up).chunk(2, dim=-1)
        x = x + F.linear(F.silu(gate) * up, layer.down)
    return _rms_norm(x, model.final_norm, s.rms_norm_eps)[-1].float() @ model.embed.float().T


def measure_step(args, world: int, rank: int, local: int) -> dict:
    """Config 2 through StepRunner (the reference's ModelRunner step drivers):
    a Qwen3-0.6B-shaped model with seeded random weights, 32 sequences per
    rank prefilled to context ~U[256, 2304] from random token ids (as the
    reference's bench_compare.py draws its prompts), then greedy decode steps
    at batch 32 from one CUDA graph: device-side metadata, the 28 layers
    (fused q/k norm + RoPE + append, paged decode, cuBLAS projections and
    MLP), LM head + argmax, and the next token ids read back every step."""
    from nano_vllm_ascend_b200.step_runner import ModelShape, StepRunner, StepSequence

    wl = WORKLOADS["decode_c2"]
    device = torch.device("cuda", local)
    ctx = rank_contexts(wl, world, rank)
    b = len(ctx)
    max_len = wl.ctx_hi + args.warmup + args.steps + 8
    runner = StepRunner(ModelShape(), device, max_model_len=max_len, max_num_seqs=b, decode_graph_batch_sizes=[b],
                        seed=100 + rank)
    g = torch.Generator().manual_seed(2000 + rank)
    seqs = [StepSequence(i, torch.randint(0, 10000, (n,), generator=g)) for i, n in enumerate(ctx)]
    runner.prepare_sequences(seqs)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    runner.prefill(seqs)  # reads the tokens back: synchronous
    t_prefill = time.perf_counter() - t0
    stream = torch.cuda.current_stream(device)
    with ClockSampler(local) as clocks:
        for _ in range(args.warmup):
            runner.decode(seqs)
        barrier_sync(world)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        w0 = time.perf_counter()
        start.record(stream)
        for _ in range(args.steps):
            runner.decode(seqs)
        end.record(stream)
        barrier_sync(world)
        wall = (time.perf_counter() - w0) / args.steps
        t_step = start.elapsed_time(end) / 1e3 / args.steps
    clk = clocks.summary()
    # parity: two sequences recomputed from scratch; each picked token must be
    # a greedy choice of the recompute's logits (bf16 may reorder near-ties)
    ok, worst = True, 0.0
    for seq in (seqs[0], seqs[-1]):
        logits = _step_reference_logits(runner.model, seq.token_ids())
        gap = float(logits.max() - logits[seq.next_token_id])
        ok, worst = ok and gap <= 5e-2, max(worst, gap)
    parity = {"parity_ok": _reduce(1.0 if ok else 0.0, world, "min") > 0.5,
              "max_logit_gap": max_over_ranks(worst, world), "sequences_checked": 2,
              "tolerance": "each sequence's last greedy token within 0.05 of the max logit of a torch recompute "
                           "(fp32 attention, same weights and dense ops) of its whole history"}
    stats = runner.decode_graph_stats()
    runner.release()
    t_step_max = max_over_ranks(t_step, world)
    seqs_all = sum_over_ranks(float(b), world)
    ctx_now = [c + args.warmup + args.steps for c in ctx]
    kv_step = kv_bytes_per_layer(ctx_now, wl.kv_heads) * wl.layers
    return {
        "metric": "decode tok/s (Qwen3-0.6B-shaped step, greedy, through StepRunner)",
        "value": seqs_all / t_step_max, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": t_step_max * 1e3, "scaling": "weak",
        "config": {"workload": "config[1] through the model step: Qwen3-0.6B shapes (28 layers, hidden 1024, "
                               "MLP 3072, vocab 151936, tied LM head), random weights, 32 seqs per GPU, "
                               "ctx~U[256,2304], CUDA graph bs 32",
                   "batch_per_gpu": b, "global_batch": int(seqs_all)},
        "parity": parity,
        "e2e": {"value": seqs_all / max_over_ranks(wall, world), "unit": "tok/s",
                "h2d_bytes_per_step": 2 * 8 * b, "d2h_bytes_per_step": 8 * b,
                "ms_per_step_wall": wall * 1e3, "note": "every step crosses token ids + positions in and the "
                                                        "next token ids out, and waits for them"},
        "kv_gbs_of_step": kv_bytes_per_layer(ctx_now, wl.kv_heads) * wl.layers / t_step_max / 1e9 * world,
        "prefill_tok_per_s": sum(ctx) / t_prefill,
        "graph_stats": stats,
        "clocks": clk,
        "vs_reference_published": {"value": 1296.05, "unit": "output tok/s",
                                   "what": "the reference on an Ascend 910B3, 32 x 256 in / 2048 out, whole run "
                                           "(bench_outputs/nano_32x256_2048.json)"},
    }


# ------------------------------------------------------------- kernels ----
def run_kernels(args, world, rank, local):
    """The hot path's kernels other than decode/prefill attention, one by one.
    Each timed kernel rotates over input/output sets whose sum exceeds the
    126 MB L2, so consecutive launches do not hit each other's lines."""
    from nano_vllm_ascend_b200 import BlockManager, ops
    from nano_vllm_ascend_b200.device_metadata import DeviceBlockTables

    device = torch.device("cuda", local)
    peak, peak_kind = peaks()
    g = torch.Generator(device=device).manual_seed(0)
    kvh, h, d, nb = 8, 16, 128, 2048
    rot = 4  # rotating sets
    kc = torch.zeros(rot * nb, BLOCK, kvh, d, dtype=torch.bfloat16, device=device)
    vc = torch.zeros_like(kc)
    out = {}
    n = 8 if args.quick else 24

    # prefill-sized append (config 3: 256 new tokens x 32 requests), 4 x 67 MB touched
    rows = 8192
    base = torch.randperm(nb * BLOCK, device=device)[:rows].sort().values
    sets = []
    for r in range(rot):
        k = torch.randn(rows, kvh, d, generator=g, device=device).to(torch.bfloat16)
        v = torch.randn(rows, kvh, d, generator=g, device=device).to(torch.bfloat16)
        sets.append((k, v, base + r * nb * BLOCK))
    t = graph_time([lambda k=k, v=v, sl=sl: ops.kv_append(kc, vc, k, v, sl) for k, v, sl in sets], n, device)
    byts = rows * kvh * d * 2 * 2 * 2 + rows * 8
    out["kv_append_8192"] = {"us": t * 1e6, "bytes": byts, "gbs": byts / t / 1e9, "frac": byts / t / 1e9 / peak}

    # q/k RMSNorm + RoPE + append, decode (32 tokens) and prefill (8192 tokens) sized
    inv = 1.0 / (1e6 ** (torch.arange(0, d, 2, dtype=torch.float32) / d))
    emb = torch.cat([torch.outer(torch.arange(40960, dtype=torch.float32), inv)] * 2, dim=-1)
    cos, sin = emb.cos().to(device), emb.sin().to(device)
    wq = torch.ones(d, dtype=torch.bfloat16, device=device)
    for tokens in (32, 8192):
        fns = []
        for r in range(rot):
            qkv = torch.randn(tokens, h + 2 * kvh, d, generator=g, device=device).to(torch.bfloat16)
            q_out = torch.empty(tokens, h, d, dtype=torch.bfloat16, device=device)
            pos = torch.randint(0, 40960, (tokens,), device=device)
            sl = base[:tokens] + r * nb * BLOCK
            fns.append(lambda qkv=qkv, q_out=q_out, pos=pos, sl=sl: ops.qk_norm_rope_append(
                qkv[:, :h], qkv[:, h:h + kvh], qkv[:, h + kvh:], wq, wq, 1e-6, cos, sin, pos, kc, vc, sl,
                query_out=q_out))
        t = graph_time(fns, n, device)
        byts = tokens * ((h + 2 * kvh) * d * 2 * 2 + 8 * 2)  # read q, k, v; write q, k, v; positions, slots
        out[f"qk_norm_rope_append_{tokens}"] = {"us": t * 1e6, "bytes": byts, "gbs": byts / t / 1e9,
                                                "frac": byts / t / 1e9 / peak}

    # device decode metadata for a 32-sequence step
    bm = BlockManager(nb, BLOCK, device)
    ctx = torch.randint(256, 2305, (32,), generator=torch.Generator().manual_seed(1000)).tolist()
    bm.prepare_prefill_metadata(list(range(32)), ctx, [0] * 32, [[] for _ in range(32)])
    dt = DeviceBlockTables(bm, 64, 64, device)
    dt.prepare_decode_metadata(list(range(32)), ctx, 1)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(50):
        dt.prepare_decode_metadata(list(range(32)), [c + 1 + i for c in ctx], 1)
    torch.cuda.synchronize()
    t_dev = (time.perf_counter() - t0) / 50
    bm2 = BlockManager(nb, BLOCK, device)
    bm2.prepare_prefill_metadata(list(range(32)), ctx, [0] * 32, [[] for _ in range(32)])
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(50):
        bm2.prepare_decode_metadata(list(range(32)), [c + 1 + i for c in ctx], 1)
    torch.cuda.synchronize()
    t_host = (time.perf_counter() - t0) / 50
    out["decode_metadata_32"] = {"host_us_device_path": t_dev * 1e6, "host_us_reference_path": t_host * 1e6}

    # LM head + greedy argmax, 32 rows over the Qwen3-0.6B vocabulary
    vocab, hid = 151936, 1024
    weight = (torch.randn(vocab, hid, generator=g, device=device) * 0.05).to(torch.bfloat16)
    hidden = torch.randn(32, hid, generator=g, device=device).to(torch.bfloat16)
    ws = torch.zeros(ops.lm_head_argmax_workspace_bytes(32), dtype=torch.uint8, device=device)
    ids = torch.empty(32, dtype=torch.int64, device=device)
    t = graph_time(lambda: ops.lm_head_argmax(hidden, weight, ws, ids), n, device)  # 311 MB weight > L2
    byts = vocab * hid * 2
    out["lm_head_argmax_32"] = {"us": t * 1e6, "bytes": byts, "gbs": byts / t / 1e9, "frac": byts / t / 1e9 / peak}
    if rank == 0:
        print(json.dumps({"metric": "kernel GB/s (graph-timed)", "value": out["kv_append_8192"]["gbs"], "unit": "GB/s",
                          "n_gpus": world, "higher_is_better": True, "dtype": "bf16", "data": "synthetic",
                          "config": {"workload": WORKLOADS["kernels"].describe}, "peak": peak, "peak_kind": peak_kind,
                          "kernels": out}), flush=True)
    return 0


# ------------------------------------------------------------ config 5 ----
def measure_c5(args, world: int, rank: int, local: int, gather: str) -> dict:
    """KV-head-sharded decode step (config 5) with the outputs all-gathered."""
    from nano_vllm_ascend_b200 import BlockManager, PagedKVCache, ops
    from nano_vllm_ascend_b200.peer_gather import PeerGather
    from nano_vllm_ascend_b200.sharding import gather_head_shards, kv_head_shard

    wl = WORKLOADS["decode_c5"]
    device = torch.device("cuda", local)
    kv_r, q_r = kv_head_shard(wl.heads, wl.kv_heads, world, rank)
    kvh, hl, hoff = len(kv_r), len(q_r), q_r.start
    b, layers = wl.batch, wl.layers
    ctx = [wl.ctx_lo] * b
    need = sum((n + 1 + BLOCK - 1) // BLOCK for n in ctx)
    num_blocks = need + 64
    pool_bytes = 2 * layers * num_blocks * BLOCK * kvh * HEAD_DIM * 2
    free, _ = torch.cuda.mem_get_info(device)
    if pool_bytes > wl.util * free:
        raise SystemExit(f"decode_c5: {pool_bytes / 1e9:.1f} GB of KV per GPU at N={world} exceeds "
                         f"{wl.util:.0%} of free HBM ({free / 1e9:.1f} GB); run it on 2, 4 or 8 GPUs")
    bm = BlockManager(num_blocks, BLOCK, device)
    bm.free_block_ids = torch.randperm(num_blocks, generator=torch.Generator().manual_seed(42)).tolist()
    slots = list(range(b))
    bm.prepare_prefill_metadata(slots, ctx, [0] * b, [[] for _ in slots])
    md = bm.prepare_decode_metadata(slots, ctx, q_len=1)
    kv = PagedKVCache(layers, num_blocks, BLOCK, kvh, HEAD_DIM, torch.bfloat16, device)
    gen = torch.Generator(device=device).manual_seed(5 + rank)
    for cache in (kv.key_cache, kv.value_cache):  # layer 0 random, the others copies (same bytes to stream)
        cache[0].normal_(generator=gen)
        for layer in range(1, layers):
            cache[layer].copy_(cache[0])
    g = torch.Generator(device=device).manual_seed(11 + rank)
    q = torch.randn(layers, b, hl, HEAD_DIM, generator=g, device=device).to(torch.bfloat16)
    k_new = torch.randn(layers, b, kvh, HEAD_DIM, generator=g, device=device).to(torch.bfloat16)
    v_new = torch.randn(layers, b, kvh, HEAD_DIM, generator=g, device=device).to(torch.bfloat16)
    tables = md.block_tables.to(device)
    ctx_d = md.context_lens.to(device=device, dtype=torch.int32)
    slot_map = md.slot_mapping.to(device)
    scale = HEAD_DIM ** -0.5
    ws = torch.zeros(ops.decode_workspace_bytes(b, hl, kvh, HEAD_DIM), dtype=torch.uint8, device=device)
    in_kernel = gather == "kernel"
    pg = PeerGather(b, wl.heads, HEAD_DIM, slots=layers, device=device) if in_kernel else None
    local_out = torch.empty(layers, b, hl, HEAD_DIM, dtype=torch.bfloat16, device=device)
    gathered = torch.empty(layers, b, wl.heads, HEAD_DIM, dtype=torch.bfloat16, device=device)

    def attend(layer, gather=True, append=False):
        kc, vc = kv.get_physical_cache(layer)
        new = dict(new_key=k_new[layer], new_value=v_new[layer], slot_mapping=slot_map) if append else {}
        if in_kernel:
            return pg.decode(q[layer], kc, vc, tables, ctx_d, scale, ws, head_offset=hoff, slot=layer, **new)
        ops.paged_decode(local_out[layer], q[layer], kc, vc, tables, ctx_d, scale, ws, **new)
        if gather and world > 1:
            return gather_head_shards(local_out[layer], out=gathered[layer])
        return local_out[layer]

    def step():
        # per layer: this step's append fused into the attention kernel, then
        # (baseline) the NCCL gather
        out = None
        for layer in range(layers):
            out = attend(layer, append=True)
        return out

    stream = torch.cuda.Stream(device)
    with torch.cuda.stream(stream):
        step()  # eager warm-up (NCCL communicator, workspace); every rank makes the same calls
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            last_out = step()
    torch.cuda.synchronize()

    with torch.cuda.stream(stream), ClockSampler(local) as clocks:
        # decode kernel alone (roofline; with the in-kernel gather the kernel
        # includes its gather), cycling layers: every rank runs the same launches
        for i in range(layers):
            attend(i, gather=False)
        barrier_sync(world)
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n_launch = layers * (1 if args.quick else 4)
        timing0 = ws[128:152].view(torch.int64).cpu() if in_kernel else None
        ev0.record(stream)
        for i in range(n_launch):
            attend(i % layers, gather=False)
        ev1.record(stream)
        ev1.synchronize()
        t_dec = ev0.elapsed_time(ev1) / 1e3 / n_launch
        gather_split = None
        if in_kernel:  # the kernel's own clock: local work, then the wait for every rank's epoch
            d = ws[128:152].view(torch.int64).cpu() - timing0
            calls = max(int(d[2]), 1)
            gather_split = {"local_us": float(d[0]) / calls / 1e3, "epoch_wait_us": float(d[1]) / calls / 1e3}
        if ops.decode_error_word(ws) != 0:
            raise RuntimeError(f"decode error word {ops.decode_error_word(ws)}")
        for _ in range(args.warmup):
            graph.replay()
        barrier_sync(world)
        ev0.record(stream)
        for _ in range(args.steps):
            graph.replay()
        ev1.record(stream)
        barrier_sync(world)
        t_step = ev0.elapsed_time(ev1) / 1e3 / args.steps

        # end to end: pinned host inputs -> device, replay, last layer's gathered output -> host
        h_q, h_k, h_v = (t.cpu().pin_memory() for t in (q, k_new, v_new))
        h_tables, h_slots, h_ctx = (t.cpu().pin_memory() for t in (tables, slot_map, ctx_d))
        h_out = torch.empty(last_out.shape, dtype=last_out.dtype).pin_memory()

        def e2e_step():
            q.copy_(h_q, non_blocking=True)
            k_new.copy_(h_k, non_blocking=True)
            v_new.copy_(h_v, non_blocking=True)
            tables.copy_(h_tables, non_blocking=True)
            slot_map.copy_(h_slots, non_blocking=True)
            ctx_d.copy_(h_ctx, non_blocking=True)
            graph.replay()
            h_out.copy_(last_out, non_blocking=True)

        for _ in range(args.warmup):
            e2e_step()
        barrier_sync(world)
        ev0.record(stream)
        for _ in range(args.steps):
            e2e_step()
        ev1.record(stream)
        barrier_sync(world)
        t_e2e = ev0.elapsed_time(ev1) / 1e3 / args.steps

        # parity: layer 0 gathered once more (the pool already holds this
        # step's rows); every rank checks all heads of a few sequences
        out0 = attend(0).clone()
        barrier_sync(world)
    clk = clocks.summary()
    if ops.decode_error_word(ws) != 0:
        raise RuntimeError(f"decode error word {ops.decode_error_word(ws)}")
    sample = spread(b)
    kc0, vc0 = kv.get_physical_cache(0)
    mine = []
    for s in sample:
        k = _gather_rows(kc0, tables[s], ctx[s] + 1)
        v = _gather_rows(vc0, tables[s], ctx[s] + 1)
        mine.append(_attend_fp32(q[0, s:s + 1].float().cpu(), k, v, scale)[0])
    refs = all_ranks((hoff, torch.stack(mine)), world)
    want = torch.zeros(len(sample), wl.heads, HEAD_DIM)
    for off, rows in refs:
        want[:, off:off + rows.shape[1]] = rows
    ok, err = _compare(out0[sample].float().cpu(), want)  # [sample, all heads] on every rank
    parity = {"parity_ok": _reduce(1.0 if ok else 0.0, world, "min") > 0.5,
              "max_abs_err": max_over_ranks(err, world), "layer": 0, "sequences_checked": len(sample),
              "heads_checked_per_rank": wl.heads,
              "tolerance": f"|err| <= {ATOL} + {RTOL}*|ref| vs fp32 torch-CPU gather+softmax, all ranks"}

    bytes_layer = kv_bytes_per_layer([n + 1 for n in ctx], kvh)
    per_rank = all_ranks({"rank": rank, "ms_per_step": t_step * 1e3, "sm_mhz": clk.get("sm_mhz"),
                          "us_per_decode_launch": t_dec * 1e6, "reasons": clk.get("reasons"),
                          **({"gather": gather_split} if gather_split else {})}, world)
    t_step_max = max_over_ranks(t_step, world)
    t_e2e_max = max_over_ranks(t_e2e, world)
    t_dec_max = max_over_ranks(t_dec, world)
    bytes_all = sum_over_ranks(float(bytes_layer * layers), world)
    peak, peak_kind = peaks()
    dec_bytes = bytes_layer + b * hl * HEAD_DIM * 2 * 2 + tables.numel() * 4 + b * 4
    nvlink_bytes = b * hl * HEAD_DIM * 2 * (world - 1)
    h2d = sum(t.numel() * t.element_size() for t in (h_q, h_k, h_v, h_tables, h_slots, h_ctx))
    d2h = h_out.numel() * h_out.element_size()
    line = {
        "metric": "paged decode-attn KV GB/s", "value": bytes_all / t_step_max / 1e9, "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": t_step_max * 1e3,
        "higher_is_better": True, "scaling": wl.scaling, "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded N(0,1) q/K/V (pool layer 0 random, copied to the other layers), "
                "seeded block tables",
        "config": {"workload": wl.describe, "layers": layers, "global_batch": b, "seq_len": wl.ctx_lo + 1,
                   "heads": [wl.heads, wl.kv_heads, HEAD_DIM], "heads_per_gpu": [hl, kvh],
                   "block_size": BLOCK, "parallelism": f"KV-head sharded x{world}",
                   "gather": "in-kernel peer stores over NVLink + epoch flags" if in_kernel
                   else "NCCL all_gather_into_tensor + permute",
                   "append": "fused into the decode kernel",
                   "cache": "inputs larger than L2: every step reads %.1f GB of KV per GPU"
                            % (bytes_layer * layers / 1e9)},
        "setup": {"pool_blocks": num_blocks},
        "tok_per_s": b / t_step_max,
        "hbm_frac_of_step": (bytes_all / t_step_max / 1e9) / (peak * world),
        "parity": parity,
        "comm": {"kind": "in-kernel all-gather (plain peer stores, no multicast)" if in_kernel else "NCCL all-gather",
                 "nvlink_bytes_per_launch": nvlink_bytes, "ranks": world},
        "roofline": {"kernel": "paged_decode_kernel (gather)" if in_kernel else "paged_decode_kernel",
                     "bound": "hbm", "achieved": dec_bytes / t_dec_max / 1e9, "peak": peak,
                     "peak_kind": peak_kind, "unit": "GB/s", "frac": dec_bytes / t_dec_max / 1e9 / peak,
                     "traffic": None, "algorithmic_bytes_per_launch": dec_bytes,
                     "nvlink_bytes_per_launch": nvlink_bytes if in_kernel else 0,
                     "us_per_launch": t_dec_max * 1e6},
        "e2e": {"value": bytes_all / t_e2e_max / 1e9, "unit": "GB/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": t_e2e_max * 1e3},
        "clocks": clk,
        "per_rank": per_rank,
        "gpu_launches": args.steps * layers,
        "cpu_baseline": None,
    }
    del graph
    if pg is not None:
        pg.close()
    return line


# ---------------------------------------------------------------- prefill ----
def prefill_flops(q_lens: list[int], kv_lens: list[int], heads: int) -> float:
    """4 * D * (visible (query, key) pairs), bottom-right causal."""
    pairs = 0
    for lq, lk in zip(q_lens, kv_lens):
        pairs += lq * (lk - lq) + lq * (lq + 1) // 2
    return 4.0 * HEAD_DIM * heads * pairs


def build_prefill(wl: Workload, device, pool_blocks: int = 0):
    """The config-3 state: a 768-token prefix cached by an earlier request
    (6 full blocks, hashed by cache_full_blocks), then 32 requests that hit it
    and prefill only their 256 new tokens."""
    from nano_vllm_ascend_b200 import BatchPrefillAttention, BlockManager, PagedKVCache
    from nano_vllm_ascend_b200.pool import num_blocks_from_memory

    prefix_len, new_len, b = wl.ctx_lo, wl.ctx_hi, wl.batch
    num_blocks = num_blocks_from_memory(wl.util, wl.layers, BLOCK, wl.kv_heads, HEAD_DIM, torch.bfloat16, device)
    if pool_blocks > 0:
        num_blocks = min(num_blocks, pool_blocks)
    bm = BlockManager(num_blocks, BLOCK, device)
    g = torch.Generator().manual_seed(42)
    bm.free_block_ids = torch.randperm(num_blocks, generator=g).tolist()
    prefix = torch.randint(0, 10000, (prefix_len,), generator=g)
    seed_prompt = torch.cat([prefix, torch.randint(0, 10000, (1,), generator=g)])
    bm.prepare_prefill_metadata([0], [prefix_len + 1], [0], [[]])
    bm.cache_full_blocks(slot=0, token_ids=seed_prompt, num_cached_blocks=0, num_full_blocks=prefix_len // BLOCK)
    kv = PagedKVCache(wl.layers, num_blocks, BLOCK, wl.kv_heads, HEAD_DIM, torch.bfloat16, device)
    gen = torch.Generator(device=device).manual_seed(5)
    used = torch.tensor(bm.block_tables[0], dtype=torch.int64, device=device)
    for layer in range(wl.layers):
        shape = (used.numel(), BLOCK, wl.kv_heads, HEAD_DIM)
        kv.key_cache[layer].index_copy_(0, used, torch.randn(shape, generator=gen, device=device, dtype=torch.bfloat16))
        kv.value_cache[layer].index_copy_(0, used,
                                          torch.randn(shape, generator=gen, device=device, dtype=torch.bfloat16))
    slots, hits, prompts = [], [], []
    for r in range(b):
        prompt = torch.cat([prefix, torch.randint(0, 10000, (new_len,), generator=g)])
        hit = bm.find_longest_prefix_blocks(prompt, max_cache_blocks=(prefix_len + new_len) // BLOCK - 1)
        assert len(hit) * BLOCK == prefix_len, "prefix must be hash-hit"
        slots.append(r + 1)
        hits.append(hit)
        prompts.append(prompt)
    md = bm.prepare_prefill_metadata(slots, [new_len] * b, [prefix_len] * b, hits)
    assert md.use_paged_prefill
    t = new_len * b
    q = torch.randn(wl.layers, t, wl.heads, HEAD_DIM, generator=gen, device=device).to(torch.bfloat16)
    k = torch.randn(wl.layers, t, wl.kv_heads, HEAD_DIM, generator=gen, device=device).to(torch.bfloat16)
    v = torch.randn(wl.layers, t, wl.kv_heads, HEAD_DIM, generator=gen, device=device).to(torch.bfloat16)
    attn = BatchPrefillAttention(wl.heads, wl.kv_heads, HEAD_DIM, BLOCK, max_mask_len=4096)
    return bm, md, kv, attn, q, k, v, num_blocks


def measure_prefill(args, world: int, rank: int, local: int, cpu_seconds: float) -> dict:
    from nano_vllm_ascend_b200 import check_errors, ops

    wl = WORKLOADS["prefill_c3"]
    device = torch.device("cuda", local)
    bm, md, kv, attn, q, k, v, num_blocks = build_prefill(wl, device, args.pool_blocks)
    b = wl.batch
    q_lens, kv_lens = [wl.ctx_hi] * b, [wl.ctx_lo + wl.ctx_hi] * b
    flops_layer = prefill_flops(q_lens, kv_lens, wl.heads)
    stream = torch.cuda.current_stream(device)

    def step():
        for layer in range(wl.layers):
            kv.write(layer, k[layer], v[layer], md.slot_mapping)
            kc, vc = kv.get_physical_cache(layer)
            attn(q[layer], k[layer], v[layer], md, kc, vc)

    step()
    torch.cuda.synchronize()
    # dominant kernel alone: prefill attention, cycling layers
    cu = torch.tensor([0] + list(range(wl.ctx_hi, wl.ctx_hi * b + 1, wl.ctx_hi)), dtype=torch.int32, device=device)
    kvl = torch.tensor(kv_lens, dtype=torch.int32, device=device)
    tables = md.block_tables.to(device)
    out = torch.empty_like(q[0])

    def pf(i):
        layer = i % wl.layers
        kc, vc = kv.get_physical_cache(layer)
        ops.paged_prefill(out, q[layer], kc, vc, tables, cu, kvl, wl.ctx_hi, HEAD_DIM ** -0.5)

    with ClockSampler(local) as clocks:
        for i in range(3):
            pf(i)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        launches = 56
        for rep in range(2):
            start.record(stream)
            for i in range(launches):
                pf(i)
            end.record(stream)
            end.synchronize()
            t_pf = start.elapsed_time(end) / 1e3 / launches
            if rep == 0 and not args.quick:
                launches = max(launches, int(0.8 / t_pf))
        for _ in range(args.warmup):
            step()
        barrier_sync(world)
        start.record(stream)
        for _ in range(args.steps):
            step()
        end.record(stream)
        barrier_sync(world)
        t_step = start.elapsed_time(end) / 1e3 / args.steps
        # e2e: pinned host q/k/v in, attention outputs back
        h_q, h_k, h_v = q.cpu().pin_memory(), k.cpu().pin_memory(), v.cpu().pin_memory()
        h_out = torch.empty(q.shape, dtype=q.dtype).pin_memory()

        def e2e_step():
            q.copy_(h_q, non_blocking=True)
            k.copy_(h_k, non_blocking=True)
            v.copy_(h_v, non_blocking=True)
            for layer in range(wl.layers):
                kv.write(layer, k[layer], v[layer], md.slot_mapping)
                kc, vc = kv.get_physical_cache(layer)
                h_out[layer].copy_(attn(q[layer], k[layer], v[layer], md, kc, vc), non_blocking=True)

        for _ in range(args.warmup):
            e2e_step()
        barrier_sync(world)
        start.record(stream)
        for _ in range(args.steps):
            e2e_step()
        end.record(stream)
        barrier_sync(world)
        t_e2e = start.elapsed_time(end) / 1e3 / args.steps
    clk = clocks.summary()
    check_errors(device)

    # parity: two requests of the last layer's output (h_out of the last e2e
    # step) vs fp32 over their 1024 paged keys (6 shared + 2 own blocks)
    layer, ok, worst = wl.layers - 1, True, 0.0
    kc, vc = kv.get_physical_cache(layer)
    for r in spread(b, 2):
        n = kv_lens[r]
        kr = _gather_rows(kc, tables[r], n)
        vr = _gather_rows(vc, tables[r], n)
        rows = slice(r * wl.ctx_hi, (r + 1) * wl.ctx_hi)
        want = _attend_fp32(q[layer, rows].float().cpu(), kr, vr, HEAD_DIM ** -0.5, causal_lq=wl.ctx_hi)
        good, err = _compare(h_out[layer, rows].float(), want)
        ok, worst = ok and good, max(worst, err)
    parity = {"parity_ok": ok, "max_abs_err": worst, "layer": layer, "requests_checked": 2,
              "tolerance": f"|err| <= {ATOL} + {RTOL}*|ref| vs fp32 torch-CPU paged gather + causal softmax"}

    t_step_max = max_over_ranks(t_step, world)
    t_e2e_max = max_over_ranks(t_e2e, world)
    flops_all = sum_over_ranks(flops_layer * wl.layers, world)
    peak, kind = peaks("bf16_tflops")
    achieved = flops_layer / t_pf / 1e12
    h2d = sum(t.numel() * t.element_size() for t in (h_q, h_k, h_v))
    line = {
        "metric": "prefix prefill attention TFLOP/s", "value": flops_all / t_step_max / 1e12, "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": t_step_max * 1e3,
        "higher_is_better": True, "scaling": wl.scaling, "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded prompts sharing a 768-token prefix (hash-hit), seeded N(0,1) q/K/V",
        "config": prefill_config(wl, world),
        "setup": {"pool_blocks": num_blocks},
        "tok_per_s": b * wl.ctx_hi * world / t_step_max,
        "parity": parity,
        "roofline": {"kernel": "prefill_kernel", "bound": "tensor", "achieved": achieved, "peak": peak,
                     "peak_kind": kind + " (burst, kernel timed alone)", "unit": "TFLOP/s",
                     "frac": achieved / peak, "traffic": profiled_traffic(wl.name, "paged_prefill"),
                     "tensor_pipe_active_pct_ncu": profiled_value(wl.name, "paged_prefill",
                                                                  "tensor_pipe_active_pct"),
                     "algorithmic_flops_per_launch": flops_layer,
                     "us_per_launch": t_pf * 1e6},
        "e2e": {"value": flops_all / t_e2e_max / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": h_out.numel() * h_out.element_size(), "ms_per_step": t_e2e_max * 1e3},
        "clocks": clk, "gpu_launches": args.steps * wl.layers * 2, "cpu_baseline": None,
    }
    if world == 1 and rank == 0 and cpu_seconds > 0:
        line["cpu_baseline"] = cpu_baseline_prefill(wl, cpu_seconds, os.cpu_count() or 1)
    return line


def prefill_config(wl: Workload, world: int) -> dict:
    return {"workload": wl.describe, "layers": wl.layers, "global_batch": wl.batch * world,
            "seq_len": wl.ctx_lo + wl.ctx_hi, "new_tokens": wl.ctx_hi, "cached_prefix": wl.ctx_lo,
            "heads": [wl.heads, wl.kv_heads, HEAD_DIM], "block_size": BLOCK,
            "parallelism": f"request-sharded x{world}, no collective",
            "cache": "per step 28 x (8192-row append + 60.16 GFLOP attention)"}


# ------------------------------------------------------------- CPU legs ----
class CpuBaseline:
    """Eager torch-CPU reference path (oracle/cpu_baseline.py) on one layer's
    worth of this workload: the sequences' blocks in a host pool, this step's
    append (index_copy_) and decode attention (gather + fp32 softmax). Every
    layer of a step is identical work, so a step runs layer() once per layer
    on the same host pool."""

    def __init__(self, wl: Workload, ctx: list[int], threads: int):
        torch.set_num_threads(threads)
        self.wl, self.ctx, self.threads = wl, ctx, threads
        b = len(ctx)
        g = torch.Generator().manual_seed(0)
        nblk = [(n + 1 + BLOCK - 1) // BLOCK for n in ctx]
        nb = sum(nblk)
        self.kc = torch.randn(nb, BLOCK, wl.kv_heads, HEAD_DIM, generator=g).to(torch.bfloat16)
        self.vc = torch.randn(nb, BLOCK, wl.kv_heads, HEAD_DIM, generator=g).to(torch.bfloat16)
        perm = torch.randperm(nb, generator=g).to(torch.int32)
        self.tables = torch.zeros(b, max(nblk), dtype=torch.int32)
        self.slots = torch.zeros(b, dtype=torch.int64)
        used = 0
        for i, m in enumerate(nblk):
            self.tables[i, :m] = perm[used : used + m]
            used += m
            self.slots[i] = int(self.tables[i, ctx[i] // BLOCK]) * BLOCK + ctx[i] % BLOCK
        self.q = torch.randn(b, wl.heads, HEAD_DIM, generator=g).to(torch.bfloat16)
        self.k = torch.randn(b, wl.kv_heads, HEAD_DIM, generator=g).to(torch.bfloat16)
        self.v = torch.randn(b, wl.kv_heads, HEAD_DIM, generator=g).to(torch.bfloat16)
        self.ctx_after = torch.tensor([n + 1 for n in ctx], dtype=torch.int32)
        self.bytes_layer = kv_bytes_per_layer([n + 1 for n in ctx], wl.kv_heads)

    def layer(self) -> None:
        from oracle import cpu_baseline

        cpu_baseline.append(self.kc, self.vc, self.k, self.v, self.slots)
        cpu_baseline.decode(self.q, self.kc, self.vc, self.tables, self.ctx_after, HEAD_DIM ** -0.5)

    def step(self) -> None:
        for _ in range(self.wl.layers):
            self.layer()

    def time_layers(self, seconds: float, min_layers: int = 1) -> tuple[float, int]:
        """Runs layer() until ``seconds`` elapsed (at least min_layers); returns (s per layer, layers)."""
        n = 0
        t0 = time.perf_counter()
        while True:
            self.layer()
            n += 1
            el = time.perf_counter() - t0
            if n >= min_layers and el >= seconds:
                return el / n, n


def cpu_baseline_decode(wl: Workload, ctx: list[int], seconds: float, threads: int) -> dict:
    base = CpuBaseline(wl, ctx, threads)
    base.layer()  # warm-up
    per_layer, n = base.time_layers(seconds)
    gbs = base.bytes_layer / per_layer / 1e9
    return {"value": gbs, "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{n} layer-steps (append + decode attention) of {len(ctx)} seqs on one layer's pool, "
                      f"{n * per_layer:.1f}s", "ms_per_layer": per_layer * 1e3,
            "tok_per_s": len(ctx) / (per_layer * wl.layers)}


def cpu_baseline_prefill(wl: Workload, seconds: float, threads: int, min_layers: int = 1) -> dict:
    """Eager torch-CPU path for one config-3 layer (append + prefill over the
    paged pool), repeated until ``seconds``; TFLOP/s of the attention."""
    from oracle import cpu_baseline

    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    b, lq, lk = wl.batch, wl.ctx_hi, wl.ctx_lo + wl.ctx_hi
    nblk = lk // BLOCK
    nb = 6 + b * (nblk - 6)
    kc = torch.randn(nb, BLOCK, wl.kv_heads, HEAD_DIM, generator=g).to(torch.bfloat16)
    vc = torch.randn(nb, BLOCK, wl.kv_heads, HEAD_DIM, generator=g).to(torch.bfloat16)
    tables = torch.zeros(b, nblk, dtype=torch.int32)
    tables[:, :6] = torch.arange(6, dtype=torch.int32)
    tables[:, 6:] = (6 + torch.arange(b * (nblk - 6), dtype=torch.int32)).view(b, nblk - 6)
    slots = torch.cat([torch.arange(int(t) * BLOCK, int(t) * BLOCK + BLOCK) for t in tables[:, 6:].flatten()])
    q = torch.randn(b * lq, wl.heads, HEAD_DIM, generator=g).to(torch.bfloat16)
    k = torch.randn(b * lq, wl.kv_heads, HEAD_DIM, generator=g).to(torch.bfloat16)
    v = torch.randn(b * lq, wl.kv_heads, HEAD_DIM, generator=g).to(torch.bfloat16)
    cu = list(range(0, b * lq + 1, lq))
    flops = prefill_flops([lq] * b, [lk] * b, wl.heads)
    n = 0
    t0 = time.perf_counter()
    while True:
        cpu_baseline.append(kc, vc, k, v, slots)
        cpu_baseline.prefill(q, kc, vc, tables, cu, [lk] * b, HEAD_DIM ** -0.5)
        n += 1
        el = time.perf_counter() - t0
        if n >= min_layers and el >= seconds:
            break
    return {"value": flops * n / el / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"{n} layer-steps (8192-row append + prefill attention of 32 x 256 queries over 1024 keys), "
                      f"{el:.1f}s", "ms_per_layer": el / n * 1e3}


def run_reference(args, world, rank) -> int:
    """The reference's path as eager torch-CPU code on the host cores (rank 0
    only): whole steps of the workload, every layer on the same one-layer
    host pool, `warmup` untimed steps then `steps` timed ones."""
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    name = args.workload or "decode_c2"
    wl = WORKLOADS[name]
    if name.startswith("prefill"):
        cpu_baseline_prefill(wl, 0.0, threads, min_layers=max(1, args.warmup))
        r = cpu_baseline_prefill(wl, 0.0, threads, min_layers=args.steps)
        line = {"impl": "reference", "metric": "prefix prefill attention TFLOP/s", "value": r["value"],
                "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": r["ms_per_layer"], "higher_is_better": True, "scaling": wl.scaling,
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": prefill_config(wl, world),
                "cpu_baseline": r,
                "e2e": {"value": r["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        line["cpu_baseline"]["sample"] += "; a step here is one layer"
        print(json.dumps(line), flush=True)
        return 0
    if name not in ("decode_c2", "decode_c4"):
        print(json.dumps({"impl": "reference", "unavailable": f"no CPU reference leg for workload {name}"}))
        return 0
    ctx = rank_contexts(wl, world, 0)
    base = CpuBaseline(wl, ctx, threads)
    for _ in range(args.warmup):
        base.step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        base.step()
    per_step = (time.perf_counter() - t0) / args.steps
    gbs = base.bytes_layer * wl.layers / per_step / 1e9
    line = {
        "impl": "reference", "metric": "paged decode-attn KV GB/s", "value": gbs, "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": per_step * 1e3,
        "higher_is_better": True, "scaling": wl.scaling, "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded N(0,1) q/K/V, seeded context lengths and block tables (no weights)",
        "config": decode_config(wl, world),
        "tok_per_s": len(ctx) / per_step,
        "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"{args.steps} whole steps ({wl.layers} x append + decode attention of rank 0's "
                                   f"{len(ctx)} sequences, each layer on the same one-layer host pool)"},
        "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ main ----
def summarize(line: dict) -> dict:
    """The fields of a workload's line kept in the headline's sub_results."""
    keep = ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "scaling", "tok_per_s",
            "hbm_frac_of_step", "parity", "roofline", "append", "comm", "e2e", "clocks", "per_rank", "config",
            "gpu_launches", "cpu_baseline")
    return {k: line[k] for k in keep if k in line}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS) + ["step_c2"], default=None,
                    help="one workload alone (default: decode_c2 headline with the other configs as sub_results)")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--pool-blocks", type=int, default=0,
                    help="cap the KV pool at this many blocks (small-footprint profiling runs)")
    ap.add_argument("--quick", action="store_true", help="short roofline loops (profiling runs)")
    ap.add_argument("--gather", choices=["kernel", "nccl"], default="kernel",
                    help="decode_c5: all-gather of the head shards inside the attention kernel or by NCCL")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    sys.path.insert(0, str(ROOT))
    world, rank, local = dist_setup(args)
    if args.impl == "reference":
        return run_reference(args, world, rank)
    cpu = world == 1 and not args.no_cpu_baseline
    try:
        if args.workload == "kernels":
            return run_kernels(args, world, rank, local)
        if args.workload == "decode_c5":
            line = measure_c5(args, world, rank, local, args.gather)
        elif args.workload == "step_c2":
            line = measure_step(args, world, rank, local)
        elif args.workload == "prefill_c3":
            line = measure_prefill(args, world, rank, local, args.cpu_seconds if cpu else 0.0)
        elif args.workload is not None:
            line = measure_decode(args, WORKLOADS[args.workload], world, rank, local, with_cpu=cpu)
        else:
            line = measure_decode(args, WORKLOADS["decode_c2"], world, rank, local, with_cpu=cpu)
            subs = {}
            free_device_memory()
            if world == 1:
                subs["prefill_c3"] = summarize(measure_prefill(args, world, rank, local,
                                                               min(args.cpu_seconds, 4.0) if cpu else 0.0))
                free_device_memory()
            subs["decode_c4"] = summarize(measure_decode(args, WORKLOADS["decode_c4"], world, rank, local,
                                                         with_cpu=False))
            free_device_memory()
            subs["step_c2"] = measure_step(args, world, rank, local)
            if world > 1 and KVH % world == 0:
                free_device_memory()
                subs["decode_c5"] = summarize(measure_c5(args, world, rank, local, "kernel"))
            line["sub_results"] = subs
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist

            if dist.is_initialized():
                dist.barrier()
                dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
